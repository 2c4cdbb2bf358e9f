// Expert-parallel dispatch rows.
//
// The sender packs one byte row per (token, destination rank):
//   [payload | route ids int32 x top | route weights fp32 x top]
// where the payload is the token's hidden row in the activation dtype (wire
// LMOE_WIRE_DTYPE) or its W8A8 activation quantisation (wire LMOE_WIRE_INT8):
// int8 [hidden] followed by fp32 scales [hidden / 128], the format of the
// reference's w8a8.quantize (operators/w8a8.py:8-22).  The owner unpacks the
// received rows into one activation row per route, dequantising an int8 payload
// to round_dtype(float(q) * s), and feeds them to the routed experts.
//
// Both kernels are one warp per (row, 128-column group): 128 B of int8 or 256 B
// of bf16 per warp, 4 or 8 B per lane, fully coalesced; HBM-bound.
#include "common.cuh"
#include "gemv.cuh"

namespace lmoe {

constexpr int kWireWarps = 8;

__host__ __device__ __forceinline__ int64_t wire_payload(int64_t hidden, bool int8, int64_t itemsize) {
  return int8 ? hidden + 4 * (hidden / kGroup) : itemsize * hidden;
}

template <int DT, bool INT8>
__global__ void __launch_bounds__(32 * kWireWarps)
    ep_pack_kernel(const typename Act<DT>::T* __restrict__ x, int64_t tokens, const int64_t* __restrict__ tok,
                   const int32_t* __restrict__ rid, const float* __restrict__ rw, int64_t rows, int64_t hidden,
                   int top, int64_t row_bytes, uint8_t* __restrict__ out, int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t groups = hidden / kGroup;
  const int64_t task = (int64_t)blockIdx.x * kWireWarps + (threadIdx.x >> 5);
  if (task >= rows * groups) return;
  const int64_t r = task / groups, g = task - r * groups;
  const int64_t pay = wire_payload(hidden, INT8, 2);
  uint8_t* row = out + r * row_bytes;
  const int64_t t = tok[r];
  if (t < 0 || t >= tokens) {
    // a token index outside x: the group is written as zeros and the caller is told
    if (lane == 0) raise_error(err, LMOE_DEVERR_BAD_INDEX);
    if (INT8) {
      *reinterpret_cast<uint32_t*>(row + g * kGroup + lane * 4) = 0u;
      if (lane == 0) *reinterpret_cast<float*>(row + hidden + 4 * g) = 0.f;
    } else {
      *reinterpret_cast<uint2*>(row + g * 2 * kGroup + lane * 8) = make_uint2(0u, 0u);
    }
  } else {
    const typename Act<DT>::T* xg = x + t * hidden + g * kGroup;
    if (INT8)
      quant_group<DT>(xg, reinterpret_cast<int8_t*>(row + g * kGroup),
                      reinterpret_cast<float*>(row + hidden + 4 * g), lane);
    else
      *reinterpret_cast<uint2*>(row + g * 2 * kGroup + lane * 8) = *reinterpret_cast<const uint2*>(xg + lane * 4);
  }
  if (g == 0 && lane < top) {
    reinterpret_cast<int32_t*>(row + pay)[lane] = rid[r * top + lane];
    reinterpret_cast<float*>(row + pay + 4 * top)[lane] = rw[r * top + lane];
  }
}

template <int DT, bool INT8>
__global__ void __launch_bounds__(32 * kWireWarps)
    ep_unpack_kernel(const uint8_t* __restrict__ buf, int64_t rows, const int64_t* __restrict__ row_of,
                     int64_t routes, int64_t hidden, int64_t row_bytes, typename Act<DT>::T* __restrict__ y,
                     int* err) {
  const int lane = threadIdx.x & 31;
  const int64_t groups = hidden / kGroup;
  const int64_t task = (int64_t)blockIdx.x * kWireWarps + (threadIdx.x >> 5);
  if (task >= routes * groups) return;
  const int64_t r = task / groups, g = task - r * groups;
  const int64_t src = row_of ? row_of[r] : r;
  uint2* dst = reinterpret_cast<uint2*>(y + r * hidden + g * kGroup + lane * 4);
  if (src < 0 || src >= rows) {
    if (lane == 0) raise_error(err, LMOE_DEVERR_BAD_INDEX);
    *dst = make_uint2(0u, 0u);
    return;
  }
  const uint8_t* row = buf + src * row_bytes;
  if (INT8) {
    const uint32_t q = *reinterpret_cast<const uint32_t*>(row + g * kGroup + lane * 4);
    const float s = *reinterpret_cast<const float*>(row + hidden + 4 * g);
    float f0, f1, f2, f3;
    i8x4_to_f32(q, f0, f1, f2, f3);
    uint2 o;
    o.x = Act<DT>::pack(__fmul_rn(f0, s), __fmul_rn(f1, s));
    o.y = Act<DT>::pack(__fmul_rn(f2, s), __fmul_rn(f3, s));
    *dst = o;
  } else {
    *dst = *reinterpret_cast<const uint2*>(row + g * 2 * kGroup + lane * 8);
  }
}

static bool wire_geometry(int64_t hidden, int64_t top, int wire, int dtype) {
  return hidden > 0 && hidden % kGroup == 0 && top >= 0 && top <= 32 &&
         (wire == LMOE_WIRE_DTYPE || wire == LMOE_WIRE_INT8) && (dtype == LMOE_BF16 || dtype == LMOE_F16);
}

static bool aligned(const void* p, uintptr_t a) { return ((uintptr_t)p & (a - 1)) == 0; }

}  // namespace lmoe

using namespace lmoe;

extern "C" int64_t lmoe_ep_row_bytes(int64_t hidden, int64_t top, int wire, int dtype) {
  if (!wire_geometry(hidden, top, wire, dtype)) return LMOE_ERR_INVALID;
  return wire_payload(hidden, wire == LMOE_WIRE_INT8, 2) + 8 * top;
}

extern "C" int lmoe_ep_pack_rows(const void* x, int64_t tokens, const int64_t* tok, const int32_t* route_ids,
                                 const float* route_w, int64_t rows, int64_t hidden, int64_t top, int wire,
                                 void* out, int dtype, int* err, void* stream) {
  if (!wire_geometry(hidden, top, wire, dtype) || rows < 0 || tokens < 0) return LMOE_ERR_INVALID;
  if (rows == 0) return LMOE_OK;
  if (!x || !tok || !out || (top > 0 && (!route_ids || !route_w))) return LMOE_ERR_INVALID;
  const bool int8 = wire == LMOE_WIRE_INT8;
  if (!aligned(x, 8) || !aligned(out, int8 ? 4 : 8)) return LMOE_ERR_INVALID;
  const int64_t row_bytes = lmoe_ep_row_bytes(hidden, top, wire, dtype);
  const int64_t blocks = (rows * (hidden / kGroup) + kWireWarps - 1) / kWireWarps;
  if (blocks > 0x7fffffffLL) return LMOE_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)blocks), block(32 * kWireWarps);
  uint8_t* o = (uint8_t*)out;
  const int tp = (int)top;
  if (dtype == LMOE_BF16) {
    const __nv_bfloat16* xp = (const __nv_bfloat16*)x;
    if (int8)
      ep_pack_kernel<LMOE_BF16, true><<<grid, block, 0, st>>>(xp, tokens, tok, route_ids, route_w, rows, hidden, tp,
                                                              row_bytes, o, err);
    else
      ep_pack_kernel<LMOE_BF16, false><<<grid, block, 0, st>>>(xp, tokens, tok, route_ids, route_w, rows, hidden, tp,
                                                               row_bytes, o, err);
  } else {
    const __half* xp = (const __half*)x;
    if (int8)
      ep_pack_kernel<LMOE_F16, true><<<grid, block, 0, st>>>(xp, tokens, tok, route_ids, route_w, rows, hidden, tp,
                                                             row_bytes, o, err);
    else
      ep_pack_kernel<LMOE_F16, false><<<grid, block, 0, st>>>(xp, tokens, tok, route_ids, route_w, rows, hidden, tp,
                                                              row_bytes, o, err);
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

extern "C" int lmoe_ep_unpack_rows(const void* buf, int64_t rows, const int64_t* row_of, int64_t routes,
                                   int64_t hidden, int64_t top, int wire, void* y, int dtype, int* err,
                                   void* stream) {
  if (!wire_geometry(hidden, top, wire, dtype) || rows < 0 || routes < 0) return LMOE_ERR_INVALID;
  if (routes == 0) return LMOE_OK;
  if (!y || (rows > 0 && !buf)) return LMOE_ERR_INVALID;
  const bool int8 = wire == LMOE_WIRE_INT8;
  if (!aligned(y, 8) || !aligned(buf, int8 ? 4 : 8)) return LMOE_ERR_INVALID;
  const int64_t row_bytes = lmoe_ep_row_bytes(hidden, top, wire, dtype);
  const int64_t blocks = (routes * (hidden / kGroup) + kWireWarps - 1) / kWireWarps;
  if (blocks > 0x7fffffffLL) return LMOE_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const dim3 grid((unsigned)blocks), block(32 * kWireWarps);
  const uint8_t* b = (const uint8_t*)buf;
  if (dtype == LMOE_BF16) {
    __nv_bfloat16* yp = (__nv_bfloat16*)y;
    if (int8)
      ep_unpack_kernel<LMOE_BF16, true><<<grid, block, 0, st>>>(b, rows, row_of, routes, hidden, row_bytes, yp, err);
    else
      ep_unpack_kernel<LMOE_BF16, false><<<grid, block, 0, st>>>(b, rows, row_of, routes, hidden, row_bytes, yp, err);
  } else {
    __half* yp = (__half*)y;
    if (int8)
      ep_unpack_kernel<LMOE_F16, true><<<grid, block, 0, st>>>(b, rows, row_of, routes, hidden, row_bytes, yp, err);
    else
      ep_unpack_kernel<LMOE_F16, false><<<grid, block, 0, st>>>(b, rows, row_of, routes, hidden, row_bytes, yp, err);
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}
