// HBM-streaming INT8 group-128 GEMV kernels and the ordered combines.
//
//  * quantize_rows      -- w8a8._quant        (qwen35_deploy/operators/w8a8.py:8-22)
//  * grouped_gemv<W8A8> -- w8a8._linear       (w8a8.py:25-48), table driven
//  * grouped_gemv<W16>  -- int8._grouped_linear (operators/int8.py:213-237)
//  * dense_gemv_w8a16   -- int8._linear for m <= 16 rows (int8.py:9-37)
//  * ordered_reduce     -- int8._ordered_reduce (int8.py:240-250)
//  * routed_reduce      -- prefill._reduce    (runtime/prefill.py:37-49)
//
// One warp owns one weight row (N index): its K bytes stream from HBM with
// 16-byte non-allocating loads, all issued before the first use, so each
// lane keeps K/512 loads in flight.  Group-of-128 sums land in 8-lane
// sub-warps, exact int32 for W8A8, and the per-group rescale runs in group
// order exactly as the reference writes it.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"

namespace lmoe {

template <int DT>
__global__ void quantize_rows_kernel(const typename Act<DT>::T* __restrict__ x, int8_t* __restrict__ q,
                                     float* __restrict__ s, int64_t rows, int64_t k) {
  const int64_t groups = k / kGroup;
  const int64_t task = (int64_t)blockIdx.x * (blockDim.x >> 5) + warp_id();
  if (task >= rows * groups) return;
  const int64_t row = task / groups, g = task % groups;
  quant_group<DT>(x + row * k + g * kGroup, q + row * k + g * kGroup, s + row * groups + g, lane_id());
}

// ----------------------------------------------------------------------------
// Table-driven grouped GEMV.  Block: 8 warps; dynamic smem holds the quantised
// (W8A8) or raw (W8A16) activation rows this block needs.
constexpr int kGemvWarps = 8;

template <int DT, bool W8A8>
__global__ void __launch_bounds__(kGemvWarps * 32) grouped_gemv_kernel(
    const typename Act<DT>::T* __restrict__ x, const int64_t* __restrict__ table, typename Act<DT>::T* __restrict__ y,
    int64_t experts, int64_t n, int64_t k, int field, int shared, int8_t* __restrict__ xq_out,
    float* __restrict__ xs_out) {
  extern __shared__ __align__(16) uint8_t smem[];
  // launched as a programmatic dependent: x and the descriptor table may be the previous
  // kernel's output, so nothing is read before it completes; the next kernel may launch at
  // once (it waits for this one before reading y)
  grid_dep_launch();
  grid_dep_wait();
  const int groups = (int)(k / kGroup);
  const int64_t row0 = (int64_t)blockIdx.x * kGemvWarps;  // flat (expert, n) row of warp 0
  const int lane = lane_id(), warp = warp_id();
  // x rows needed by this block: shared -> row 0 only; else rows e_first..e_last
  const int64_t e_first = row0 / n;
  const int64_t e_hi = (row0 + kGemvWarps - 1) / n;
  const int64_t e_last = e_hi < experts - 1 ? e_hi : experts - 1;
  const int nx = shared ? 1 : (int)(e_last - e_first + 1);
  const int64_t xrow0 = shared ? 0 : e_first;

  int8_t* sq = reinterpret_cast<int8_t*>(smem);                     // [nx, k] int8
  float* ss = reinterpret_cast<float*>(smem + ((nx * k + 15) & ~15));  // [nx, groups]
  if constexpr (W8A8) {
    for (int t = warp; t < nx * groups; t += kGemvWarps) {
      const int r = t / groups, g = t % groups;
      const int64_t xr = xrow0 + r;
      quant_group<DT>(x + xr * k + (int64_t)g * kGroup, sq + (int64_t)r * k + g * kGroup, ss + r * groups + g, lane);
    }
    __syncthreads();
    if (xq_out != nullptr) {
      // optional copy-out of the quantised rows: the block holding a row's
      // first output (flat row xr * n, or block 0 when shared) publishes it
      for (int r = 0; r < nx; ++r) {
        const int64_t xr = xrow0 + r;
        const bool owner = shared ? (blockIdx.x == 0) : ((xr * n) / kGemvWarps == (int64_t)blockIdx.x);
        if (!owner) continue;
        for (int64_t i = threadIdx.x; i < k; i += blockDim.x) xq_out[xr * k + i] = sq[(int64_t)r * k + i];
        for (int i = threadIdx.x; i < groups; i += blockDim.x) xs_out[xr * groups + i] = ss[r * groups + i];
      }
    }
  }

  const int64_t flat = row0 + warp;
  if (flat >= experts * n) return;
  const int64_t e = flat / n, nn = flat % n;
  const int8_t* Q = reinterpret_cast<const int8_t*>(table[e * 5 + field]);
  const float* S = reinterpret_cast<const float*>(table[e * 5 + field + 1]);
  const int xr = shared ? 0 : (int)(e - e_first);
  const int8_t* wrow = Q + nn * k;
  const float* srow = S + nn * groups;

  const int chunks = (int)(k / 16);
  uint4 w[kMaxChunksPerLane];
  row_load(wrow, chunks, lane, w);
  float acc;
  if constexpr (W8A8)
    acc = row_dot_w8a8(w, srow, sq + (int64_t)xr * k, ss + xr * groups, chunks, lane);
  else
    acc = row_dot_w16<DT>(w, srow, x + (shared ? 0 : e) * k, chunks, lane);
  if (lane == 0) y[e * n + nn] = Act<DT>::from_f(acc);
}

// ----------------------------------------------------------------------------
// Dense W8A16 GEMV for m <= kDenseMaxM rows: one warp per weight row, the
// dequantised weights are reused for all m activation rows.  Launched as a
// programmatic dependent: the weight rows do not depend on the previous kernel, so
// each warp requests its first chunks before waiting for it; the m activation rows
// (which may be that kernel's output) are read after the wait with ordinary loads,
// never through the read-only path.  The next kernel may launch at once: it waits for
// this one before reading y.
constexpr int kDenseMaxM = 16;

template <int DT, int MM>
__global__ void __launch_bounds__(kGemvWarps * 32) dense_gemv_w8a16_kernel(
    const typename Act<DT>::T* __restrict__ x, const int8_t* __restrict__ q, const float* __restrict__ scale,
    typename Act<DT>::T* __restrict__ y, int m, int64_t n, int64_t k) {
  using T = typename Act<DT>::T;
  const int lane = lane_id();
  const int64_t nn = (int64_t)blockIdx.x * kGemvWarps + warp_id();
  const bool live = nn < n;
  const int groups = (int)(k / kGroup);
  const int chunks = (int)(k / 16);
  const int8_t* wrow = q + (live ? nn : 0) * k;
  const float* srow = scale + (live ? nn : 0) * groups;
  grid_dep_launch();
  uint4 w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int c = lane + 32 * i;
    if (live && c < chunks) w[i] = ldg_stream(wrow + c * 16);
  }
  grid_dep_wait();
  if (!live) return;
  float acc[MM];
#pragma unroll
  for (int r = 0; r < MM; ++r) acc[r] = 0.f;
  for (int c0 = 0; c0 < chunks; c0 += 32 * 4) {
    if (c0 > 0) {
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int c = c0 + lane + 32 * i;
        if (c < chunks) w[i] = ldg_stream(wrow + c * 16);
      }
    }
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int c = c0 + lane + 32 * i;
      if (c >= chunks) continue;
      const float sc = __ldg(srow + (c >> 3));
      float wf[16];
      const uint32_t wv[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        float f0, f1, f2, f3;
        i8x4_to_f32(wv[j], f0, f1, f2, f3);
        wf[4 * j] = Act<DT>::round(__fmul_rn(f0, sc));
        wf[4 * j + 1] = Act<DT>::round(__fmul_rn(f1, sc));
        wf[4 * j + 2] = Act<DT>::round(__fmul_rn(f2, sc));
        wf[4 * j + 3] = Act<DT>::round(__fmul_rn(f3, sc));
      }
#pragma unroll
      for (int r = 0; r < MM; ++r) {
        if (r >= m) break;
        const uint4* xv = reinterpret_cast<const uint4*>(x + (int64_t)r * k + c * 16);
        const uint4 xa = xv[0], xb = xv[1];
        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          acc[r] = fmaf(Act<DT>::lo_f(xw[j]), wf[2 * j], acc[r]);
          acc[r] = fmaf(Act<DT>::hi_f(xw[j]), wf[2 * j + 1], acc[r]);
        }
      }
    }
  }
#pragma unroll
  for (int r = 0; r < MM; ++r) {
    if (r >= m) break;
    float a = acc[r];
#pragma unroll
    for (int o = 16; o; o >>= 1) a += __shfl_xor_sync(0xffffffffu, a, o);
    if (lane == 0) y[(int64_t)r * n + nn] = Act<DT>::from_f(a);
  }
}

// ----------------------------------------------------------------------------
template <int DT>
__global__ void ordered_reduce_kernel(const typename Act<DT>::T* __restrict__ v, const int64_t* __restrict__ table,
                                      const float* __restrict__ w, typename Act<DT>::T* __restrict__ y, int64_t n,
                                      int64_t experts) {
  const int64_t col = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (col >= n) return;
  float acc = 0.f;
  for (int64_t e = 0; e < experts; ++e) {
    const float wt = w[table[e * 5 + 4]];
    const float val = Act<DT>::round(__fmul_rn(Act<DT>::to_f(v[e * n + col]), wt));
    acc = Act<DT>::round(__fadd_rn(acc, val));
  }
  y[col] = Act<DT>::from_f(acc);
}

// prefill._reduce: 8 columns per thread, 16-byte vectors (n % 8 == 0) or scalar tail
template <int DT>
__global__ void routed_reduce_kernel(const typename Act<DT>::T* __restrict__ down, const int64_t* __restrict__ ordered,
                                     const int64_t* __restrict__ slots, const float* __restrict__ w,
                                     typename Act<DT>::T* __restrict__ y, int64_t n, int top) {
  const int64_t t = blockIdx.y;
  const int64_t col = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 8;
  if (col >= n) return;
  float acc[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
  for (int i = 0; i < top; ++i) {
    const int64_t route = ordered[t * top + i];
    const float wt = w[t * top + slots[t * top + i]];
    const typename Act<DT>::T* src = down + route * n + col;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      if (col + j < n) {
        const float val = Act<DT>::round(__fmul_rn(Act<DT>::to_f(src[j]), wt));
        acc[j] = Act<DT>::round(__fadd_rn(acc[j], val));
      }
    }
  }
#pragma unroll
  for (int j = 0; j < 8; ++j)
    if (col + j < n) y[t * n + col + j] = Act<DT>::from_f(acc[j]);
}

}  // namespace lmoe

using namespace lmoe;

// ============================================================================ C ABI
extern "C" int lmoe_abi_version(void) { return 3; }

extern "C" int lmoe_quantize_rows(const void* x, int8_t* q, float* s, int64_t rows, int64_t k, int dtype,
                                  void* stream) {
  if (!x || !q || !s || rows < 0 || k <= 0 || k % kGroup) return LMOE_ERR_INVALID;
  if (rows == 0) return LMOE_OK;
  const int64_t tasks = rows * (k / kGroup);
  const dim3 grid((unsigned)((tasks + 7) / 8));
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    quantize_rows_kernel<LMOE_BF16><<<grid, 256, 0, st>>>((const __nv_bfloat16*)x, q, s, rows, k);
  else if (dtype == LMOE_F16)
    quantize_rows_kernel<LMOE_F16><<<grid, 256, 0, st>>>((const __half*)x, q, s, rows, k);
  else
    return LMOE_ERR_INVALID;
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

template <bool W8A8>
static int launch_grouped(const void* x, const int64_t* table, void* y, int64_t experts, int64_t n, int64_t k,
                          int field, int shared, int dtype, int8_t* xq, float* xs, void* stream) {
  if (!x || !table || !y || experts < 0 || n <= 0 || k <= 0 || k % kGroup || k > 16 * 32 * kMaxChunksPerLane)
    return LMOE_ERR_INVALID;
  if (field != 0 && field != 2) return LMOE_ERR_INVALID;
  if (experts == 0) return LMOE_OK;
  const int64_t rows = experts * n;
  const unsigned blocks = (unsigned)((rows + kGemvWarps - 1) / kGemvWarps);
  // worst case x rows per block: shared -> 1, else up to kGemvWarps distinct experts
  const int nx = shared ? 1 : (int)std::min<int64_t>(experts, kGemvWarps / std::max<int64_t>(1, n) + 2);
  size_t smem = 0;
  if (W8A8) smem = ((size_t)nx * k + 15) / 16 * 16 + (size_t)nx * (k / kGroup) * 4;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16) {
    auto kern = grouped_gemv_kernel<LMOE_BF16, W8A8>;
    if (smem > 48 * 1024) LMOE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(launch_pdl(kern, dim3(blocks), dim3(kGemvWarps * 32), smem, st, (const __nv_bfloat16*)x, table,
                               (__nv_bfloat16*)y, experts, n, k, field, shared, xq, xs));
  } else if (dtype == LMOE_F16) {
    auto kern = grouped_gemv_kernel<LMOE_F16, W8A8>;
    if (smem > 48 * 1024) LMOE_CUDA_CHECK(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(launch_pdl(kern, dim3(blocks), dim3(kGemvWarps * 32), smem, st, (const __half*)x, table,
                               (__half*)y, experts, n, k, field, shared, xq, xs));
  } else {
    return LMOE_ERR_INVALID;
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

namespace lmoe {
// in-library launcher for the table-driven grouped GEMV (used by the decode chain)
int lmoe_grouped_launch(bool w8a8, const void* x, const int64_t* table, void* y, int64_t experts, int64_t n,
                        int64_t k, int field, int shared, int dtype, cudaStream_t st) {
  return w8a8 ? launch_grouped<true>(x, table, y, experts, n, k, field, shared, dtype, nullptr, nullptr, st)
              : launch_grouped<false>(x, table, y, experts, n, k, field, shared, dtype, nullptr, nullptr, st);
}
}  // namespace lmoe

extern "C" int lmoe_grouped_linear_w8a16(const void* x, const int64_t* table, void* y, int64_t experts, int64_t n,
                                         int64_t k, int field, int shared, int dtype, void* stream) {
  return launch_grouped<false>(x, table, y, experts, n, k, field, shared, dtype, nullptr, nullptr, stream);
}

extern "C" int lmoe_grouped_linear_w8a8(const void* x, const int64_t* table, void* y, int64_t experts, int64_t n,
                                        int64_t k, int field, int shared, int dtype, int8_t* xq, float* xs,
                                        void* stream) {
  return launch_grouped<true>(x, table, y, experts, n, k, field, shared, dtype, xq, xs, stream);
}

// dense GEMV path of lmoe_linear_w8a16 (m <= kDenseMaxM); the tensor-core path lives in grouped_gemm.cu
int lmoe_dense_gemv_w8a16(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                          int64_t k, int dtype, cudaStream_t st) {
  if (m <= 0 || m > kDenseMaxM) return LMOE_ERR_INVALID;
  const size_t smem = 0;
  if ((uintptr_t)x & 15) return LMOE_ERR_INVALID;
  const unsigned blocks = (unsigned)((n + kGemvWarps - 1) / kGemvWarps);
#define LMOE_DENSE_CASE(MM)                                                                                      \
  if (dtype == LMOE_BF16) {                                                                                      \
    auto kern = dense_gemv_w8a16_kernel<LMOE_BF16, MM>;                                                          \
    LMOE_CUDA_CHECK(launch_pdl(kern, dim3(blocks), dim3(kGemvWarps * 32), smem, st, (const __nv_bfloat16*)x, q,  \
                               scale, (__nv_bfloat16*)y, (int)m, n, k));                                         \
  } else {                                                                                                       \
    auto kern = dense_gemv_w8a16_kernel<LMOE_F16, MM>;                                                           \
    LMOE_CUDA_CHECK(launch_pdl(kern, dim3(blocks), dim3(kGemvWarps * 32), smem, st, (const __half*)x, q, scale,  \
                               (__half*)y, (int)m, n, k));                                                       \
  }
  if (m == 1) {
    LMOE_DENSE_CASE(1)
  } else if (m <= 4) {
    LMOE_DENSE_CASE(4)
  } else if (m <= 8) {
    LMOE_DENSE_CASE(8)
  } else {
    LMOE_DENSE_CASE(16)
  }
#undef LMOE_DENSE_CASE
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

extern "C" int lmoe_ordered_reduce(const void* values, const int64_t* table, const float* weights, void* y, int64_t n,
                                   int64_t experts, int dtype, void* stream) {
  if (!values || !table || !weights || !y || n <= 0 || experts < 0) return LMOE_ERR_INVALID;
  const unsigned blocks = (unsigned)((n + 255) / 256);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    ordered_reduce_kernel<LMOE_BF16><<<blocks, 256, 0, st>>>((const __nv_bfloat16*)values, table, weights,
                                                             (__nv_bfloat16*)y, n, experts);
  else if (dtype == LMOE_F16)
    ordered_reduce_kernel<LMOE_F16><<<blocks, 256, 0, st>>>((const __half*)values, table, weights, (__half*)y, n,
                                                            experts);
  else
    return LMOE_ERR_INVALID;
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

extern "C" int lmoe_routed_reduce(const void* down, const int64_t* ordered, const int64_t* slots, const float* weights,
                                  void* y, int64_t tokens, int64_t n, int64_t top, int dtype, void* stream) {
  if (!down || !ordered || !slots || !weights || !y || tokens < 0 || n <= 0 || top <= 0) return LMOE_ERR_INVALID;
  if (tokens == 0) return LMOE_OK;
  if (tokens > 65535) return LMOE_ERR_UNSUPPORTED;
  const dim3 grid((unsigned)(((n + 7) / 8 + 127) / 128), (unsigned)tokens);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    routed_reduce_kernel<LMOE_BF16><<<grid, 128, 0, st>>>((const __nv_bfloat16*)down, ordered, slots, weights,
                                                          (__nv_bfloat16*)y, n, (int)top);
  else if (dtype == LMOE_F16)
    routed_reduce_kernel<LMOE_F16><<<grid, 128, 0, st>>>((const __half*)down, ordered, slots, weights, (__half*)y, n,
                                                         (int)top);
  else
    return LMOE_ERR_INVALID;
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}
