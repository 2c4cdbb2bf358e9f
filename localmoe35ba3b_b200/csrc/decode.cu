// One-token MoE decode: the reference's Int8Experts decode branch
// (qwen35_deploy/operators/int8.py:158-187) with the gated HF shared expert
// (modeling_qwen3_5_moe.py:781-790), as a short chain of launches on the
// caller's stream with no host synchronisation (so it can be captured in a
// CUDA graph):
//   1. decode_table_kernel   ids -> the [top (+2), 5] descriptor table in
//                            ascending expert order (int8.py:170-179), built on
//                            the device instead of after an ids.cpu() sync
//   2. grouped GEMV          gate_up of the routed experts (W8A8 or W8A16) and,
//                            with a shared expert, its gate/up rows (W8A16, the
//                            Int8Linear path)
//   3. silu_rows_kernel      hidden = round(round(silu(g)) * u) (int8.py:182-184)
//   4. grouped GEMV          down of the routed experts and of the shared expert
//   5. reduce_combine_kernel the ordered combine of _ordered_reduce
//                            (int8.py:240-250), then + round(sigmoid(x.gate) *
//                            shared), then + residual
#include <algorithm>

#include "common.cuh"

namespace lmoe {

int lmoe_grouped_launch(bool w8a8, const void* x, const int64_t* table, void* y, int64_t experts, int64_t n,
                        int64_t k, int field, int shared, int dtype, cudaStream_t st);

constexpr int kDecodeMaxTop = 32;

// Table row r (r-th smallest expert id; ties by slot) = (gate_up.q, gate_up.scale,
// down.q, down.scale, slot).  Shared expert rows follow: (gate.q, gate.s, down.q,
// down.s, 0) and (up.q, up.s, 0, 0, 0).  An id outside [0, E) raises
// LMOE_DEVERR_BAD_EXPERT and is replaced by expert 0, so no read leaves the bank.
__global__ void decode_table_kernel(const int64_t* __restrict__ ids, int top, int64_t E, const int8_t* qg,
                                    const float* sg, const int8_t* qd, const float* sd, int64_t H, int64_t I,
                                    const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu,
                                    const float* sh_su, const int8_t* sh_qd, const float* sh_sd,
                                    int64_t* __restrict__ table, int* err) {
  const int lane = threadIdx.x;
  int64_t e = lane < top ? ids[lane] : INT64_MAX;
  if (lane < top && (e < 0 || e >= E)) {
    raise_error(err, LMOE_DEVERR_BAD_EXPERT);
    e = 0;
  }
  int rank = 0;
  for (int j = 0; j < top; ++j) {
    const int64_t o = __shfl_sync(0xffffffffu, e, j);
    rank += (o < e || (o == e && j < lane)) ? 1 : 0;
  }
  if (lane < top) {
    int64_t* row = table + (int64_t)rank * 5;
    row[0] = (int64_t)(qg + e * 2 * I * H);
    row[1] = (int64_t)(sg + e * 2 * I * (H / kGroup));
    row[2] = (int64_t)(qd + e * H * I);
    row[3] = (int64_t)(sd + e * H * (I / kGroup));
    row[4] = lane;
  }
  if (lane == 0 && sh_qg != nullptr) {
    int64_t* row = table + (int64_t)top * 5;
    row[0] = (int64_t)sh_qg;
    row[1] = (int64_t)sh_sg;
    row[2] = (int64_t)sh_qd;
    row[3] = (int64_t)sh_sd;
    row[4] = 0;
    row[5] = (int64_t)sh_qu;
    row[6] = (int64_t)sh_su;
    row[7] = 0;
    row[8] = 0;
    row[9] = 0;
  }
}

__device__ __forceinline__ float silu_exact(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// rows 0..top-1: gate/up halves of the routed gate_up rows [top, 2I];
// row top (when gsh != nullptr): the shared expert's gate and up rows [2, I]
template <int DT>
__global__ void silu_rows_kernel(const typename Act<DT>::T* __restrict__ gu, const typename Act<DT>::T* __restrict__ gsh,
                                 int top, int64_t I, typename Act<DT>::T* __restrict__ h,
                                 typename Act<DT>::T* __restrict__ hsh) {
  using A = Act<DT>;
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  const int rows = top + (gsh != nullptr ? 1 : 0);
  if (idx >= rows * I) return;
  const int64_t r = idx / I, c = idx % I;
  float g, u;
  if (r < top) {
    g = A::to_f(gu[r * 2 * I + c]);
    u = A::to_f(gu[r * 2 * I + I + c]);
  } else {
    g = A::to_f(gsh[c]);
    u = A::to_f(gsh[I + c]);
  }
  const float v = __fmul_rn(A::round(silu_exact(g)), u);
  if (r < top)
    h[r * I + c] = A::from_f(v);
  else
    hsh[c] = A::from_f(v);
}

constexpr int kCombineThreadsDec = 256;

// out[c] = ordered combine of the routed rows (+ gated shared row) (+ residual)
template <int DT>
__global__ void __launch_bounds__(kCombineThreadsDec) reduce_combine_kernel(
    const typename Act<DT>::T* __restrict__ v, const int64_t* __restrict__ table, const float* __restrict__ w, int top,
    int64_t H, const typename Act<DT>::T* __restrict__ vsh, const typename Act<DT>::T* __restrict__ x,
    const typename Act<DT>::T* __restrict__ gate_w, const typename Act<DT>::T* __restrict__ residual,
    typename Act<DT>::T* __restrict__ out) {
  using A = Act<DT>;
  __shared__ float red[kCombineThreadsDec / 32];
  float sig = 1.f;
  if (vsh != nullptr && gate_w != nullptr) {
    float part = 0.f;
    for (int64_t c = threadIdx.x; c < H; c += kCombineThreadsDec) part = fmaf(A::to_f(x[c]), A::to_f(gate_w[c]), part);
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane_id() == 0) red[warp_id()] = part;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kCombineThreadsDec / 32; ++i) tot += red[i];
    const float logit = A::round(tot);
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-logit))));
  }
  const int64_t c = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= H) return;
  float acc = 0.f;
  for (int i = 0; i < top; ++i) {
    const float wt = w[table[i * 5 + 4]];
    acc = A::round(__fadd_rn(acc, A::round(__fmul_rn(A::to_f(v[(int64_t)i * H + c]), wt))));
  }
  if (vsh != nullptr) {
    const float s = A::to_f(vsh[c]);
    acc = A::round(__fadd_rn(acc, gate_w != nullptr ? A::round(__fmul_rn(sig, s)) : s));
  }
  if (residual != nullptr) acc = A::round(__fadd_rn(A::to_f(residual[c]), acc));
  out[c] = A::from_f(acc);
}

struct DecodeWs {
  int64_t off_table, off_gu, off_gsh, off_h, off_hsh, off_v, off_vsh, bytes;
  static int64_t align(int64_t v) { return (v + 255) & ~int64_t(255); }
  DecodeWs(int64_t top, int64_t H, int64_t I) {
    int64_t o = 0;
    off_table = o;  o = align(o + (top + 2) * 5 * 8);
    off_gu = o;     o = align(o + top * 2 * I * 2);
    off_gsh = o;    o = align(o + 2 * I * 2);
    off_h = o;      o = align(o + top * I * 2);
    off_hsh = o;    o = align(o + I * 2);
    off_v = o;      o = align(o + top * H * 2);
    off_vsh = o;    o = align(o + H * 2);
    bytes = o;
  }
};

}  // namespace lmoe

using namespace lmoe;

extern "C" int64_t lmoe_decode_workspace_size(int64_t top, int64_t H, int64_t I) {
  if (top <= 0 || top > kDecodeMaxTop || H <= 0 || I <= 0) return -1;
  return DecodeWs(top, H, I).bytes;
}

extern "C" int lmoe_decode_moe(const void* x, const float* weights, const int64_t* ids, int64_t top, const int8_t* qg,
                               const float* sg, const int8_t* qd, const float* sd, int64_t E, int64_t H, int64_t I,
                               const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                               const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w, const void* residual,
                               void* out, int dtype, int w8a8, void* ws, int* err, void* stream) {
  if (!x || !weights || !ids || !qg || !sg || !qd || !sd || !out || !ws) return LMOE_ERR_INVALID;
  if (top <= 0 || top > kDecodeMaxTop || E <= 0 || H <= 0 || I <= 0 || H % kGroup || I % kGroup) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  const bool with_shared = sh_qg != nullptr;
  if (with_shared && (!sh_sg || !sh_qu || !sh_su || !sh_qd || !sh_sd)) return LMOE_ERR_INVALID;
  const DecodeWs L(top, H, I);
  uint8_t* base = (uint8_t*)ws;
  int64_t* table = (int64_t*)(base + L.off_table);
  void* gu = base + L.off_gu;
  void* gsh = base + L.off_gsh;
  void* h = base + L.off_h;
  void* hsh = base + L.off_hsh;
  void* v = base + L.off_v;
  void* vsh = base + L.off_vsh;
  cudaStream_t st = (cudaStream_t)stream;

  decode_table_kernel<<<1, 32, 0, st>>>(ids, (int)top, E, qg, sg, qd, sd, H, I, sh_qg, sh_sg, sh_qu, sh_su, sh_qd,
                                        sh_sd, table, err);
  LMOE_CUDA_CHECK(cudaGetLastError());
  int rc;
  // gate_up: routed rows share x; the shared expert's gate/up rows use the W8A16 arithmetic
  if ((rc = lmoe_grouped_launch(w8a8 != 0, x, table, gu, top, 2 * I, H, 0, 1, dtype, st))) return rc;
  if (with_shared && (rc = lmoe_grouped_launch(false, x, table + top * 5, gsh, 2, I, H, 0, 1, dtype, st))) return rc;
  const int64_t n_silu = (top + (with_shared ? 1 : 0)) * I;
  const unsigned sb = (unsigned)((n_silu + 255) / 256);
  if (dtype == LMOE_BF16)
    silu_rows_kernel<LMOE_BF16><<<sb, 256, 0, st>>>((const __nv_bfloat16*)gu,
                                                    with_shared ? (const __nv_bfloat16*)gsh : nullptr, (int)top, I,
                                                    (__nv_bfloat16*)h, (__nv_bfloat16*)hsh);
  else
    silu_rows_kernel<LMOE_F16><<<sb, 256, 0, st>>>((const __half*)gu, with_shared ? (const __half*)gsh : nullptr,
                                                   (int)top, I, (__half*)h, (__half*)hsh);
  LMOE_CUDA_CHECK(cudaGetLastError());
  // down: routed row e reads hidden row e; the shared expert reads its own hidden row
  if ((rc = lmoe_grouped_launch(w8a8 != 0, h, table, v, top, H, I, 2, 0, dtype, st))) return rc;
  if (with_shared && (rc = lmoe_grouped_launch(false, hsh, table + top * 5, vsh, 1, H, I, 2, 1, dtype, st))) return rc;
  const unsigned cb = (unsigned)((H + kCombineThreadsDec - 1) / kCombineThreadsDec);
  if (dtype == LMOE_BF16)
    reduce_combine_kernel<LMOE_BF16><<<cb, kCombineThreadsDec, 0, st>>>(
        (const __nv_bfloat16*)v, table, weights, (int)top, H, with_shared ? (const __nv_bfloat16*)vsh : nullptr,
        (const __nv_bfloat16*)x, (const __nv_bfloat16*)sh_gate_w, (const __nv_bfloat16*)residual,
        (__nv_bfloat16*)out);
  else
    reduce_combine_kernel<LMOE_F16><<<cb, kCombineThreadsDec, 0, st>>>(
        (const __half*)v, table, weights, (int)top, H, with_shared ? (const __half*)vsh : nullptr, (const __half*)x,
        (const __half*)sh_gate_w, (const __half*)residual, (__half*)out);
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}
