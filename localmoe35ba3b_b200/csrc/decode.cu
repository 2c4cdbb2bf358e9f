// One-token MoE decode: the reference's Int8Experts decode branch
// (qwen35_deploy/operators/int8.py:158-187) with the gated HF shared expert
// (modeling_qwen3_5_moe.py:781-790), in two launches on the caller's stream with
// no host synchronisation (so it can be captured in a CUDA graph):
//   1. decode_gate_up_kernel  one warp per (expert, hidden column): the gate and
//      up rows' dot products (W8A8 or W8A16 routed, W8A16 shared), then
//      hidden = round(round(silu(g)) * u) (int8.py:182-184)
//   2. decode_down_kernel     one warp per output column: the down rows of every
//      selected expert, folded as they finish into the ordered combine of
//      _ordered_reduce (int8.py:240-250), then + round(sigmoid(x.gate) * shared),
//      then + residual
// Each block rebuilds the experts' ascending order from the router's ids
// (int8.py:170-179's table, without the ids.cpu() sync and the upload), issues its
// weight rows' loads, and only then (while they are in flight) quantises the
// activation rows it reads for W8A8 (w8a8._quant).  The per-row arithmetic is the
// grouped GEMV's (gemv.cuh), step for step.
#include <algorithm>

#include "common.cuh"
#include "gemv.cuh"

namespace lmoe {

constexpr int kDecodeMaxTop = 32;
constexpr int kDecWarps = 8;
constexpr int kDecBatch = 8;  // down rows whose loads are in flight together
constexpr int kDecMaxGroups = 32;  // K <= 4096
constexpr int kDecScPerLane = 4;   // down: prefetched scales per lane (rows x groups <= 128)

// Warp 0: s_eid[r] = the r-th smallest expert id (ties by slot), s_slot[r] its slot.
// An id outside [0, E) becomes expert 0 (no read leaves the bank) and, when
// `report`, raises LMOE_DEVERR_BAD_EXPERT.
__device__ __forceinline__ void expert_ranks(const int64_t* ids, int top, int64_t E, int64_t* s_eid, int* s_slot,
                                             int* err, bool report) {
  const int lane = lane_id();
  int64_t e = lane < top ? ids[lane] : INT64_MAX;
  if (lane < top && (e < 0 || e >= E)) {
    if (report) raise_error(err, LMOE_DEVERR_BAD_EXPERT);
    e = 0;
  }
  int rank = 0;
  for (int j = 0; j < top; ++j) {
    const int64_t o = __shfl_sync(0xffffffffu, e, j);
    rank += (o < e || (o == e && j < lane)) ? 1 : 0;
  }
  if (lane < top) {
    s_eid[rank] = e;
    if (s_slot) s_slot[rank] = lane;
  }
}

__device__ __forceinline__ float silu_exact(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// Programmatic dependent launch: the down kernel is launched so that it may start
// while the gate_up kernel is still running; it waits (grid_dep_wait) before its first
// read of the gate_up kernel's output, and the gate_up kernel lets it launch once its
// own loads are out (grid_dep_launch).

// rows 0..top-1: the routed experts in ascending id order; row top: the shared
// expert (when sh_qg != nullptr).  hid [rows, I].
template <int DT, bool W8A8, int MAXI>
__global__ void __launch_bounds__(kDecWarps * 32)
    decode_gate_up_kernel(const typename Act<DT>::T* __restrict__ x, const int64_t* __restrict__ ids, int top,
                          int64_t E, const int8_t* __restrict__ qg, const float* __restrict__ sg, int64_t H, int64_t I,
                          const int8_t* __restrict__ sh_qg, const float* __restrict__ sh_sg,
                          const int8_t* __restrict__ sh_qu, const float* __restrict__ sh_su,
                          typename Act<DT>::T* __restrict__ hid, int* err) {
  using A = Act<DT>;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int64_t s_eid[kDecodeMaxTop];
  __shared__ float s_sc[kDecWarps * 2 * kDecMaxGroups];
  const int lane = lane_id(), warp = warp_id();
  const int groups = (int)(H / kGroup);
  int8_t* xq = reinterpret_cast<int8_t*>(smem);                   // [H]
  float* xs = reinterpret_cast<float*>(smem + ((H + 15) & ~15));  // [H / 128]
  // launched so that it may start before the previous kernel ends: the ids, x and the
  // hidden buffer (which the previous call's down kernel reads) all wait for it
  grid_dep_wait();
  if (warp == 0) expert_ranks(ids, top, E, s_eid, nullptr, err, blockIdx.x == 0);
  __syncthreads();
  // the rows' loads go out first; the activation quantisation overlaps them
  const int rows = top + (sh_qg != nullptr ? 1 : 0);
  const int64_t flat = (int64_t)blockIdx.x * kDecWarps + warp;
  const bool live = flat < rows * I;
  const int r = live ? (int)(flat / I) : 0;
  const int64_t c = live ? flat % I : 0;
  const int8_t *gq, *uq;
  const float *gs, *us;
  if (r < top) {
    const int64_t e = s_eid[r];
    gq = qg + (e * 2 * I + c) * H;
    uq = qg + (e * 2 * I + I + c) * H;
    gs = sg + (e * 2 * I + c) * groups;
    us = sg + (e * 2 * I + I + c) * groups;
  } else {
    gq = sh_qg + c * H;
    uq = sh_qu + c * H;
    gs = sh_sg + c * groups;
    us = sh_su + c * groups;
  }
  const int chunks = (int)(H / 16);
  uint4 wg[MAXI], wu[MAXI];  // MAXI = H / 512 chunks per lane: fewer registers, more resident warps
  // the two rows' group scales travel with the weights (lane i < groups: gate scale i,
  // groups <= i < 2 * groups: up scale i - groups), so the dots wait on no second load
  float sc0 = 0.f, sc1 = 0.f;
  if (live) {
    row_load(gq, chunks, lane, wg);
    row_load(uq, chunks, lane, wu);
    if (lane < 2 * groups) sc0 = lane < groups ? gs[lane] : us[lane - groups];
    if (lane + 32 < 2 * groups) sc1 = lane + 32 < groups ? gs[lane + 32] : us[lane + 32 - groups];
  }
  grid_dep_launch();
  if (W8A8)
    for (int g = warp; g < groups; g += kDecWarps) quant_group<DT>(x + g * kGroup, xq + g * kGroup, xs + g, lane);
  float* wsc = s_sc + warp * 2 * kDecMaxGroups;  // [gate groups][up groups]
  if (lane < 2 * groups) wsc[lane] = sc0;
  if (lane + 32 < 2 * groups) wsc[lane + 32] = sc1;
  __syncthreads();
  if (!live) return;
  float g, u;
  if (W8A8 && r < top) {
    g = row_dot_w8a8(wg, wsc, xq, xs, chunks, lane);
    u = row_dot_w8a8(wu, wsc + groups, xq, xs, chunks, lane);
  } else {  // W8A16 routed experts, and the shared expert (Int8Linear arithmetic)
    g = row_dot_w16<DT>(wg, wsc, x, chunks, lane);
    u = row_dot_w16<DT>(wu, wsc + groups, x, chunks, lane);
  }
  if (lane == 0) hid[(int64_t)r * I + c] = A::from_f(__fmul_rn(A::round(silu_exact(A::round(g))), A::round(u)));
}

// out[n] = ordered combine over the routed experts of round(round(v) * w_slot),
// + round(sig * round(v_shared)) with sig = round(sigmoid(round(x . gate))), + residual.
template <int DT, bool W8A8, int MAXI>
__global__ void __launch_bounds__(kDecWarps * 32)
    decode_down_kernel(const typename Act<DT>::T* __restrict__ x, const float* __restrict__ weights,
                       const int64_t* __restrict__ ids, int top, int64_t E, const int8_t* __restrict__ qd,
                       const float* __restrict__ sd, int64_t H, int64_t I, const int8_t* __restrict__ sh_qd,
                       const float* __restrict__ sh_sd, const typename Act<DT>::T* __restrict__ gate_w,
                       const typename Act<DT>::T* __restrict__ residual, const typename Act<DT>::T* __restrict__ hid,
                       typename Act<DT>::T* __restrict__ out, int* err) {
  using A = Act<DT>;
  extern __shared__ __align__(16) uint8_t smem[];
  __shared__ int64_t s_eid[kDecodeMaxTop];
  __shared__ int s_slot[kDecodeMaxTop];
  __shared__ float red[kDecWarps];
  __shared__ float s_sc[kDecWarps * 32 * kDecScPerLane];
  const int lane = lane_id(), warp = warp_id();
  const int gI = (int)(I / kGroup);
  int8_t* hq = reinterpret_cast<int8_t*>(smem);                         // [top, I]
  float* hs = reinterpret_cast<float*>(smem + ((top * I + 15) & ~15));  // [top, I / 128]
  if (warp == 0) expert_ranks(ids, top, E, s_eid, s_slot, err, false);
  __syncthreads();
  // this column's weight rows go out first (the shared row and the first batch of
  // routed rows); the hidden rows' quantisation and the gate's dot product overlap them
  const int64_t n = (int64_t)blockIdx.x * kDecWarps + warp;
  const bool live = n < H;
  const int chunks = (int)(I / 16);
  constexpr int BATCH = MAXI == 1 ? kDecBatch : 2;  // rows in flight together, within the register budget
  const bool with_shared = sh_qd != nullptr;
  const bool gated = with_shared && gate_w != nullptr;
  uint4 wsh[MAXI];
  uint4 w[BATCH][MAXI];
  // every row's group scales travel with the first weights (entry i = row i / gI,
  // group i % gI; the shared row last) into the warp's shared buffer, so the dots
  // wait on no second load; too many to prefetch: the dots read them from memory
  const int nsc = (top + (with_shared ? 1 : 0)) * gI;
  const bool pre = nsc <= 32 * kDecScPerLane;
  float scv[kDecScPerLane];
  if (live) {
    if (with_shared) row_load(sh_qd + n * I, chunks, lane, wsh);
#pragma unroll
    for (int j = 0; j < BATCH; ++j)
      if (j < top) row_load(qd + (s_eid[j] * H + n) * I, chunks, lane, w[j]);
    if (pre) {
#pragma unroll
      for (int k = 0; k < kDecScPerLane; ++k) {
        const int i = lane + 32 * k;
        if (i < nsc) {
          const int r = i / gI, g = i % gI;
          scv[k] = r < top ? sd[(s_eid[r] * H + n) * gI + g] : sh_sd[n * gI + g];
        }
      }
    }
  }
  if (gated) {
    float part = 0.f;
    for (int64_t c = threadIdx.x; c < H; c += kDecWarps * 32) part = fmaf(A::to_f(x[c]), A::to_f(gate_w[c]), part);
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[warp] = part;
  }
  // everything above reads only what existed before the gate_up kernel started; the
  // hidden rows below are its output
  grid_dep_wait();
  grid_dep_launch();  // the next call's gate_up kernel may launch (it waits on this one at its start)
  if (W8A8)
    for (int t = warp; t < top * gI; t += kDecWarps) {
      const int r = t / gI, g = t % gI;
      quant_group<DT>(hid + (int64_t)r * I + g * kGroup, hq + (int64_t)r * I + g * kGroup, hs + r * gI + g, lane);
    }
  float* wsc = s_sc + warp * 32 * kDecScPerLane;
  if (live && pre) {
#pragma unroll
    for (int k = 0; k < kDecScPerLane; ++k)
      if (lane + 32 * k < nsc) wsc[lane + 32 * k] = scv[k];
  }
  __syncthreads();
  if (!live) return;
  float sig = 1.f;
  if (gated) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kDecWarps; ++i) tot += red[i];
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-A::round(tot)))));
  }
  float acc = 0.f;
  for (int r0 = 0; r0 < top; r0 += BATCH) {
    if (r0 > 0) {
#pragma unroll
      for (int j = 0; j < BATCH; ++j)
        if (r0 + j < top) row_load(qd + (s_eid[r0 + j] * H + n) * I, chunks, lane, w[j]);
    }
#pragma unroll
    for (int j = 0; j < BATCH; ++j) {
      const int r = r0 + j;
      if (r >= top) break;
      const float* srow = pre ? wsc + r * gI : sd + (s_eid[r] * H + n) * gI;
      const float v = W8A8 ? row_dot_w8a8(w[j], srow, hq + (int64_t)r * I, hs + r * gI, chunks, lane)
                           : row_dot_w16<DT>(w[j], srow, hid + (int64_t)r * I, chunks, lane);
      acc = A::round(__fadd_rn(acc, A::round(__fmul_rn(A::round(v), weights[s_slot[r]]))));
    }
  }
  if (with_shared) {
    const float s = A::round(row_dot_w16<DT>(wsh, pre ? wsc + top * gI : sh_sd + n * gI, hid + (int64_t)top * I,
                                             chunks, lane));
    acc = A::round(__fadd_rn(acc, gated ? A::round(__fmul_rn(sig, s)) : s));
  }
  if (residual != nullptr) acc = A::round(__fadd_rn(A::to_f(residual[n]), acc));
  if (lane == 0) out[n] = A::from_f(acc);
}

struct DecodeWs {
  int64_t off_h, bytes;
  static int64_t align(int64_t v) { return (v + 255) & ~int64_t(255); }
  DecodeWs(int64_t top, int64_t H, int64_t I) {
    (void)H;
    off_h = 0;
    bytes = align((top + 1) * I * 2);  // hidden rows: routed + shared
  }
};

template <int DT, bool W8A8>
static int launch_decode(const void* x, const float* weights, const int64_t* ids, int top, const int8_t* qg,
                         const float* sg, const int8_t* qd, const float* sd, int64_t E, int64_t H, int64_t I,
                         const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                         const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w, const void* residual,
                         void* out, void* hid, int* err, cudaStream_t st) {
  using T = typename Act<DT>::T;
  const int rows = top + (sh_qg != nullptr ? 1 : 0);
  const unsigned b1 = (unsigned)((rows * I + kDecWarps - 1) / kDecWarps);
  const size_t sm1 = (size_t)((H + 15) & ~15) + (size_t)(H / kGroup) * 4;
  if (H <= 2048)
    LMOE_CUDA_CHECK(launch_pdl(decode_gate_up_kernel<DT, W8A8, 4>, dim3(b1), dim3(kDecWarps * 32), sm1, st,
                               (const T*)x, ids, top, E, qg, sg, H, I, sh_qg, sh_sg, sh_qu, sh_su, (T*)hid, err));
  else
    LMOE_CUDA_CHECK(launch_pdl(decode_gate_up_kernel<DT, W8A8, kMaxChunksPerLane>, dim3(b1), dim3(kDecWarps * 32),
                               sm1, st, (const T*)x, ids, top, E, qg, sg, H, I, sh_qg, sh_sg, sh_qu, sh_su, (T*)hid,
                               err));
  LMOE_CUDA_CHECK(cudaGetLastError());
  const unsigned b2 = (unsigned)((H + kDecWarps - 1) / kDecWarps);
  const size_t sm2 = W8A8 ? (size_t)((top * I + 15) & ~15) + (size_t)top * (I / kGroup) * 4 : 16;
  if (sm2 > 227 * 1024) return LMOE_ERR_UNSUPPORTED;
  if (sm2 > 48 * 1024) {
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(decode_down_kernel<DT, W8A8, 1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)sm2));
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(decode_down_kernel<DT, W8A8, kMaxChunksPerLane>,
                                         cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm2));
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(b2);
  cfg.blockDim = dim3(kDecWarps * 32);
  cfg.dynamicSmemBytes = sm2;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (I <= 512)
    LMOE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_down_kernel<DT, W8A8, 1>, (const T*)x, weights, ids, top, E, qd,
                                       sd, H, I, sh_qd, sh_sd, (const T*)sh_gate_w, (const T*)residual,
                                       (const T*)hid, (T*)out, err));
  else
    LMOE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, decode_down_kernel<DT, W8A8, kMaxChunksPerLane>, (const T*)x, weights,
                                       ids, top, E, qd, sd, H, I, sh_qd, sh_sd, (const T*)sh_gate_w,
                                       (const T*)residual, (const T*)hid, (T*)out, err));
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

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
  if (H > 16 * 32 * kMaxChunksPerLane || I > 16 * 32 * kMaxChunksPerLane) return LMOE_ERR_UNSUPPORTED;
  const int t = (int)top;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    return w8a8 ? launch_decode<LMOE_BF16, true>(x, weights, ids, t, qg, sg, qd, sd, E, H, I, sh_qg, sh_sg, sh_qu, sh_su,
                                                 sh_qd, sh_sd, sh_gate_w, residual, out, ws, err, st)
                : launch_decode<LMOE_BF16, false>(x, weights, ids, t, qg, sg, qd, sd, E, H, I, sh_qg, sh_sg, sh_qu,
                                                  sh_su, sh_qd, sh_sd, sh_gate_w, residual, out, ws, err, st);
  return w8a8 ? launch_decode<LMOE_F16, true>(x, weights, ids, t, qg, sg, qd, sd, E, H, I, sh_qg, sh_sg, sh_qu, sh_su,
                                              sh_qd, sh_sd, sh_gate_w, residual, out, ws, err, st)
              : launch_decode<LMOE_F16, false>(x, weights, ids, t, qg, sg, qd, sd, E, H, I, sh_qg, sh_sg, sh_qu, sh_su,
                                               sh_qd, sh_sd, sh_gate_w, residual, out, ws, err, st);
}
