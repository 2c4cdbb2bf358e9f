// One-token MoE decode: the reference's Int8Experts decode branch
// (qwen35_deploy/operators/int8.py:158-187) with the gated HF shared expert
// (modeling_qwen3_5_moe.py:781-790), in two launches on the caller's stream with
// no host synchronisation (so it can be captured in a CUDA graph):
//   1. decode_gu_kernel  one CTA per (selected expert, block of CB hidden columns):
//      the block's gate rows and up rows (contiguous in the bank) and their
//      group scales arrive in shared memory by a few bulk copies issued at once,
//      then one warp per column computes both dot products (W8A8 or W8A16 routed,
//      W8A16 shared) and hidden = round(round(silu(g)) * u) (int8.py:182-184)
//   2. decode_dn_kernel  one CTA per block of CBd output columns: the down rows
//      of every selected expert and of the shared expert for those columns
//      arrive the same way -- issued before the kernel waits for kernel 1, so
//      they stream while kernel 1 computes -- then one warp per column computes
//      the down dots, folding them in ascending expert order into the ordered
//      combine of _ordered_reduce (int8.py:240-250), then
//      + round(sigmoid(round(x . gate)) * shared), then + residual.
// The weight bytes of a whole layer are requested at the kernels' start, so HBM
// streams them at full rate instead of one row per warp per round trip.  Each
// row's K is split over the 32 lanes of its warp (16 bytes per lane per chunk);
// the group partial sums are added in group order, as the reference's loop over
// groups does (w8a8.py:37-40).  Each CTA rebuilds the experts' ascending order
// from the router's ids (int8.py:170-179's table, without the ids.cpu() sync and
// the upload).  The per-row arithmetic is the grouped GEMV's (gemv.cuh).
#include "common.cuh"
#include "gemv.cuh"

namespace lmoe {

constexpr int kDecodeMaxTop = 32;
constexpr int kDecThreads = 512;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecGuSmemMax = 140 * 1024;  // kernel 1's shared memory, so a kernel-2 CTA fits beside it
constexpr int kDecDnSmemMax = 84 * 1024;

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

// every lane waits (bounded) for the barrier's first phase; false after a timeout
__device__ __forceinline__ bool dec_wait(uint32_t bar, int* err) { return mbar_wait_drain(bar, 0, err); }

// one weight row of `chunks` 16-byte chunks from shared memory: chunk lane + 32 i -> w[i]
template <int MAXI>
__device__ __forceinline__ void row_lds(uint32_t srow, int chunks, int lane, uint4 (&w)[MAXI]) {
#pragma unroll
  for (int i = 0; i < MAXI; ++i)
    if (lane + 32 * i < chunks) w[i] = lds128(srow + (uint32_t)(lane + 32 * i) * 16u);
}

struct GuSmem {
  int64_t wg, wu, sg, su, xq, xs, bars, bytes;
  __host__ __device__ GuSmem(int64_t CB, int64_t H) {
    const int64_t GH = H / kGroup;
    wg = 0;
    wu = CB * H;
    sg = 2 * CB * H;
    su = sg + CB * GH * 4;
    xq = su + CB * GH * 4;
    xs = xq + H;
    bars = (xs + GH * 4 + 15) & ~int64_t(15);
    bytes = bars + (CB / 8) * 8;
  }
};

// rows 0..top-1: the routed experts in ascending id order; row top: the shared
// expert (when sh_qg != nullptr).  hid [rows, I].  Grid: rows x (I / CB) CTAs.
template <int DT, bool W8A8, int MAXI>
__global__ void __launch_bounds__(kDecThreads) decode_gu_kernel(
    const typename Act<DT>::T* __restrict__ x, const int64_t* __restrict__ ids, int top, int64_t E,
    const int8_t* __restrict__ qg, const float* __restrict__ sg, int64_t H, int64_t I, const int8_t* __restrict__ sh_qg,
    const float* __restrict__ sh_sg, const int8_t* __restrict__ sh_qu, const float* __restrict__ sh_su, int CB,
    typename Act<DT>::T* __restrict__ hid, int* err) {
  using A = Act<DT>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t s_eid[kDecodeMaxTop];
  const int lane = lane_id(), warp = warp_id();
  const int GH = (int)(H / kGroup);
  const GuSmem L(CB, H);
  const uint32_t sb = smem_u32(smem);
  const int npieces = CB / 8;
  if (threadIdx.x == 0) {
    for (int p = 0; p < npieces; ++p) mbar_init(sb + (uint32_t)L.bars + 8u * p, 1);
    fence_mbar_init();
  }
  // launched so that it may start before the previous kernel ends: the ids, x and the
  // hidden buffer (which the previous call's down kernel reads) all wait for it
  grid_dep_wait();
  if (warp == 0) expert_ranks(ids, top, E, s_eid, nullptr, err, blockIdx.x == 0);
  __syncthreads();
  const int nblk = (int)(I / CB);
  const int r = blockIdx.x / nblk;
  const int64_t c0 = (int64_t)(blockIdx.x % nblk) * CB;
  if (threadIdx.x == 0) {
    const int8_t *gq, *uq;
    const float *gs, *us;
    if (r < top) {
      const int64_t e = s_eid[r];
      gq = qg + (e * 2 * I + c0) * H;
      uq = qg + (e * 2 * I + I + c0) * H;
      gs = sg + (e * 2 * I + c0) * GH;
      us = sg + (e * 2 * I + I + c0) * GH;
    } else {
      gq = sh_qg + c0 * H;
      uq = sh_qu + c0 * H;
      gs = sh_sg + c0 * GH;
      us = sh_su + c0 * GH;
    }
    // pieces of 8 columns, each on its own barrier, so warps start as their rows land
    const uint32_t wbytes = (uint32_t)(8 * H), sbytes = (uint32_t)(8 * GH * 4);
    for (int p = 0; p < npieces; ++p) {
      const uint32_t bar = sb + (uint32_t)L.bars + 8u * p;
      mbar_arrive_expect_tx(bar, 2 * (wbytes + sbytes));
      bulk_g2s(sb + (uint32_t)(L.wg + p * 8 * H), gq + p * 8 * H, wbytes, bar);
      bulk_g2s(sb + (uint32_t)(L.wu + p * 8 * H), uq + p * 8 * H, wbytes, bar);
      bulk_g2s(sb + (uint32_t)(L.sg + p * 8 * GH * 4), gs + p * 8 * GH, sbytes, bar);
      bulk_g2s(sb + (uint32_t)(L.su + p * 8 * GH * 4), us + p * 8 * GH, sbytes, bar);
    }
  }
  grid_dep_launch();  // the down kernel may start and stream its own rows beside this one
  int8_t* xq = reinterpret_cast<int8_t*>(smem + L.xq);
  float* xs = reinterpret_cast<float*>(smem + L.xs);
  if (W8A8 && r < top)
    for (int g = warp; g < GH; g += kDecWarps) quant_group<DT>(x + g * kGroup, xq + g * kGroup, xs + g, lane);
  __syncthreads();
  const int chunks = (int)(H / 16);
  for (int j = warp; j < CB; j += kDecWarps) {
    if (!dec_wait(sb + (uint32_t)L.bars + 8u * (j / 8), err)) return;
    uint4 wg[MAXI], wu[MAXI];
    row_lds(sb + (uint32_t)(L.wg + j * H), chunks, lane, wg);
    row_lds(sb + (uint32_t)(L.wu + j * H), chunks, lane, wu);
    const float* gsr = reinterpret_cast<const float*>(smem + L.sg) + j * GH;
    const float* usr = reinterpret_cast<const float*>(smem + L.su) + j * GH;
    float g, u;
    if (W8A8 && r < top) {
      g = row_dot_w8a8(wg, gsr, xq, xs, chunks, lane);
      u = row_dot_w8a8(wu, usr, xq, xs, chunks, lane);
    } else {  // W8A16 routed experts, and the shared expert (Int8Linear arithmetic)
      g = row_dot_w16<DT>(wg, gsr, x, chunks, lane);
      u = row_dot_w16<DT>(wu, usr, x, chunks, lane);
    }
    if (lane == 0) hid[(int64_t)r * I + c0 + j] = A::from_f(__fmul_rn(A::round(silu_exact(A::round(g))), A::round(u)));
  }
}

struct DnSmem {
  int64_t w, sc, hq, hs, bar, bytes;
  __host__ __device__ DnSmem(int64_t rows, int64_t top, int64_t CBd, int64_t I) {
    const int64_t GI = I / kGroup;
    w = 0;
    sc = rows * CBd * I;
    hq = sc + rows * CBd * GI * 4;
    hs = hq + top * I;
    bar = (hs + top * GI * 4 + 15) & ~int64_t(15);
    bytes = bar + 8;
  }
};

// out[n] = ordered combine over the routed experts of round(round(v) * w_slot),
// + round(sig * round(v_shared)) with sig = round(sigmoid(round(x . gate))), + residual.
// Grid: H / CBd CTAs.
template <int DT, bool W8A8, int MAXI>
__global__ void __launch_bounds__(kDecThreads) decode_dn_kernel(
    const typename Act<DT>::T* __restrict__ x, const float* __restrict__ weights, const int64_t* __restrict__ ids,
    int top, int64_t E, const int8_t* __restrict__ qd, const float* __restrict__ sd, int64_t H, int64_t I,
    const int8_t* __restrict__ sh_qd, const float* __restrict__ sh_sd, const typename Act<DT>::T* __restrict__ gate_w,
    const typename Act<DT>::T* __restrict__ residual, const typename Act<DT>::T* __restrict__ hid, int CBd,
    typename Act<DT>::T* __restrict__ out, int* err) {
  using A = Act<DT>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t s_eid[kDecodeMaxTop];
  __shared__ int s_slot[kDecodeMaxTop];
  __shared__ float red[kDecWarps];
  const int lane = lane_id(), warp = warp_id();
  const int GI = (int)(I / kGroup);
  const bool with_shared = sh_qd != nullptr;
  const bool gated = with_shared && gate_w != nullptr;
  const int rows = top + (with_shared ? 1 : 0);
  const DnSmem L(rows, top, CBd, I);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar = sb + (uint32_t)L.bar;
  const int64_t n0 = (int64_t)blockIdx.x * CBd;
  if (threadIdx.x == 0) {
    mbar_init(bar, 1);
    fence_mbar_init();
  }
  // the ids were written before the gate_up kernel started (it waited for them before
  // letting this kernel launch): this kernel's weight rows go out before it waits
  if (warp == 0) expert_ranks(ids, top, E, s_eid, s_slot, err, false);
  __syncthreads();
  if (threadIdx.x == 0) {
    const uint32_t wb = (uint32_t)(CBd * I), sbt = (uint32_t)(CBd * GI * 4);
    mbar_arrive_expect_tx(bar, (uint32_t)rows * (wb + sbt));
    for (int rr = 0; rr < rows; ++rr) {
      const int8_t* q = rr < top ? qd + (s_eid[rr] * H + n0) * I : sh_qd + n0 * I;
      const float* s = rr < top ? sd + (s_eid[rr] * H + n0) * GI : sh_sd + n0 * GI;
      bulk_g2s(sb + (uint32_t)(L.w + (int64_t)rr * CBd * I), q, wb, bar);
      bulk_g2s(sb + (uint32_t)(L.sc + (int64_t)rr * CBd * GI * 4), s, sbt, bar);
    }
  }
  if (gated) {
    float part = 0.f;
    for (int64_t c = threadIdx.x; c < H; c += kDecThreads) part = fmaf(A::to_f(x[c]), A::to_f(gate_w[c]), part);
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[warp] = part;
  }
  // everything above reads only what existed before the gate_up kernel started; the
  // hidden rows below are its output
  grid_dep_wait();
  grid_dep_launch();  // the next call's gate_up kernel may launch (it waits on this one at its start)
  int8_t* hq = reinterpret_cast<int8_t*>(smem + L.hq);
  float* hs = reinterpret_cast<float*>(smem + L.hs);
  if (W8A8)
    for (int t = warp; t < top * GI; t += kDecWarps) {
      const int rr = t / GI, g = t % GI;
      quant_group<DT>(hid + (int64_t)rr * I + g * kGroup, hq + (int64_t)rr * I + g * kGroup, hs + rr * GI + g, lane);
    }
  __syncthreads();
  float sig = 1.f;
  if (gated) {
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < kDecWarps; ++i) tot += red[i];
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-A::round(tot)))));
  }
  if (!dec_wait(bar, err)) return;
  const int chunks = (int)(I / 16);
  const float* scs = reinterpret_cast<const float*>(smem + L.sc);
  for (int j = warp; j < CBd; j += kDecWarps) {
    const int64_t n = n0 + j;
    float acc = 0.f;
    for (int rr = 0; rr < top; ++rr) {
      uint4 w[MAXI];
      row_lds(sb + (uint32_t)(L.w + ((int64_t)rr * CBd + j) * I), chunks, lane, w);
      const float* srow = scs + ((int64_t)rr * CBd + j) * GI;
      const float v = W8A8 ? row_dot_w8a8(w, srow, hq + (int64_t)rr * I, hs + rr * GI, chunks, lane)
                           : row_dot_w16<DT>(w, srow, hid + (int64_t)rr * I, chunks, lane);
      acc = A::round(__fadd_rn(acc, A::round(__fmul_rn(A::round(v), weights[s_slot[rr]]))));
    }
    if (with_shared) {
      uint4 w[MAXI];
      row_lds(sb + (uint32_t)(L.w + ((int64_t)top * CBd + j) * I), chunks, lane, w);
      const float s =
          A::round(row_dot_w16<DT>(w, scs + ((int64_t)top * CBd + j) * GI, hid + (int64_t)top * I, chunks, lane));
      acc = A::round(__fadd_rn(acc, gated ? A::round(__fmul_rn(sig, s)) : s));
    }
    if (residual != nullptr) acc = A::round(__fadd_rn(A::to_f(residual[n]), acc));
    if (lane == 0) out[n] = A::from_f(acc);
  }
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

// columns per CTA: the largest block whose rows fit the kernel's shared-memory budget
static int pick_cb(int64_t H, int64_t I) {
  for (int cb = 32; cb >= 8; cb >>= 1)
    if (I % cb == 0 && GuSmem(cb, H).bytes <= kDecGuSmemMax) return cb;
  return 0;
}
static int pick_cbd(int64_t rows, int64_t top, int64_t H, int64_t I) {
  for (int cb = 16; cb >= 4; cb >>= 1)
    if (H % cb == 0 && DnSmem(rows, top, cb, I).bytes <= kDecDnSmemMax) return cb;
  return 0;
}

template <typename K>
static int set_smem(K kernel, int64_t bytes) {
  LMOE_CUDA_CHECK(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return LMOE_OK;
}

template <int DT, bool W8A8, int MAXG, int MAXD>
static int launch_decode_t(const void* x, const float* weights, const int64_t* ids, int top, const int8_t* qg,
                           const float* sg, const int8_t* qd, const float* sd, int64_t E, int64_t H, int64_t I,
                           const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                           const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w, const void* residual,
                           void* out, void* hid, int* err, int cb, int cbd, cudaStream_t st) {
  using T = typename Act<DT>::T;
  const int rows = top + (sh_qg != nullptr ? 1 : 0);
  const int64_t sm1 = GuSmem(cb, H).bytes, sm2 = DnSmem(rows, top, cbd, I).bytes;
  auto k1 = decode_gu_kernel<DT, W8A8, MAXG>;
  auto k2 = decode_dn_kernel<DT, W8A8, MAXD>;
  int rc = set_smem(k1, sm1);
  if (rc || (rc = set_smem(k2, sm2))) return rc;
  LMOE_CUDA_CHECK(launch_pdl(k1, dim3((unsigned)(rows * (I / cb))), dim3(kDecThreads), (size_t)sm1, st, (const T*)x,
                             ids, top, E, qg, sg, H, I, sh_qg, sh_sg, sh_qu, sh_su, cb, (T*)hid, err));
  LMOE_CUDA_CHECK(launch_pdl(k2, dim3((unsigned)(H / cbd)), dim3(kDecThreads), (size_t)sm2, st, (const T*)x, weights,
                             ids, top, E, qd, sd, H, I, sh_qd, sh_sd, (const T*)sh_gate_w, (const T*)residual,
                             (const T*)hid, cbd, (T*)out, err));
  return LMOE_OK;
}

template <int DT, bool W8A8>
static int launch_decode(const void* x, const float* weights, const int64_t* ids, int top, const int8_t* qg,
                         const float* sg, const int8_t* qd, const float* sd, int64_t E, int64_t H, int64_t I,
                         const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                         const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w, const void* residual,
                         void* out, void* hid, int* err, cudaStream_t st) {
  const int rows = top + (sh_qg != nullptr ? 1 : 0);
  const int cb = pick_cb(H, I), cbd = pick_cbd(rows, top, H, I);
  if (cb == 0 || cbd == 0) return LMOE_ERR_UNSUPPORTED;
  // MAXI = 16-byte chunks per lane of one row: H / 512 (gate_up), I / 512 (down)
#define LMOE_DEC(MG, MD)                                                                                           \
  return launch_decode_t<DT, W8A8, MG, MD>(x, weights, ids, top, qg, sg, qd, sd, E, H, I, sh_qg, sh_sg, sh_qu, sh_su, \
                                           sh_qd, sh_sd, sh_gate_w, residual, out, hid, err, cb, cbd, st)
  if (H <= 2048) {
    if (I <= 512) LMOE_DEC(4, 1);
    LMOE_DEC(4, kMaxChunksPerLane);
  }
  if (I <= 512) LMOE_DEC(kMaxChunksPerLane, 1);
  LMOE_DEC(kMaxChunksPerLane, kMaxChunksPerLane);
#undef LMOE_DEC
}

static bool a16(const void* p) { return p == nullptr || ((uintptr_t)p & 15) == 0; }

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
  // the weight rows and scales travel by bulk copies: 16-byte aligned sources
  if (!a16(qg) || !a16(sg) || !a16(qd) || !a16(sd) || !a16(sh_qg) || !a16(sh_sg) || !a16(sh_qu) || !a16(sh_su) ||
      !a16(sh_qd) || !a16(sh_sd) || !a16(x) || !a16(ws))
    return LMOE_ERR_INVALID;
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
