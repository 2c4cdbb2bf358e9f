// One-token MoE decode: the reference's Int8Experts decode branch
// (qwen35_deploy/operators/int8.py:158-187) with the gated HF shared expert
// (modeling_qwen3_5_moe.py:781-790), as ONE launch on the caller's stream with no
// host synchronisation (so it can be captured in a CUDA graph).
//
// decode_layer_kernel, one CTA per SM (persistent), two phases:
//   1. gate_up: a CTA takes blocks of CB hidden columns of one selected expert
//      (or of the shared expert): the block's gate rows and up rows (contiguous in
//      the bank) and their group scales arrive in shared memory by a few bulk
//      copies; one warp per column computes both dot products (W8A8 or W8A16
//      routed, W8A16 shared) and hidden = round(round(silu(g)) * u)
//      (int8.py:182-184), written to the workspace;
//   -- grid barrier (every CTA's hidden columns written) --
//   2. down: a CTA takes blocks of CBd output columns: the down rows of every
//      selected expert and of the shared expert for those columns, then one warp
//      per column computes the down dots, folding them in ascending expert order
//      into the ordered combine of _ordered_reduce (int8.py:240-250),
//      + round(sigmoid(round(x . gate)) * shared), + residual.
// Both phases' first blocks are requested at the kernel's start, so all of a
// layer's weight bytes (29.2 MB at the benchmark geometry) stream from HBM at once
// while phase 1 computes.  Each row's K is split over the 32 lanes of its warp
// (16 bytes per lane per chunk); the group partial sums are added in group order,
// as the reference's loop over groups does (w8a8.py:37-40).  Each CTA rebuilds
// the experts' ascending order from the router's ids (int8.py:170-179's table,
// without the ids.cpu() sync and the upload).  The per-row arithmetic is the
// grouped GEMV's (gemv.cuh).
//
// The grid barrier needs every CTA resident at once: the grid is at most the
// number of CTAs the device can hold (checked on the host), the kernel lets a
// dependent launch start only after the barrier, and the barrier's wait is
// bounded (a timeout sets LMOE_DEVERR_TIMEOUT and the CTAs return).
#include "common.cuh"
#include "gemm.cuh"
#include "gemv.cuh"

namespace lmoe {

constexpr int kDecodeMaxTop = 32;
constexpr int kDecThreads = 512;
constexpr int kDecWarps = kDecThreads / 32;
constexpr int kDecRowsMax = 8;  // down rows whose dots are computed together (one chunk per lane)
constexpr int kDecSmemMax = 220 * 1024;  // both phases' shared-memory regions

// Warp 0: s_eid[r] = the r-th smallest expert id (ties by slot) and s_w[r] the
// routing weight of its slot.  An id outside [0, E) becomes expert 0 (no read leaves
// the bank) and, when `report`, raises LMOE_DEVERR_BAD_EXPERT.
__device__ __forceinline__ void expert_ranks_w(const int64_t* ids, const float* weights, int top, int64_t E,
                                               int64_t* s_eid, float* s_w, int* err, bool report) {
  const int lane = lane_id();
  int64_t e = lane < top ? ids[lane] : INT64_MAX;
  const float wv = lane < top ? weights[lane] : 0.f;
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
    s_w[rank] = wv;
  }
}

__device__ __forceinline__ float silu_exact(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

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

// Grid barrier over all CTAs of a launch (every CTA resident), on one 64-bit word:
// the low half counts arrivals, the high half is the generation.  Each CTA adds 1;
// the last to arrive adds (1 << 32) - nctas, which restores the count to 0 and
// advances the generation in the same atomic; the others wait for the generation
// their own arrival returned to change.  The word's low half must be 0 before the
// first launch on a workspace, and every completed barrier leaves it 0.  The wait
// is bounded.
__device__ __forceinline__ bool grid_barrier(unsigned long long* bar, unsigned nctas, int* err) {
  __shared__ int s_ok;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long v = atomicAdd(bar, 1ull);
    const unsigned gen = (unsigned)(v >> 32);
    int ok = 1;
    if ((unsigned)v == nctas - 1) {
      atomicAdd(bar, (1ull << 32) - nctas);
    } else {
      volatile unsigned* hi = reinterpret_cast<volatile unsigned*>(bar) + 1;
      const uint64_t t0 = gtime_ns();
      while (*hi == gen) {
        if (gtime_ns() - t0 > LMOE_WAIT_NS) {
          raise_error(err, LMOE_DEVERR_TIMEOUT);
          ok = 0;
          break;
        }
      }
    }
    __threadfence();
    s_ok = ok;
  }
  __syncthreads();
  return s_ok != 0;
}

struct LayerArgs {
  const void* x;
  const float* weights;
  const int64_t* ids;
  int top;
  int64_t E, H, I;
  const int8_t *qg, *qd, *sh_qg, *sh_qu, *sh_qd;
  const float *sg, *sd, *sh_sg, *sh_su, *sh_sd;
  const void* gate_w;
  const void* residual;
  void* hid;
  void* out;
  unsigned long long* bar;
  int* err;
  int CB, CBd, n_gu, n_dn;
  int64_t gu_bytes;  // shared-memory bytes of the phase-1 region (the phase-2 region follows)
};

template <int DT, bool W8A8, int MAXG, int MAXD>
__global__ void __launch_bounds__(kDecThreads, 1) decode_layer_kernel(const LayerArgs a) {
  using A = Act<DT>;
  using T = typename A::T;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ int64_t s_eid[kDecodeMaxTop];
  __shared__ float s_w[kDecodeMaxTop];
  __shared__ float red[kDecWarps];
  __shared__ float s_t[kDecWarps][32];  // phase 2: per warp, its lanes' group terms
  const int lane = lane_id(), warp = warp_id();
  const int top = a.top;
  const int64_t H = a.H, I = a.I;
  const int GH = (int)(H / kGroup), GI = (int)(I / kGroup);
  const bool with_shared = a.sh_qg != nullptr;
  const bool gated = with_shared && a.gate_w != nullptr;
  const int rows = top + (with_shared ? 1 : 0);
  const T* x = (const T*)a.x;
  T* hid = (T*)a.hid;
  const GuSmem G(a.CB, H);
  const DnSmem D(rows, top, a.CBd, I);
  const uint32_t sb = smem_u32(smem);
  const uint32_t sd0 = sb + (uint32_t)a.gu_bytes;  // phase-2 region
  uint8_t* dsm = smem + a.gu_bytes;
  const int npieces = a.CB / 8;
  const int nblk = (int)(I / a.CB);
  if (threadIdx.x == 0) {
    for (int p = 0; p < npieces; ++p) mbar_init(sb + (uint32_t)G.bars + 8u * p, 1);
    mbar_init(sd0 + (uint32_t)D.bar, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Copies of one block.  A warp's bulk copies issue one after another (tens of ns
  // each), so a block's copies are spread over the warps: expect_* (warp 0, its lanes)
  // arms the barriers, copy_*(blk, k) issues copy k from the calling thread.  A copy
  // that lands before its barrier is armed is fine: the barrier's phase cannot complete
  // before the arming arrival.
  // gate_up block blk = pieces of 8 columns, each on its own barrier (gate rows, up
  // rows, their scales: 4 copies per piece), so warps start as their rows land
  const int n_gu_copies = 4 * npieces, n_dn_copies = 2 * rows;
  auto expect_gu = [&]() {
    const uint32_t wbytes = (uint32_t)(8 * H), sbytes = (uint32_t)(8 * GH * 4);
    if (lane < npieces) mbar_arrive_expect_tx(sb + (uint32_t)G.bars + 8u * lane, 2 * (wbytes + sbytes));
  };
  auto copy_gu = [&](int blk, int k) {
    const int r = blk / nblk;
    const int64_t c0 = (int64_t)(blk % nblk) * a.CB;
    const uint32_t wbytes = (uint32_t)(8 * H), sbytes = (uint32_t)(8 * GH * 4);
    const int p = k >> 2, which = k & 3;
    const uint32_t bar = sb + (uint32_t)G.bars + 8u * p;
    const int64_t row = c0 + p * 8 + ((which & 1) ? I : 0);  // gate rows, then up rows
    if (r < top) {
      const int64_t e = s_eid[r];
      if (which < 2) bulk_g2s(sb + (uint32_t)((which ? G.wu : G.wg) + p * 8 * H), a.qg + (e * 2 * I + row) * H, wbytes, bar);
      else bulk_g2s(sb + (uint32_t)((which & 1 ? G.su : G.sg) + p * 8 * GH * 4), a.sg + (e * 2 * I + row) * GH, sbytes, bar);
    } else {
      const int64_t srow = c0 + p * 8;
      const int8_t* q = (which & 1) ? a.sh_qu : a.sh_qg;
      const float* sc = (which & 1) ? a.sh_su : a.sh_sg;
      if (which < 2) bulk_g2s(sb + (uint32_t)((which ? G.wu : G.wg) + p * 8 * H), q + srow * H, wbytes, bar);
      else bulk_g2s(sb + (uint32_t)((which & 1 ? G.su : G.sg) + p * 8 * GH * 4), sc + srow * GH, sbytes, bar);
    }
  };
  // down block blk: per row (routed experts in ascending order, then the shared
  // expert) its CBd weight rows and their scales, all on one barrier
  auto expect_dn = [&]() {
    const uint32_t wb = (uint32_t)(a.CBd * I), sbt = (uint32_t)(a.CBd * GI * 4);
    if (lane == 0) mbar_arrive_expect_tx(sd0 + (uint32_t)D.bar, (uint32_t)rows * (wb + sbt));
  };
  auto copy_dn = [&](int blk, int k) {
    const int64_t n0 = (int64_t)blk * a.CBd;
    const uint32_t wb = (uint32_t)(a.CBd * I), sbt = (uint32_t)(a.CBd * GI * 4);
    const uint32_t bar = sd0 + (uint32_t)D.bar;
    const int rr = k >> 1;
    if ((k & 1) == 0) {
      const int8_t* q = rr < top ? a.qd + (s_eid[rr] * H + n0) * I : a.sh_qd + n0 * I;
      bulk_g2s(sd0 + (uint32_t)(D.w + (int64_t)rr * a.CBd * I), q, wb, bar);
    } else {
      const float* sc = rr < top ? a.sd + (s_eid[rr] * H + n0) * GI : a.sh_sd + n0 * GI;
      bulk_g2s(sd0 + (uint32_t)(D.sc + (int64_t)rr * a.CBd * GI * 4), sc, sbt, bar);
    }
  };
  // one warp issues all of a block's copies (later blocks, which are rare)
  auto issue_gu = [&](int blk) {
    expect_gu();
    __syncwarp();
    for (int k = lane; k < n_gu_copies; k += 32) copy_gu(blk, k);
  };
  auto issue_dn = [&](int blk) {
    expect_dn();
    __syncwarp();
    for (int k = lane; k < n_dn_copies; k += 32) copy_dn(blk, k);
  };

  // launched so that it may start before the previous kernel ends: the ids, the
  // routing weights, x and the hidden buffer (which the previous call reads) all
  // wait for it
  grid_dep_wait();
  int8_t* xq = reinterpret_cast<int8_t*>(smem + G.xq);
  float* xs = reinterpret_cast<float*>(smem + G.xs);
  const bool has_gu = (int)blockIdx.x < a.n_gu, first_dn = !has_gu && (int)blockIdx.x < a.n_dn;
  if (warp == 0) {
    // the experts' order and their routing weights; arm the first block's barriers
    expert_ranks_w(a.ids, a.weights, top, a.E, s_eid, s_w, a.err, blockIdx.x == 0);
    __syncwarp();
    if (has_gu) expect_gu();
    // a CTA with no gate_up block streams its down rows at once; the others once their
    // gate_up rows have landed, so that the two phases do not share the HBM stream
    else if (first_dn) expect_dn();
  } else {
    // meanwhile the other warps pull x (and the shared gate's weight) towards L1
    for (int64_t c = (int64_t)(threadIdx.x - 32) * 64; c < H; c += (int64_t)(kDecThreads - 32) * 64) {
      prefetch_l1(x + c);
      if (gated) prefetch_l1((const T*)a.gate_w + c);
    }
  }
  __syncthreads();
  // the first block's copies, one warp each
  if (lane == 0) {
    if (has_gu)
      for (int k = warp; k < n_gu_copies; k += kDecWarps) copy_gu(blockIdx.x, k);
    else if (first_dn)
      for (int k = warp; k < n_dn_copies; k += kDecWarps) copy_dn(blockIdx.x, k);
  }
  __syncwarp();
  // every warp quantises groups of x (W8A8) and forms part of the shared gate's logit
  if (W8A8)
    for (int g = warp; g < GH; g += kDecWarps) quant_group<DT>(x + g * kGroup, xq + g * kGroup, xs + g, lane);
  if (gated && warp > 0) {
    const T* gw = (const T*)a.gate_w;
    float part = 0.f;
    for (int64_t c = threadIdx.x - 32; c < H; c += kDecThreads - 32) part = fmaf(A::to_f(x[c]), A::to_f(gw[c]), part);
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane == 0) red[warp] = part;
  }
  __syncthreads();

  // ---- phase 1: gate_up + SwiGLU
  int ok = 1;
  const int chunks1 = (int)(H / 16);
  int it = 0;
  for (int blk = blockIdx.x; blk < a.n_gu && ok; blk += gridDim.x, ++it) {
    const int r = blk / nblk;
    const int64_t c0 = (int64_t)(blk % nblk) * a.CB;
    for (int j = warp; j < a.CB; j += kDecWarps) {
      if (!mbar_wait_drain(sb + (uint32_t)G.bars + 8u * (j / 8), it & 1, a.err)) {
        ok = 0;
        break;
      }
      uint4 wg[MAXG], wu[MAXG];
      row_lds(sb + (uint32_t)(G.wg + j * H), chunks1, lane, wg);
      row_lds(sb + (uint32_t)(G.wu + j * H), chunks1, lane, wu);
      const float* gsr = reinterpret_cast<const float*>(smem + G.sg) + j * GH;
      const float* usr = reinterpret_cast<const float*>(smem + G.su) + j * GH;
      float g, u;
      if (W8A8 && r < top) {
        g = row_dot_w8a8_ilp(wg, gsr, xq, xs, chunks1, lane);
        u = row_dot_w8a8_ilp(wu, usr, xq, xs, chunks1, lane);
      } else {  // W8A16 routed experts, and the shared expert (Int8Linear arithmetic)
        g = row_dot_w16<DT>(wg, gsr, x, chunks1, lane);
        u = row_dot_w16<DT>(wu, usr, x, chunks1, lane);
      }
      if (lane == 0) hid[(int64_t)r * I + c0 + j] = A::from_f(__fmul_rn(A::round(silu_exact(A::round(g))), A::round(u)));
    }
    if (it == 0 && (int)blockIdx.x < a.n_dn && warp < n_dn_copies) {
      // all of this CTA's first gate_up pieces have landed: its down rows go out now,
      // from each warp that has a down copy to issue once its own columns are done
      for (int p = 0; p < npieces; ++p)
        if (!mbar_wait_drain(sb + (uint32_t)G.bars + 8u * p, 0, a.err)) ok = 0;
      if (warp == 0) expect_dn();
      if (lane == 0)
        for (int k = warp; k < n_dn_copies; k += kDecWarps) copy_dn(blockIdx.x, k);
      __syncwarp();
    }
    ok = __syncthreads_and(ok);  // every warp is done with this block's rows
    if (warp == 0 && ok && blk + (int)gridDim.x < a.n_gu) issue_gu(blk + gridDim.x);
  }
  const bool passed = grid_barrier(a.bar, gridDim.x, a.err);
  grid_dep_launch();  // every CTA of this launch is resident: a dependent may take SMs as they leave
  if (!passed || !ok) {
    // never leave this CTA with its phase-2 copies still in flight
    if ((int)blockIdx.x < a.n_dn) mbar_wait_drain(sd0 + (uint32_t)D.bar, 0, a.err);
    return;
  }

  // ---- phase 2: down + ordered combine + gated shared expert + residual
  int8_t* hq = reinterpret_cast<int8_t*>(dsm + D.hq);
  float* hs = reinterpret_cast<float*>(dsm + D.hs);
  // the hidden rows (routed and shared, activation dtype) in the phase-1 region, whose
  // reads and copies are all complete
  const T* hx = reinterpret_cast<const T*>(smem + G.wg);
  if ((int)blockIdx.x < a.n_dn) {
    // every hidden row into shared memory in one L2 round trip (the rows come from
    // other CTAs: read through L2), then the W8A8 quantisation from there
    const int n16 = (int)(rows * I * 2 / 16);
    const uint32_t hx0 = sb + (uint32_t)G.wg;
    for (int b0 = 0; b0 < n16; b0 += 2 * kDecThreads) {
      uint4 v[2];
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = b0 + i * kDecThreads + (int)threadIdx.x;
        if (idx < n16) v[i] = __ldcg(reinterpret_cast<const uint4*>(hid) + idx);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int idx = b0 + i * kDecThreads + (int)threadIdx.x;
        if (idx < n16) sts128(hx0 + (uint32_t)idx * 16u, v[i]);
      }
    }
    __syncthreads();
    if (W8A8) {
      // two (row, group) quantisations per pass, independent so that they overlap
      for (int t0 = warp; t0 < top * GI; t0 += 2 * kDecWarps) {
        float v[2][4];
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int t = min(t0 + u * kDecWarps, top * GI - 1);
          const int rr = t / GI, g = t % GI;
          const uint2 raw = *reinterpret_cast<const uint2*>(hx + (int64_t)rr * I + g * kGroup + lane * 4);
          v[u][0] = A::lo_f(raw.x);
          v[u][1] = A::hi_f(raw.x);
          v[u][2] = A::lo_f(raw.y);
          v[u][3] = A::hi_f(raw.y);
        }
#pragma unroll
        for (int u = 0; u < 2; ++u) {
          const int t = t0 + u * kDecWarps;
          if (t < top * GI) {
            const int rr = t / GI, g = t % GI;
            quant_vals(v[u], hq + (int64_t)rr * I + g * kGroup, hs + rr * GI + g, lane);
          }
        }
      }
    }
  }
  __syncthreads();
  float sig = 1.f;
  if (gated) {
    float tot = 0.f;
#pragma unroll
    for (int i = 1; i < kDecWarps; ++i) tot += red[i];
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-A::round(tot)))));
  }
  const int chunks2 = (int)(I / 16);
  const float* scs = reinterpret_cast<const float*>(dsm + D.sc);
  const T* res = (const T*)a.residual;
  T* out = (T*)a.out;
  int it2 = 0;
  for (int blk = blockIdx.x; blk < a.n_dn; blk += gridDim.x, ++it2) {
    const int64_t n0 = (int64_t)blk * a.CBd;
    // per column j (one warp): its residual and the shared expert's hidden chunk are
    // loaded before the weights' wait
    const int j0 = warp;
    const bool have_col = j0 < a.CBd;
    float resv = 0.f;
    if (have_col && res != nullptr) resv = A::to_f(res[n0 + j0]);
    if (!__syncthreads_and(mbar_wait_drain(sd0 + (uint32_t)D.bar, it2 & 1, a.err) ? 1 : 0)) return;
    for (int j = warp; j < a.CBd; j += kDecWarps) {
      const int64_t n = n0 + j;
      if (j != j0 && res != nullptr) resv = A::to_f(res[n]);
      float acc = 0.f;
      if (W8A8 && top * GI <= 32) {
        // one lane per (routed row rr = lane / GI, 128-group g = lane % GI): the group's
        // exact int32 dot (8 chunks, visited from a lane-dependent start so that the 8
        // lanes of a shared-memory phase read different banks), t = (dot * xs) * ws;
        // then lane 0 adds each row's groups in group order and folds the rows in
        // ascending expert order, as row_dot_w8a8 and the combine below do
        const int rr = lane / GI, g = lane - rr * GI;
        float t = 0.f;
        if (rr < top) {
          const uint32_t wrow = sd0 + (uint32_t)(D.w + ((int64_t)rr * a.CBd + j) * I + g * kGroup);
          const uint32_t xrow = smem_u32(hq + (int64_t)rr * I + g * kGroup);
          int dsum = 0;
#pragma unroll
          for (int c = 0; c < kGroup / 16; ++c) {
            const uint32_t off = (uint32_t)(((c + lane) & 7) * 16);
            const uint4 wv = lds128(wrow + off), xv = lds128(xrow + off);
            dsum = dp4a(wv.x, xv.x, dsum);
            dsum = dp4a(wv.y, xv.y, dsum);
            dsum = dp4a(wv.z, xv.z, dsum);
            dsum = dp4a(wv.w, xv.w, dsum);
          }
          t = __fmul_rn(__fmul_rn((float)dsum, hs[rr * GI + g]), scs[((int64_t)rr * a.CBd + j) * GI + g]);
        }
        s_t[warp][lane] = t;
        __syncwarp();
        if (lane == 0) {
          for (int r = 0; r < top; ++r) {
            float v = 0.f;
            for (int q = 0; q < GI; ++q) v = __fadd_rn(v, s_t[warp][r * GI + q]);
            acc = A::round(__fadd_rn(acc, A::round(__fmul_rn(A::round(v), s_w[r]))));
          }
        }
        acc = __shfl_sync(0xffffffffu, acc, 0);
        __syncwarp();
      } else {
      constexpr int kDecRows = MAXD == 1 ? kDecRowsMax : 1;  // keep the rows' chunks in registers
      for (int r0 = 0; r0 < top; r0 += kDecRows) {
        uint4 w[kDecRows][MAXD];
        const float* srow[kDecRows];
        const int8_t* xr[kDecRows];
        const float* xsr[kDecRows];
        float v[kDecRows];
#pragma unroll
        for (int k = 0; k < kDecRows; ++k) {
          const int rr = min(r0 + k, top - 1);  // rows past top repeat the last one (unused)
          row_lds(sd0 + (uint32_t)(D.w + ((int64_t)rr * a.CBd + j) * I), chunks2, lane, w[k]);
          srow[k] = scs + ((int64_t)rr * a.CBd + j) * GI;
          xr[k] = hq + (int64_t)rr * I;
          xsr[k] = hs + rr * GI;
        }
        if (W8A8) {
          rows_dot_w8a8_ilp<MAXD, kDecRows>(w, srow, xr, xsr, chunks2, lane, v);
        } else {
#pragma unroll
          for (int k = 0; k < kDecRows; ++k)
            v[k] = row_dot_w16<DT, MAXD>(w[k], srow[k], hx + (int64_t)min(r0 + k, top - 1) * I, chunks2, lane);
        }
#pragma unroll
        for (int k = 0; k < kDecRows; ++k)
          if (r0 + k < top) acc = A::round(__fadd_rn(acc, A::round(__fmul_rn(A::round(v[k]), s_w[r0 + k]))));
      }
      }
      if (with_shared) {
        uint4 w[MAXD];
        row_lds(sd0 + (uint32_t)(D.w + ((int64_t)top * a.CBd + j) * I), chunks2, lane, w);
        const float sv = A::round(
            row_dot_w16<DT, MAXD>(w, scs + ((int64_t)top * a.CBd + j) * GI, hx + (int64_t)top * I, chunks2, lane));
        acc = A::round(__fadd_rn(acc, gated ? A::round(__fmul_rn(sig, sv)) : sv));
      }
      if (res != nullptr) acc = A::round(__fadd_rn(resv, acc));
      if (lane == 0) out[n] = A::from_f(acc);
    }
    __syncthreads();
    if (warp == 0 && blk + (int)gridDim.x < a.n_dn) issue_dn(blk + gridDim.x);
  }

}

// The grid barrier's two words come first, at a fixed offset, so that a workspace
// reused for another geometry keeps them where the previous calls left them (zero).
struct DecodeWs {
  int64_t off_bar, off_h, bytes;
  static int64_t align(int64_t v) { return (v + 255) & ~int64_t(255); }
  DecodeWs(int64_t top, int64_t H, int64_t I) {
    (void)H;
    off_bar = 0;
    off_h = 256;                                  // hidden rows: routed + shared
    bytes = off_h + align((top + 1) * I * 2);
  }
};

static int64_t a128(int64_t v) { return (v + 127) & ~int64_t(127); }

// columns per CTA: the largest blocks whose rows fit both phases' shared memory
static bool pick_blocks(int64_t rows, int64_t top, int64_t H, int64_t I, int& cb, int& cbd) {
  for (cb = 32; cb >= 8; cb >>= 1) {
    if (I % cb) continue;
    for (cbd = 16; cbd >= 4; cbd >>= 1)
      if (H % cbd == 0 && a128(GuSmem(cb, H).bytes) + DnSmem(rows, top, cbd, I).bytes <= kDecSmemMax &&
          rows * I * 2 <= GuSmem(cb, H).bytes)  // phase 2 stages the hidden rows in the phase-1 region
        return true;
  }
  return false;
}

template <int DT, bool W8A8, int MAXG, int MAXD>
static int launch_layer(LayerArgs& a, int rows, cudaStream_t st) {
  auto k = decode_layer_kernel<DT, W8A8, MAXG, MAXD>;
  a.gu_bytes = a128(GuSmem(a.CB, a.H).bytes);
  const int64_t smem = a.gu_bytes + DnSmem(rows, a.top, a.CBd, a.I).bytes;
  LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributePreferredSharedMemoryCarveout,
                                       (int)cudaSharedmemCarveoutMaxShared));
  // every CTA must be resident at once for the grid barrier
  int per_sm = 0;
  LMOE_CUDA_CHECK(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, k, kDecThreads, (size_t)smem));
  const int64_t resident = (int64_t)per_sm * sm_count();
  if (resident <= 0) return LMOE_ERR_UNSUPPORTED;
  const int64_t want = a.n_gu > a.n_dn ? a.n_gu : a.n_dn;
  const unsigned grid = (unsigned)(want < resident ? want : resident);
  LMOE_CUDA_CHECK(launch_pdl(k, dim3(grid), dim3(kDecThreads), (size_t)smem, st, a));
  return LMOE_OK;
}

template <int DT, bool W8A8>
static int launch_decode(LayerArgs& a, int rows, cudaStream_t st) {
  if (!pick_blocks(rows, a.top, a.H, a.I, a.CB, a.CBd)) return LMOE_ERR_UNSUPPORTED;
  a.n_gu = (int)(rows * (a.I / a.CB));
  a.n_dn = (int)(a.H / a.CBd);
  // MAXI = 16-byte chunks per lane of one row: H / 512 (gate_up), I / 512 (down)
  if (a.H <= 2048) {
    if (a.I <= 512) return launch_layer<DT, W8A8, 4, 1>(a, rows, st);
    return launch_layer<DT, W8A8, 4, kMaxChunksPerLane>(a, rows, st);
  }
  if (a.I <= 512) return launch_layer<DT, W8A8, kMaxChunksPerLane, 1>(a, rows, st);
  return launch_layer<DT, W8A8, kMaxChunksPerLane, kMaxChunksPerLane>(a, rows, st);
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
  const DecodeWs W(top, H, I);
  LayerArgs a = {};
  a.x = x;
  a.weights = weights;
  a.ids = ids;
  a.top = (int)top;
  a.E = E;
  a.H = H;
  a.I = I;
  a.qg = qg;
  a.qd = qd;
  a.sh_qg = sh_qg;
  a.sh_qu = sh_qu;
  a.sh_qd = sh_qd;
  a.sg = sg;
  a.sd = sd;
  a.sh_sg = sh_sg;
  a.sh_su = sh_su;
  a.sh_sd = sh_sd;
  a.gate_w = sh_gate_w;
  a.residual = residual;
  a.hid = (char*)ws + W.off_h;
  a.bar = (unsigned long long*)((char*)ws + W.off_bar);
  a.out = out;
  a.err = err;
  const int rows = (int)top + (with_shared ? 1 : 0);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    return w8a8 ? launch_decode<LMOE_BF16, true>(a, rows, st) : launch_decode<LMOE_BF16, false>(a, rows, st);
  return w8a8 ? launch_decode<LMOE_F16, true>(a, rows, st) : launch_decode<LMOE_F16, false>(a, rows, st);
}
