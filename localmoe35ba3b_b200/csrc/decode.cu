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
constexpr int kDecMaxS = 64;             // shared-expert columns per gate_up block

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

// Shared memory: the phase-1 region (gate_up) and the phase-2 region (down) overlap,
// both from offset 0 -- the down rows are copied in once every gate_up read is done (their
// HBM bytes were prefetched into L2 meanwhile) -- and the mbarriers sit after both.
// Phase 1: a routed block of CB columns (its CB gate and CB up rows) and a slice of S
// columns of the shared expert (S gate and S up rows), their group scales, and x
// quantised (W8A8).
struct GuSmem {
  int64_t wg, wu, sg, su, shg, shu, ssg, ssu, xq, xs, bytes;
  __host__ __device__ GuSmem(int64_t CB, int64_t S, int64_t H) {
    const int64_t GH = H / kGroup;
    wg = 0;
    wu = CB * H;
    sg = 2 * CB * H;
    su = sg + CB * GH * 4;
    shg = su + CB * GH * 4;
    shu = shg + S * H;
    ssg = shu + S * H;
    ssu = ssg + S * GH * 4;
    xq = ssu + S * GH * 4;
    xs = xq + H;
    bytes = (xs + GH * 4 + 127) & ~int64_t(127);
  }
};

// Phase 2: CBd down rows of every selected expert and of the shared expert, their
// scales, the hidden rows quantised (W8A8) and in the activation dtype.
struct DnSmem {
  int64_t w, sc, hq, hs, hx, bytes;
  __host__ __device__ DnSmem(int64_t rows, int64_t top, int64_t CBd, int64_t I) {
    const int64_t GI = I / kGroup;
    w = 0;
    sc = rows * CBd * I;
    hq = sc + rows * CBd * GI * 4;
    hs = hq + top * I;
    hx = (hs + top * GI * 4 + 15) & ~int64_t(15);
    bytes = (hx + rows * I * 2 + 127) & ~int64_t(127);
  }
};

// barriers: one per 8-column piece of the routed block, one for the shared slice, one
// for the down rows
__host__ __device__ inline int64_t dec_bars_bytes(int64_t CB) { return (CB / 8 + 2) * 8; }

// Grid barrier over all CTAs of a launch (every CTA resident), on a 64-bit counter that
// only grows: each CTA adds 1 and waits until the counter reaches the next multiple of
// the grid size, so the last arrival releases everyone with no second write.  That
// needs the counter to start every launch at a multiple of the grid size, so each grid
// size has its own counter (slot gridDim.x of kDecBarSlots); the workspace's counters
// start at zero.  Arrival and wait are split so that a CTA can issue work that needs no
// other CTA in between; the wait is bounded.
constexpr int kDecBarSlots = 1024;
__device__ __forceinline__ unsigned long long grid_arrive(unsigned long long* ctr, unsigned nctas) {
  __shared__ unsigned long long s_target;
  __threadfence();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned long long v = atomicAdd(ctr, 1ull);
    s_target = (v / nctas + 1) * nctas;
  }
  __syncthreads();
  return s_target;
}
__device__ __forceinline__ bool grid_wait(unsigned long long* ctr, unsigned long long target, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) {
    volatile unsigned long long* c = ctr;
    int ok = 1;
    const uint64_t t0 = gtime_ns();
    while (*c < target) {
      if (gtime_ns() - t0 > LMOE_WAIT_NS) {
        raise_error(err, LMOE_DEVERR_TIMEOUT);
        ok = 0;
        break;
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
  int CB, CBd, S, n_gu, n_dn;  // S: shared-expert columns per gate_up block (multiple of 4)
  int64_t bar_off;             // shared-memory offset of the mbarriers (after both regions)
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
  __shared__ float s_sh[2][kDecMaxS];    // phase 1: the shared slice's gate and up dots
  const int lane = lane_id(), warp = warp_id();
  const int top = a.top;
  const int64_t H = a.H, I = a.I;
  const int GH = (int)(H / kGroup), GI = (int)(I / kGroup);
  const bool with_shared = a.sh_qg != nullptr;
  const bool gated = with_shared && a.gate_w != nullptr;
  const int rows = top + (with_shared ? 1 : 0);
  const T* x = (const T*)a.x;
  T* hid = (T*)a.hid;
  const GuSmem G(a.CB, a.S, H);
  const DnSmem D(rows, top, a.CBd, I);
  const uint32_t sb = smem_u32(smem);
  const int npieces = a.CB / 8;
  const uint32_t bars = sb + (uint32_t)a.bar_off;
  const uint32_t bar_sh = bars + 8u * npieces, bar_dn = bars + 8u * (npieces + 1);
  const int nblk = (int)(I / a.CB);
  if (threadIdx.x == 0) {
    for (int p = 0; p < npieces + 2; ++p) mbar_init(bars + 8u * p, 1);
    fence_mbar_init();
  }
  __syncthreads();

  // Copies of one block.  A warp's bulk copies issue one after another (tens of ns
  // each), so a block's copies are spread over the warps: expect_* (warp 0, its lanes)
  // arms the barriers, copy_*(blk, k) issues copy k from the calling thread.  A copy
  // that lands before its barrier is armed is fine: the barrier's phase cannot complete
  // before the arming arrival.
  // gate_up block blk: the routed rows in pieces of 8 columns, each on its own barrier
  // (gate rows, up rows, their scales: 4 copies per piece), so warps start as their rows
  // land, and the shared expert's slice of ns(blk) columns on one barrier (4 copies)
  auto sh_cols = [&](int blk) -> int {
    const int64_t c0 = (int64_t)blk * a.S;
    return with_shared && c0 < I ? (int)min((int64_t)a.S, I - c0) : 0;
  };
  const int n_gu_copies = 4 * npieces + 4, n_dn_copies = 2 * rows;
  auto expect_gu = [&](int blk) {
    const uint32_t wbytes = (uint32_t)(8 * H), sbytes = (uint32_t)(8 * GH * 4);
    if (lane < npieces) mbar_arrive_expect_tx(bars + 8u * lane, 2 * (wbytes + sbytes));
    // (the first block's shared slice is armed and requested before the dependency wait)
    const int ns = sh_cols(blk);
    if (lane == 0 && ns > 0 && blk != (int)blockIdx.x) mbar_arrive_expect_tx(bar_sh, (uint32_t)(2 * ns * (H + GH * 4)));
  };
  auto copy_gu = [&](int blk, int k) {
    const int r = blk / nblk;
    const int64_t c0 = (int64_t)(blk % nblk) * a.CB;
    if (k < 4 * npieces) {
      const uint32_t wbytes = (uint32_t)(8 * H), sbytes = (uint32_t)(8 * GH * 4);
      const int p = k >> 2, which = k & 3;
      const uint32_t bar = bars + 8u * p;
      const int64_t row = c0 + p * 8 + ((which & 1) ? I : 0);  // gate rows, then up rows
      const int64_t e = s_eid[r];
      if (which < 2) bulk_g2s(sb + (uint32_t)((which ? G.wu : G.wg) + p * 8 * H), a.qg + (e * 2 * I + row) * H, wbytes, bar);
      else bulk_g2s(sb + (uint32_t)((which & 1 ? G.su : G.sg) + p * 8 * GH * 4), a.sg + (e * 2 * I + row) * GH, sbytes, bar);
    } else {
      const int ns = sh_cols(blk), which = k - 4 * npieces;
      if (ns == 0) return;
      const int64_t s0 = (int64_t)blk * a.S;
      const int8_t* q = (which & 1) ? a.sh_qu : a.sh_qg;
      const float* sc = (which & 1) ? a.sh_su : a.sh_sg;
      if (which < 2) bulk_g2s(sb + (uint32_t)((which ? G.shu : G.shg)), q + s0 * H, (uint32_t)(ns * H), bar_sh);
      else bulk_g2s(sb + (uint32_t)((which & 1 ? G.ssu : G.ssg)), sc + s0 * GH, (uint32_t)(ns * GH * 4), bar_sh);
    }
  };
  // down block blk: per row (routed experts in ascending order, then the shared
  // expert) its CBd weight rows and their scales, all on one barrier; prefetch_dn pulls
  // the same bytes into L2 (no shared memory) while phase 1 runs
  auto dn_src = [&](int blk, int k, const void*& src, uint32_t& bytes, uint32_t& dst) {
    const int64_t n0 = (int64_t)blk * a.CBd;
    const int rr = k >> 1;
    if ((k & 1) == 0) {
      src = rr < top ? a.qd + (s_eid[rr] * H + n0) * I : a.sh_qd + n0 * I;
      bytes = (uint32_t)(a.CBd * I);
      dst = sb + (uint32_t)(D.w + (int64_t)rr * a.CBd * I);
    } else {
      src = rr < top ? a.sd + (s_eid[rr] * H + n0) * GI : a.sh_sd + n0 * GI;
      bytes = (uint32_t)(a.CBd * GI * 4);
      dst = sb + (uint32_t)(D.sc + (int64_t)rr * a.CBd * GI * 4);
    }
  };
  auto expect_dn = [&]() {
    const uint32_t wb = (uint32_t)(a.CBd * I), sbt = (uint32_t)(a.CBd * GI * 4);
    if (lane == 0) mbar_arrive_expect_tx(bar_dn, (uint32_t)rows * (wb + sbt));
  };
  auto copy_dn = [&](int blk, int k) {
    const void* src;
    uint32_t bytes, dst;
    dn_src(blk, k, src, bytes, dst);
    bulk_g2s(dst, src, bytes, bar_dn);
  };
  auto prefetch_dn = [&](int blk, int k) {
    const void* src;
    uint32_t bytes, dst;
    dn_src(blk, k, src, bytes, dst);
    bulk_prefetch_l2(src, bytes);
  };
  // one warp issues all of a block's copies (later blocks, which are rare)
  auto issue_gu = [&](int blk) {
    expect_gu(blk);
    __syncwarp();
    for (int k = lane; k < n_gu_copies; k += 32) copy_gu(blk, k);
  };
  auto issue_dn = [&](int blk) {
    expect_dn();
    __syncwarp();
    for (int k = lane; k < n_dn_copies; k += 32) copy_dn(blk, k);
  };

  const bool has_gu = (int)blockIdx.x < a.n_gu, has_dn = (int)blockIdx.x < a.n_dn;
  // the shared expert's rows depend on nothing the previous kernel writes: this CTA's first
  // slice of them is requested, and its shared down rows pulled towards L2, before waiting
  const int ns0 = has_gu ? sh_cols(blockIdx.x) : 0;
  if (threadIdx.x == 0) {
    if (ns0 > 0) {
      mbar_arrive_expect_tx(bar_sh, (uint32_t)(2 * ns0 * (H + GH * 4)));
      for (int k = 4 * npieces; k < n_gu_copies; ++k) copy_gu(blockIdx.x, k);
    }
    if (has_dn && with_shared) {
      prefetch_dn(blockIdx.x, 2 * top);
      prefetch_dn(blockIdx.x, 2 * top + 1);
    }
  }
  // launched so that it may start before the previous kernel ends: the ids, the
  // routing weights, x and the hidden buffer (which the previous call reads) all
  // wait for it
  grid_dep_wait();
  int8_t* xq = reinterpret_cast<int8_t*>(smem + G.xq);
  float* xs = reinterpret_cast<float*>(smem + G.xs);
  if (warp == 0) {
    // the experts' order and their routing weights; arm the first block's barriers
    expert_ranks_w(a.ids, a.weights, top, a.E, s_eid, s_w, a.err, blockIdx.x == 0);
    __syncwarp();
    if (has_gu) expect_gu(blockIdx.x);
  } else {
    // meanwhile the other warps pull x (and the shared gate's weight) towards L1
    for (int64_t c = (int64_t)(threadIdx.x - 32) * 64; c < H; c += (int64_t)(kDecThreads - 32) * 64) {
      prefetch_l1(x + c);
      if (gated) prefetch_l1((const T*)a.gate_w + c);
    }
  }
  __syncthreads();
  // the first block's routed copies, one warp each
  if (lane == 0 && has_gu)
    for (int k = warp; k < 4 * npieces; k += kDecWarps) copy_gu(blockIdx.x, k);
  __syncwarp();
  // every warp quantises groups of x (W8A8) and forms part of the shared gate's logit;
  // then the first down block's L2 prefetches (needed only after the grid barrier)
  if (W8A8)
    for (int g = warp; g < GH; g += kDecWarps) quant_group<DT>(x + g * kGroup, xq + g * kGroup, xs + g, lane);
  if (lane == 0 && has_dn)
    for (int k = warp; k < 2 * top; k += kDecWarps) prefetch_dn(blockIdx.x, k);
  __syncwarp();
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
      if (!mbar_wait_drain(bars + 8u * (j / 8), it & 1, a.err)) {
        ok = 0;
        break;
      }
      uint4 wg[MAXG], wu[MAXG];
      row_lds(sb + (uint32_t)(G.wg + j * H), chunks1, lane, wg);
      row_lds(sb + (uint32_t)(G.wu + j * H), chunks1, lane, wu);
      const float* gsr = reinterpret_cast<const float*>(smem + G.sg) + j * GH;
      const float* usr = reinterpret_cast<const float*>(smem + G.su) + j * GH;
      float g, u;
      if (W8A8) {
        g = row_dot_w8a8_ilp(wg, gsr, xq, xs, chunks1, lane);
        u = row_dot_w8a8_ilp(wu, usr, xq, xs, chunks1, lane);
      } else {
        g = row_dot_w16<DT>(wg, gsr, x, chunks1, lane);
        u = row_dot_w16<DT>(wu, usr, x, chunks1, lane);
      }
      if (lane == 0) hid[(int64_t)r * I + c0 + j] = A::from_f(__fmul_rn(A::round(silu_exact(A::round(g))), A::round(u)));
    }
    // the shared expert's slice (W8A16, the reference's Int8Linear arithmetic): one row dot
    // per warp, from the last warp down (the first warps took the extra routed columns)
    const int ns = sh_cols(blk);
    if (ns > 0) {
      for (int rd = kDecWarps - 1 - warp; rd < 2 * ns && ok; rd += kDecWarps) {
        if (!mbar_wait_drain(bar_sh, it & 1, a.err)) {
          ok = 0;
          break;
        }
        const int jj = rd % ns, up = rd / ns;
        uint4 w[MAXG];
        row_lds(sb + (uint32_t)((up ? G.shu : G.shg) + jj * H), chunks1, lane, w);
        const float* srow = reinterpret_cast<const float*>(smem + (up ? G.ssu : G.ssg)) + jj * GH;
        const float v = row_dot_w16<DT>(w, srow, x, chunks1, lane);
        if (lane == 0) s_sh[up][jj] = v;
      }
    }
    ok = __syncthreads_and(ok);  // every warp is done with this block's rows
    if (ns > 0 && ok)
      for (int jj = threadIdx.x; jj < ns; jj += kDecThreads)
        hid[(int64_t)top * I + (int64_t)blk * a.S + jj] =
            A::from_f(__fmul_rn(A::round(silu_exact(A::round(s_sh[0][jj]))), A::round(s_sh[1][jj])));
    if (warp == 0 && ok && blk + (int)gridDim.x < a.n_gu) issue_gu(blk + gridDim.x);
    __syncthreads();  // s_sh is read before the next block's dots write it
  }
  // arrive at the grid barrier, then (needing no other CTA) bring this CTA's first down
  // block from L2 into the now free shared memory, then wait for every CTA's hidden rows
  unsigned long long* const ctr = a.bar + gridDim.x;  // this grid size's counter
  const unsigned long long target = grid_arrive(ctr, gridDim.x);
  grid_dep_launch();  // every CTA of this launch is resident: a dependent may take SMs as they leave
  if (has_dn && ok) {
    if (warp == 0) expect_dn();
    __syncwarp();
    if (lane == 0)
      for (int k = warp; k < n_dn_copies; k += kDecWarps) copy_dn(blockIdx.x, k);
    __syncwarp();
  }
  const bool passed = grid_wait(ctr, target, a.err);
  if (!passed || !ok) {
    // never leave this CTA with its phase-2 copies still in flight
    if (has_dn && ok) mbar_wait_drain(bar_dn, 0, a.err);
    return;
  }

  // ---- phase 2: down + ordered combine + gated shared expert + residual
  int8_t* hq = reinterpret_cast<int8_t*>(smem + D.hq);
  float* hs = reinterpret_cast<float*>(smem + D.hs);
  const T* hx = reinterpret_cast<const T*>(smem + D.hx);
  if (has_dn) {
    // every hidden row into shared memory in one L2 round trip (the rows come from
    // other CTAs: read through L2), then the W8A8 quantisation from there
    const int n16 = (int)(rows * I * 2 / 16);
    const uint32_t hx0 = sb + (uint32_t)D.hx;
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
  const float* scs = reinterpret_cast<const float*>(smem + D.sc);
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
    if (!__syncthreads_and(mbar_wait_drain(bar_dn, it2 & 1, a.err) ? 1 : 0)) return;
    for (int j = warp; j < a.CBd; j += kDecWarps) {
      const int64_t n = n0 + j;
      if (j != j0 && res != nullptr) resv = A::to_f(res[n]);
      // the shared expert's down row first (it needs nothing from the routed rows, and its
      // latency then overlaps theirs)
      float sv = 0.f;
      if (with_shared) {
        uint4 w[MAXD];
        row_lds(sb + (uint32_t)(D.w + ((int64_t)top * a.CBd + j) * I), chunks2, lane, w);
        sv = A::round(
            row_dot_w16<DT, MAXD>(w, scs + ((int64_t)top * a.CBd + j) * GI, hx + (int64_t)top * I, chunks2, lane));
      }
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
          const uint32_t wrow = sb + (uint32_t)(D.w + ((int64_t)rr * a.CBd + j) * I + g * kGroup);
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
          row_lds(sb + (uint32_t)(D.w + ((int64_t)rr * a.CBd + j) * I), chunks2, lane, w[k]);
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
      if (with_shared) acc = A::round(__fadd_rn(acc, gated ? A::round(__fmul_rn(sig, sv)) : sv));
      if (res != nullptr) acc = A::round(__fadd_rn(resv, acc));
      if (lane == 0) out[n] = A::from_f(acc);
    }
    __syncthreads();
    if (warp == 0 && blk + (int)gridDim.x < a.n_dn) issue_dn(blk + gridDim.x);
  }

}

// The grid barrier's counters come first, at a fixed offset, so that a workspace reused
// for another geometry keeps them where the previous calls left them (each a multiple of
// its grid size; zero in a new workspace).
struct DecodeWs {
  int64_t off_bar, off_h, bytes;
  static int64_t align(int64_t v) { return (v + 255) & ~int64_t(255); }
  DecodeWs(int64_t top, int64_t H, int64_t I) {
    (void)H;
    off_bar = 0;
    off_h = kDecBarSlots * 8;                     // hidden rows: routed + shared
    bytes = off_h + align((top + 1) * I * 2);
  }
};

// gate_up blocks of cb routed columns (top * I / cb of them), each with a slice of s
// shared-expert columns (s a multiple of 4, so that a slice's scale rows copy in 16-byte
// units), and down blocks of cbd columns: the largest blocks whose phases fit in shared
// memory (both regions overlap)
static int64_t dec_smem(int64_t rows, int64_t top, int64_t H, int64_t I, int cb, int s, int cbd) {
  const int64_t p1 = GuSmem(cb, s, H).bytes, p2 = DnSmem(rows, top, cbd, I).bytes;
  return (p1 > p2 ? p1 : p2) + dec_bars_bytes(cb);
}
static bool pick_blocks(int64_t rows, int64_t top, int64_t H, int64_t I, bool with_shared, int& cb, int& s,
                        int& cbd) {
  for (cb = 32; cb >= 8; cb >>= 1) {
    if (I % cb) continue;
    const int64_t n_gu = top * (I / cb);
    s = with_shared ? (int)((((I + n_gu - 1) / n_gu) + 3) & ~int64_t(3)) : 0;
    if (s > kDecMaxS) continue;
    for (cbd = 16; cbd >= 4; cbd >>= 1)
      if (H % cbd == 0 && dec_smem(rows, top, H, I, cb, s, cbd) <= kDecSmemMax) return true;
  }
  return false;
}

template <int DT, bool W8A8, int MAXG, int MAXD>
static int launch_layer(LayerArgs& a, int rows, cudaStream_t st) {
  auto k = decode_layer_kernel<DT, W8A8, MAXG, MAXD>;
  const int64_t p1 = GuSmem(a.CB, a.S, a.H).bytes, p2 = DnSmem(rows, a.top, a.CBd, a.I).bytes;
  a.bar_off = p1 > p2 ? p1 : p2;
  const int64_t smem = dec_smem(rows, a.top, a.H, a.I, a.CB, a.S, a.CBd);
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
  if (grid >= (unsigned)kDecBarSlots) return LMOE_ERR_UNSUPPORTED;
  LMOE_CUDA_CHECK(launch_pdl(k, dim3(grid), dim3(kDecThreads), (size_t)smem, st, a));
  return LMOE_OK;
}

template <int DT, bool W8A8>
static int launch_decode(LayerArgs& a, int rows, cudaStream_t st) {
  if (!pick_blocks(rows, a.top, a.H, a.I, a.sh_qg != nullptr, a.CB, a.S, a.CBd)) return LMOE_ERR_UNSUPPORTED;
  a.n_gu = (int)(a.top * (a.I / a.CB));
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
