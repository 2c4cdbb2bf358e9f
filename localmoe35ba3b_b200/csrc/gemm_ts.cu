// gate_up of the routed experts (+ the shared expert) with the fused SwiGLU
// epilogue, on tcgen05 MMAs whose A operand -- the dequantised weights --
// lives in tensor memory.
//
// Replaces prefill._routed for gate_up plus the SiLU*up step
// (qwen35_deploy/runtime/prefill.py:12-34, gpu_routes.py:39-44 and :74-75).
// Arithmetic as the reference: w = round_dtype(float(q) * scale)
// (int8.py:19-21, prefill.py:24-25) into an fp32 accumulator;
// hidden = round(round(silu(round(gate))) * round(up)).
//
// Layout: the MMA's M side is 128 weight rows of one expert (64 gate rows and
// the matching 64 up rows), its N side is a tile of <= 128 routes rounded up to
// 16, K streams in 128-wide int8 stages (one scale group).
//   W  int8 [128 x 128]  TMA -> 128B-swizzled smem ring (4 stages, two
//                        producer warps)
//      bf16              dequant warps -> tensor memory (tcgen05.st): the MMA's
//                        A operand, 64 columns per stage; weights never pass
//                        through shared memory in 16-bit form
//   X  bf16 [N x 128]    two 64-column chunks per stage (TMA boxes of 32 route
//                        rows, or 128 for a full tile) -> 128B-swizzled smem:
//                        the MMA's B operand
//   MMA stage s (4 of them) = A slot s + X stage s, with one "ready" barrier
//   (dequantisers + the activation bytes) and one "freed" barrier (the MMAs'
//   commit), so the single MMA-issuing thread waits and commits once per stage
//   D  fp32 [128 lanes x 128 columns] in tensor memory, two buffers
// Shared-memory traffic per MAC is therefore the int8 tile (TMA write + one
// read) and the route rows (TMA write + the MMA's read), about half of what an
// MMA with both operands in shared memory needs; with N <= 128 the MMA time
// scales with the tile's routes, so small experts cost little beyond their
// weight stream.
// Warp roles (512 threads): w0 + w3 weight TMA (alternate stages), w1 TMEM
// owner + MMA issuer, w2 activation TMA, w4-11 dequantisers (warp w writes
// TMEM lanes of quadrant w % 4, K half (w - 4) / 4), w12-15 epilogue
// (quadrant w % 4; up rows in w12-13, gate rows and the SiLU math in w14-15,
// on other SMSPs than the MMA issuer w1).
// Every wait is bounded (LMOE_WAIT_NS); a timeout raises the CTA abort flag and
// the caller's error word, every role drains and the CTA exits.
#include "common.cuh"
#include "gemm.cuh"
#include "routes.cuh"

namespace lmoe {
namespace ts {

constexpr int kBM = 128;       // weight rows per unit: MMA M
constexpr int kBK8 = 128;      // int8 stage K (one scale group)
constexpr int kNS8 = 4;        // int8 stages
constexpr int kBKB = 64;       // activation chunk K (one 128-byte swizzle atom)
constexpr int kBChunks = kBK8 / kBKB;  // chunks per activation stage: one stage per int8 stage
constexpr int kNA = 4;         // MMA stages: tensor-memory A slot + shared-memory activation stage
constexpr int kBoxRows = 32;   // activation TMA box rows
constexpr int kThreads = 512;
constexpr int kConvWarps = 8;
constexpr int kA8Bytes = kBM * kBK8;              // 16 KB
constexpr int kBBytes = kTileRoutes * kBKB * 2;   // 16 KB per chunk
constexpr int kBStage = kBChunks * kBBytes;       // 32 KB per activation stage
constexpr int kAccCols = kTileRoutes;             // fp32 accumulator columns per buffer
constexpr int kACol0 = 2 * kAccCols;              // A slots follow the two accumulators
constexpr int kASlotCols = kBK8 / 2;              // 64 columns hold 128 16-bit K values
constexpr int kTmemCols = 512;
constexpr int kUPitch = 80;                       // bytes per up row in the exchange buffer
constexpr int kUBytes = 64 * kUPitch;             // [64 rows][32 routes] 16-bit, padded rows
constexpr int kHBytes = 32 * 64 * 2;              // [32 routes][64 columns] 16-bit
constexpr int kDPitch = 136;                      // down stage row: 128 columns + 8 of padding (16-bit)
constexpr int kDStageBytes = 32 * kDPitch * 2;    // down: [32 routes][136] 16-bit
static_assert(2 * kDStageBytes <= 2 * kUBytes + 2 * kHBytes, "down staging fits the gate_up exchange area");
static_assert(kACol0 + kNA * kASlotCols <= kTmemCols, "tensor memory budget");
static_assert(kNS8 % 2 == 0, "two weight producers own alternate stages");

struct Smem {
  static constexpr int a8 = 0;
  static constexpr int b = a8 + kNS8 * kA8Bytes;
  static constexpr int u = b + kNA * kBStage;
  static constexpr int h = u + 2 * kUBytes;
  static constexpr int wts = h + 2 * kHBytes;   // down: the unit's 128 routing weights (fp32)
  static constexpr int bars = wts + 128 * 4;
  // full8, empty8 (kNS8 each); ready, freed (kNA each); tfull, tempty (2 each); drain
  static constexpr int nbars = 2 * kNS8 + 2 * kNA + 4 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int bytes = misc + 64;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};
static_assert(Smem::alloc <= 232448, "shared memory per block");

struct Params {
  int64_t K;               // gate_up: hidden; down: I
  int64_t inter;           // gate_up: I (bank rows [0, I) gate, [I, 2I) up)
  int64_t rows_e;          // rows of one expert's weight: gate_up 2I, down hidden
  const Tile* tiles;
  const int32_t* hdr;
  int64_t rows_bank;       // experts * rows_e
  int64_t rows_sh;         // rows of the shared expert's tensor(s): I (gate, up) or hidden (down)
  const float* s_bank;     // [experts * rows_e, K/128]
  const float* s_g;        // shared gate (down: the shared down) scales
  const float* s_u;        // shared up scales
  const float* rweight;    // down: routing weight of each route row
  int experts;             // tiles with expert == experts are the shared expert
  void* y;                 // gate_up: hidden [rows, I]; down: weighted rows [rows, hidden]
  int64_t ldy;
  int* err;
  // dense linear (tiles == nullptr): tiles of <= 128 of the dense_rows rows, expert 0
  int64_t dense_rows;
  // split K: unit u covers K stages [ks * gs, min(G, (ks + 1) * gs)) of its tile and block,
  // ks = u % ksplit; with ksplit > 1 (down only) the epilogue stores the fp32 sums to
  // partial[ks][row][ldy] instead of y
  int ksplit;
  float* partial;
};

struct Unit {
  int start, count, nb, expert;
  int ks, g0, g1;  // K split and its stage range
  bool shared;
  int64_t rlo, rhi;  // tensor-map rows of the unit's two 64-row halves (gate_up: gate, up)
};

// Unit u = (route tile u / nblocks, output block u % nblocks): gate_up blocks are 64
// hidden columns (64 gate + the matching 64 up rows), down blocks 128 output columns
// (128 consecutive rows of the expert's down weight).
template <bool DOWN>
__device__ __forceinline__ bool get_unit(const Params& p, int u, int nblocks, Unit& o) {
  const int S = p.ksplit;
  o.ks = u % S;
  u /= S;
  const int t = u / nblocks;
  Tile tl;
  if (p.tiles == nullptr) {
    if ((int64_t)t * kTileRoutes >= p.dense_rows) return false;
    tl.expert = 0;
    tl.start = t * kTileRoutes;
    tl.count = (int)min((int64_t)kTileRoutes, p.dense_rows - (int64_t)t * kTileRoutes);
  } else {
    if (t >= p.hdr[kHdrNumTiles]) return false;
    tl = p.tiles[t];
  }
  const int G = (int)(p.K / kBK8), gs = (G + S - 1) / S;
  o.g0 = o.ks * gs;
  o.g1 = min(G, o.g0 + gs);
  o.nb = u - t * nblocks;
  o.expert = tl.expert;
  o.start = tl.start;
  o.count = tl.count;
  o.shared = tl.expert == p.experts;
  const int64_t ebase = o.shared ? 0 : (int64_t)tl.expert * p.rows_e;
  if (DOWN) {
    o.rlo = ebase + (int64_t)o.nb * 128;
    o.rhi = o.rlo + 64;
  } else {
    const int64_t col = (int64_t)o.nb * 64;
    o.rlo = ebase + col;
    o.rhi = (o.shared ? 0 : ebase + p.inter) + col;
  }
  return o.count > 0;
}

__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err) {
  int ok = 1;
  if (lane_id() == 0) ok = mbar_wait(bar, parity, abort, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// silu(g) = g / (1 + exp(-g)) with an IEEE round-to-nearest division, as the reference
// computes it in fp32 before rounding to the activation dtype.
__device__ __forceinline__ float silu_exact(float g) { return __fdiv_rn(g, __fadd_rn(1.0f, expf(-g))); }

// The same quotient without a data-dependent branch, so that the 32 SiLUs of an epilogue
// chunk overlap: P. Markstein's FMA correction ("Computation of elementary functions on the
// IBM RISC System/6000 processor", IBM J. Res. Dev. 34(1), 1990). The approximate reciprocal
// y of d is refined once (e = 1 - d*y, y += e*y), the quotient q = g*y is corrected by its
// exact residual r = g - d*q (one fma: q += r*y), and an exact quotient (r = 0) is kept as it
// is, which preserves the sign of a zero quotient.  silu_fast_ok bounds the inputs for which
// d = 1 + exp(-g) stays in [1, 2^116] and g is finite; there the result equals silu_exact bit
// for bit for every bf16 and fp16 input (checked on the GPU over all 65,536 values of each
// type by lmoe_selftest_silu); other inputs take silu_exact.
__device__ __forceinline__ bool silu_fast_ok(float g) { return g >= -80.f && g <= 3.0e38f; }
__device__ __forceinline__ float silu_fast(float g) {
  const float d = __fadd_rn(1.0f, expf(-g));
  float y;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(d));
  const float e = __fmaf_rn(-d, y, 1.0f);
  y = __fmaf_rn(e, y, y);
  const float q = __fmul_rn(g, y);
  const float r = __fmaf_rn(-d, q, g);
  return r == 0.f ? q : __fmaf_rn(r, y, q);
}

// DOWN = false: gate_up + SwiGLU; DOWN = true: down + routing weight.
template <int DT, bool DOWN>
__global__ void __launch_bounds__(kThreads, 1)
    grouped_ts_kernel(const __grid_constant__ CUtensorMap tm_bank, const __grid_constant__ CUtensorMap tm_g,
                      const __grid_constant__ CUtensorMap tm_u, const __grid_constant__ CUtensorMap tm_x,
                      const __grid_constant__ CUtensorMap tm_x128, const Params p) {
  using A = Act<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sA8 = s_base + Smem::a8;
  const uint32_t sB = s_base + Smem::b;
  const uint32_t bar0 = s_base + Smem::bars;
  uint32_t* sTmem = (uint32_t*)(smem + Smem::misc);
  volatile uint32_t* sHave = (volatile uint32_t*)(smem + Smem::misc + 4);
  volatile int* sAbort = (volatile int*)(smem + Smem::misc + 8);

  auto full8 = [&](int s) { return bar0 + 8u * s; };
  auto empty8 = [&](int s) { return bar0 + 8u * (kNS8 + s); };
  // MMA stage s: ready(s) completes when the 8 dequantiser warps have written A slot s
  // and the activation stage s has landed; freed(s) when the MMAs reading both are done
  auto ready = [&](int s) { return bar0 + 8u * (2 * kNS8 + s); };
  auto freed = [&](int s) { return bar0 + 8u * (2 * kNS8 + kNA + s); };
  auto tfull = [&](int b) { return bar0 + 8u * (2 * kNS8 + 2 * kNA + b); };
  auto tempty = [&](int b) { return bar0 + 8u * (2 * kNS8 + 2 * kNA + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * kNS8 + 2 * kNA + 4);

  const int nblocks = DOWN ? (int)(p.rows_e / 128) : (int)(p.inter / 64);
  const int G = (int)(p.K / kBK8);
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS8; ++s) {
      mbar_init(full8(s), 1);
      mbar_init(empty8(s), kConvWarps);
    }
    for (int s = 0; s < kNA; ++s) {
      mbar_init(ready(s), kConvWarps + 1);  // + the activation producer's expect-tx arrival
      mbar_init(freed(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), 4);
    }
    mbar_init(drain, 1);
    *sAbort = 0;
    fence_mbar_init();
  }
  if ((warp == 0 || warp == 3) && lane == 0) {
    prefetch_tmap(&tm_bank);
    prefetch_tmap(&tm_g);
    prefetch_tmap(&tm_u);
  }
  if (warp == 2 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_x128);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sTmem), kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();  // the next kernel's CTAs may take each SM as this kernel's CTA leaves it
  const uint32_t tmem = *sTmem;
  const int stride = gridDim.x;

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ weight TMA
    // two producer warps take alternate stages: one warp's bulk copies on
    // different barriers complete one after another (about one HBM latency
    // each), so a second warp doubles the weight stream; stage s always
    // belongs to warp (s & 1) since kNS8 is even
    if (lane == 0) {
      const int mine = warp == 3 ? 1 : 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok; u += stride) {
        Unit un;
        if (!get_unit<DOWN>(p, u, nblocks, un)) break;
        for (int g = un.g0; g < un.g1; ++g, ++it) {
          if ((it & 1) != mine) continue;
          const int s8 = it % kNS8;
          if (!mbar_wait(empty8(s8), ((it / kNS8) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(full8(s8), kA8Bytes);
          if (DOWN) {
            // 128 consecutive rows of one down weight: two 64-row boxes
            const CUtensorMap* m = un.shared ? &tm_g : &tm_bank;
            tma_load_2d(sA8 + s8 * kA8Bytes, m, full8(s8), g * kBK8, (int)un.rlo);
            tma_load_2d(sA8 + s8 * kA8Bytes + kA8Bytes / 2, m, full8(s8), g * kBK8, (int)un.rhi);
          } else if (un.shared) {
            tma_load_2d(sA8 + s8 * kA8Bytes, &tm_g, full8(s8), g * kBK8, (int)un.rlo);
            tma_load_2d(sA8 + s8 * kA8Bytes + kA8Bytes / 2, &tm_u, full8(s8), g * kBK8, (int)un.rhi);
          } else {
            // one box for both halves: the bank viewed as [2E][I][K], box 2 x 64 x 128 B at
            // (expert's gate half, 64 rows of block nb): the gate rows, then the up rows
            tma_load_3d(sA8 + s8 * kA8Bytes, &tm_bank, full8(s8), g * kBK8, un.nb * 64, 2 * un.expert);
          }
        }
      }
      for (int k = max(0, it - kNS8); k < it; ++k)
        if ((k & 1) == mine) mbar_wait_drain(full8(k % kNS8), (k / kNS8) & 1, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      // one thread issues every MMA: the issue path (about 70-90 cycles per MMA
      // plus each wait and commit) is this kernel's critical path, so a stage
      // costs one wait, 8 MMAs and one commit
      int it = 0, ui = 0;
      bool ok = true, issued = false;
      const uint64_t bd0 = sdesc_k_sw128(sB);
      for (int u = blockIdx.x; ok; u += stride, ++ui) {
        Unit un;
        if (!get_unit<DOWN>(p, u, nblocks, un)) break;
        const int NT = (un.count + 15) & ~15;
        const uint32_t idesc = idesc_f16(DT == LMOE_BF16 ? 1 : 0, kBM, NT);
        const int b = ui & 1;
        if (!mbar_wait(tempty(b), ((ui >> 1) & 1) ^ 1, sAbort, p.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(b * kAccCols);
        for (int g = un.g0; g < un.g1; ++g, ++it) {
          const int s = it % kNA;
          if (!mbar_wait(ready(s), (it / kNA) & 1, sAbort, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint32_t acol = tmem + (uint32_t)(kACol0 + s * kASlotCols);
          const uint64_t bd = bd0 + (uint64_t)((s * kBStage) >> 4);
#pragma unroll
          for (int h = 0; h < kBChunks; ++h)
#pragma unroll
            for (int kk = 0; kk < kBKB / 16; ++kk)
              mma_f16_ts(dt, acol + (uint32_t)(h * 32 + kk * 8), bd + (uint64_t)(((h * kBBytes) >> 4) + kk * 2), idesc,
                         (g != un.g0) || ((h | kk) != 0));
          mma_commit(freed(s));
          issued = true;
        }
        // also after an abort, so the epilogue's wait ends
        if (issued) mma_commit(tfull(b));
      }
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, p.err);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation TMA
    // the activation rows are the previous kernel's output (permute_rows_kernel for
    // gate_up, the gate_up kernel for down): this kernel may be launched before that
    // kernel ends, and only this role reads its output
    grid_dep_wait();
    if (lane == 0) {
      int ib = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok; u += stride) {
        Unit un;
        if (!get_unit<DOWN>(p, u, nblocks, un)) break;
        // boxes of 32 route rows covering the tile; rows past the tile are read
        // (other tiles' rows, or zeros past the tensor) but never stored
        // a full-height tile takes one 128-row box (larger boxes stream faster),
        // a smaller one the 32-row boxes covering its routes
        // one barrier per stage: a warp's bulk copies stream at about one barrier
        // stage per 0.4 us whatever their size, so both K chunks of the int8 stage
        // land on the same barrier
        const bool big = un.count > 3 * kBoxRows;
        const int nbox = big ? 1 : (un.count + kBoxRows - 1) / kBoxRows;
        const uint32_t bytes = kBChunks * (big ? (uint32_t)kBBytes : (uint32_t)(nbox * kBoxRows * kBKB * 2));
        for (int g = un.g0; g < un.g1; ++g, ++ib) {
          const int s = ib % kNA;
          if (!mbar_wait(freed(s), ((ib / kNA) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(ready(s), bytes);
          for (int h = 0; h < kBChunks; ++h) {
            const uint32_t dst = sB + s * kBStage + h * kBBytes;
            const int kx = (g * kBChunks + h) * kBKB;
            if (big) {
              tma_load_2d(dst, &tm_x128, ready(s), kx, un.start);
            } else {
              for (int i = 0; i < nbox; ++i)
                tma_load_2d(dst + i * (kBoxRows * kBKB * 2), &tm_x, ready(s), kx, un.start + kBoxRows * i);
            }
          }
        }
      }
      // never leave a bulk copy in flight into shared memory that is about to be
      // released: the last stages' ready phases also need the dequantisers'
      // arrivals, which come within microseconds (or, after an abort, the bounded
      // wait runs out)
      for (int k = max(0, ib - kNA); k < ib; ++k) mbar_wait_drain(ready(k % kNA), (k / kNA) & 1, p.err);
    }
    __syncwarp();
  } else if (warp >= 4 && warp < 4 + kConvWarps) {
    // ------------------------------------------------------------ dequantise into tensor memory
    // thread = weight row r of the unit (TMEM lane), K half kh of the stage:
    // 4 x 16-byte loads (8 lanes of a phase read 8 rows at 8 different 16-byte
    // positions under the swizzle: no bank conflicts), 64 products, one
    // 32-column tensor-memory store
    const int qd = warp & 3, kh = (warp - 4) >> 2;
    const int r = qd * 32 + lane;
    const uint32_t tl = tmem + ((uint32_t)(qd * 32) << 16);
    int it8 = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok; u += stride) {
      Unit un;
      if (!get_unit<DOWN>(p, u, nblocks, un)) break;
      // TMEM lanes 0-63 take the up rows (shared-memory rows 64-127 of the stage),
      // lanes 64-127 the gate rows (rows 0-63): the epilogue's SiLU work then runs
      // in warps 14-15, away from the MMA issuer's SMSP
      // (down: TMEM lane r = row r of the unit)
      const int srow = DOWN ? r : (r ^ 64);
      const bool up = !DOWN && srow >= 64;
      const int64_t grow = DOWN ? un.rlo + r : (up ? un.rhi : un.rlo) + (srow & 63);
      const int64_t rmax = un.shared ? p.rows_sh : p.rows_bank;
      const float* sp = (un.shared ? (up ? p.s_u : p.s_g) : p.s_bank) + grow * G;
      const bool valid = grow < rmax;
      float sc = valid ? __ldg(sp + un.g0) : 0.f;
      float sn = (un.g0 + 1 < un.g1 && valid) ? __ldg(sp + un.g0 + 1) : 0.f;
      float sm = (un.g0 + 2 < un.g1 && valid) ? __ldg(sp + un.g0 + 2) : 0.f;
      for (int g = un.g0; g < un.g1; ++g, ++it8) {
        const int s8 = it8 % kNS8;
        const int a = it8 % kNA;
        if (!warp_wait(full8(s8), (it8 / kNS8) & 1, sAbort, p.err)) { ok = false; break; }
        const uint32_t a8 = sA8 + s8 * kA8Bytes + srow * 128;
        uint4 v[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) v[j] = lds128(a8 + (uint32_t)(((kh * 4 + j) ^ (srow & 7)) << 4));
        if (!warp_wait(freed(a), ((it8 / kNA) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
        uint32_t o[32];
        const uint64_t sc2 = splat2(sc);
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const uint32_t wv[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
          for (int m = 0; m < 4; ++m) deq4<DT>(wv[m], sc2, o[j * 8 + 2 * m], o[j * 8 + 2 * m + 1]);
        }
        tmem_st32(tl + (uint32_t)(kACol0 + a * kASlotCols + kh * 32), o);
        tmem_st_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(ready(a));
          mbar_arrive(empty8(s8));
        }
        sc = sn;
        sn = sm;
        sm = (g + 3 < un.g1 && valid) ? __ldg(sp + g + 3) : 0.f;
      }
    }
  } else if (warp >= 12) {
    // ------------------------------------------------------------ epilogue
    // per 32-route chunk: the up warps (q = 0, 1: TMEM lanes 0-63) hand their
    // rounded values to the gate warps (q = 2, 3; same lane = same hidden column)
    // through shared memory; the gate warps form hidden, transpose it through
    // shared memory to [route][column] and store 16-byte row pieces
    const int q = warp - 12;
    const int row = q * 32 + lane;
    typename A::T* y = (typename A::T*)p.y;
    uint8_t* ubase = smem + Smem::u;
    uint8_t* hbase = smem + Smem::h;
    int ui = 0, chunk = 0;
    for (int u = blockIdx.x;; u += stride, ++ui) {
      Unit un;
      if (!get_unit<DOWN>(p, u, nblocks, un)) break;
      const int b = ui & 1;
      // down: this thread's route weight loads before the accumulator wait, so its
      // latency overlaps it (shared-expert rows are not weighted)
      float wrow = 1.f;
      if (DOWN && p.rweight != nullptr && !un.shared && row < un.count) wrow = __ldg(p.rweight + un.start + row);
      if (q == 0 && lane == 0) *sHave = mbar_wait_drain(tfull(b), (ui >> 1) & 1, p.err) ? 1u : 0u;
      named_barrier(1, 128);
      const bool have = *sHave != 0;
      if (DOWN) reinterpret_cast<float*>(smem + Smem::wts)[row] = wrow;  // the previous unit's reads are done
      named_barrier(1, 128);
      tc_fence_after();
      const int NT = (un.count + 15) & ~15;
      const int nch = (NT + 31) / 32;
      const uint32_t taddr = tmem + (uint32_t)(b * kAccCols) + ((uint32_t)(q * 32) << 16);
      const int64_t col0 = (int64_t)un.nb * (DOWN ? 128 : 64);
      for (int c = 0; c < nch; ++c, ++chunk) {
        uint32_t acc[32];
        tmem_ld32(taddr + (uint32_t)(c * 32), acc);
        tmem_ld_wait();
        if (c == nch - 1) {  // last tensor-memory read of this unit: hand the buffer back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty(b));
        }
        if (!have) continue;
        if constexpr (DOWN) {
          if (p.partial != nullptr) {
            // split K: this split's fp32 sums, route rows of ldy floats (a warp stores 32
            // consecutive columns of one route at a time)
            const int ntok = min(32, un.count - c * 32);
            float* dst = p.partial + ((int64_t)un.ks * p.dense_rows + un.start + c * 32) * p.ldy + col0 + row;
#pragma unroll
            for (int jj = 0; jj < 32; ++jj)
              if (jj < ntok) dst[(int64_t)jj * p.ldy] = __uint_as_float(acc[jj]);
            continue;
          }
          // lane = output column col0 + row of the unit; per route j of the chunk
          // v = round(round(acc) * w_route) (shared-expert rows: round(acc)), written
          // transposed to a [32 routes][128 columns] 16-bit stage, then 16-byte row
          // pieces: 128 threads = 32 routes x 4 pieces of 64 bytes
          uint16_t* st = reinterpret_cast<uint16_t*>(ubase + (chunk & 1) * kDStageBytes);
          const int ntok = min(32, un.count - c * 32);
          // the chunk's 32 routing weights from the unit's shared copy (broadcast reads)
          float w[32];
          const uint32_t wsrc = smem_u32(smem + Smem::wts) + (uint32_t)(c * 32 * 4);
#pragma unroll
          for (int jj = 0; jj < 32; jj += 4) {
            const uint4 t = lds128(wsrc + jj * 4);
            w[jj] = __uint_as_float(t.x);
            w[jj + 1] = __uint_as_float(t.y);
            w[jj + 2] = __uint_as_float(t.z);
            w[jj + 3] = __uint_as_float(t.w);
          }
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            float v = A::round(__uint_as_float(acc[jj]));
            if (p.rweight != nullptr && !un.shared) v = __fmul_rn(v, w[jj]);
            st[jj * kDPitch + row] = A::bits(v);
          }
          named_barrier(2, 128);
          const int tok = row >> 2, piece = row & 3;
          if (tok < ntok) {
            typename A::T* dst = y + (int64_t)(un.start + c * 32 + tok) * p.ldy + col0 + piece * 32;
            const uint32_t src = smem_u32(st) + (uint32_t)(tok * kDPitch * 2 + piece * 64);
#pragma unroll
            for (int k = 0; k < 4; ++k) reinterpret_cast<uint4*>(dst)[k] = lds128(src + k * 16);
          }
          continue;
        }
        uint8_t* ub = ubase + (chunk & 1) * kUBytes;
        uint8_t* hb = hbase + (chunk & 1) * kHBytes;
        const int hc = row & 63;  // hidden column of this lane
        if (q < 2) {
          uint32_t pk[16];
#pragma unroll
          for (int j = 0; j < 16; ++j) pk[j] = A::pack(__uint_as_float(acc[2 * j]), __uint_as_float(acc[2 * j + 1]));
#pragma unroll
          for (int k = 0; k < 4; ++k)
            sts128(smem_u32(ub + hc * kUPitch + k * 16), make_uint4(pk[4 * k], pk[4 * k + 1], pk[4 * k + 2], pk[4 * k + 3]));
        }
        named_barrier(2 + (q & 1), 64);
        if (q >= 2) {
          uint32_t uu[16];
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            const uint4 t = lds128(smem_u32(ub + hc * kUPitch + k * 16));
            uu[4 * k] = t.x;
            uu[4 * k + 1] = t.y;
            uu[4 * k + 2] = t.z;
            uu[4 * k + 3] = t.w;
          }
          uint16_t* hrow = reinterpret_cast<uint16_t*>(hb);
          // branch-free SiLU, 8 routes at a time (their latencies overlap), then (rarely) the
          // exact division for gate values outside silu_fast's range
#pragma unroll
          for (int j0 = 0; j0 < 32; j0 += 8) {
            float hv[8];
            bool slow = false;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const int jj = j0 + j;
              const float gv = A::round(__uint_as_float(acc[jj]));
              const float upv = (jj & 1) ? A::hi_f(uu[jj >> 1]) : A::lo_f(uu[jj >> 1]);
              slow |= !silu_fast_ok(gv);
              hv[j] = __fmul_rn(A::round(silu_fast(gv)), upv);
            }
            if (slow) {
#pragma unroll
              for (int j = 0; j < 8; ++j) {
                const int jj = j0 + j;
                const float gv = A::round(__uint_as_float(acc[jj]));
                const float upv = (jj & 1) ? A::hi_f(uu[jj >> 1]) : A::lo_f(uu[jj >> 1]);
                if (!silu_fast_ok(gv)) hv[j] = __fmul_rn(A::round(silu_exact(gv)), upv);
              }
            }
#pragma unroll
            for (int j = 0; j < 8; ++j) hrow[(j0 + j) * 64 + hc] = A::bits(hv[j]);
          }
          named_barrier(4, 64);
          // 64 threads: route e >> 1, columns (e & 1) * 32 .. + 31
          const int e = (q - 2) * 32 + lane;
          const int tok = e >> 1, half = e & 1;
          const int ntok = min(32, un.count - c * 32);
          if (tok < ntok) {
            typename A::T* dst = y + (int64_t)(un.start + c * 32 + tok) * p.ldy + col0 + half * 32;
#pragma unroll
            for (int k = 0; k < 4; ++k)
              reinterpret_cast<uint4*>(dst)[k] = lds128(smem_u32(hb + tok * 128 + half * 64 + k * 16));
          }
        }
      }
      if (!have) break;  // the MMA issuer gave up: stop instead of waiting on every later unit
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

}  // namespace ts

template <bool DOWN>
static int launch_ts(const GemmLaunch& L, cudaStream_t st) {
  if ((L.ldy % 8) != 0 || (((uintptr_t)L.y) & 15)) return LMOE_ERR_INVALID;
  if (L.grid_tiles <= 0) return LMOE_OK;
  CUtensorMap tb, tg, tu, tx, tx128;
  int rc = DOWN ? make_int8_map(&tb, L.q_bank, L.experts * L.N, L.K)
                : make_int8_pair_map(&tb, L.q_bank, L.experts, L.inter, L.K);
  if (rc) return rc;
  tg = tb;
  tu = tb;
  if (L.q_lo && (rc = make_int8_map(&tg, L.q_lo, L.rows_lo, L.K))) return rc;
  if (!DOWN && L.q_hi && (rc = make_int8_map(&tu, L.q_hi, L.rows_hi, L.K))) return rc;
  if ((rc = make_act_map(&tx, L.x, L.x_rows, L.K, L.dtype, ts::kBoxRows))) return rc;
  if ((rc = make_act_map(&tx128, L.x, L.x_rows, L.K, L.dtype, kTileRoutes))) return rc;
  ts::Params p = {};
  p.K = L.K;
  p.inter = DOWN ? 0 : L.inter;
  p.rows_e = L.N;
  p.tiles = L.tiles;
  p.hdr = L.hdr;
  p.rows_bank = L.experts * L.N;
  p.rows_sh = L.q_lo ? L.rows_lo : 0;
  p.s_bank = L.s_bank;
  p.s_g = L.s_lo;
  p.s_u = DOWN ? nullptr : L.s_hi;
  p.rweight = L.rweight;
  p.experts = (int)L.experts;
  p.y = L.y;
  p.ldy = L.ldy;
  p.err = L.err;
  p.dense_rows = L.tiles == nullptr ? L.dense_rows : 0;
  p.ksplit = L.ksplit > 1 ? L.ksplit : 1;
  p.partial = L.partial;
  const int64_t units = (DOWN ? L.N / 128 : L.inter / 64) * L.grid_tiles * p.ksplit;
  const int64_t sms = sm_count();
  const int64_t ctas = units < sms ? units : sms;
  const size_t smem = ts::Smem::alloc;
  // programmatic dependent launch: CTAs may start on SMs that the previous kernel's
  // CTAs have left (their weight streams start at once; the activation producer waits)
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)ctas);
  cfg.blockDim = dim3(ts::kThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (L.dtype == LMOE_BF16) {
    auto k = ts::grouped_ts_kernel<LMOE_BF16, DOWN>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, tb, tg, tu, tx, tx128, p));
  } else if (L.dtype == LMOE_F16) {
    auto k = ts::grouped_ts_kernel<LMOE_F16, DOWN>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(cudaLaunchKernelEx(&cfg, k, tb, tg, tu, tx, tx128, p));
  } else {
    return LMOE_ERR_INVALID;
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

int launch_swiglu_ts(const GemmLaunch& L, cudaStream_t st) {
  if (L.mode != kSwiGLU || L.tiles == nullptr) return LMOE_ERR_INVALID;
  if (L.K % kGroup || L.K <= 0 || L.inter % 64 || L.inter <= 0 || L.N != 2 * L.inter) return LMOE_ERR_INVALID;
  return launch_ts<false>(L, st);
}

namespace ts {
// every 16-bit pattern of the dtype as the gate value: count the inputs where the kernel's
// SiLU (silu_fast inside its range, silu_exact outside) differs from silu_exact (NaN = NaN)
template <int DT>
__global__ void selftest_silu_kernel(int* mismatches) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= 65536) return;
  const uint16_t b = (uint16_t)i;
  const float g = DT == LMOE_BF16 ? __uint_as_float((uint32_t)b << 16) : __half2float(__ushort_as_half(b));
  const float a = silu_exact(g);
  const float f = silu_fast_ok(g) ? silu_fast(g) : silu_exact(g);
  if (!(a != a && f != f) && __float_as_uint(a) != __float_as_uint(f)) atomicAdd(mismatches, 1);
}
}  // namespace ts

int selftest_silu(int dtype, int* mismatches, cudaStream_t st) {
  if (mismatches == nullptr) return LMOE_ERR_INVALID;
  if (dtype == LMOE_BF16) ts::selftest_silu_kernel<LMOE_BF16><<<256, 256, 0, st>>>(mismatches);
  else if (dtype == LMOE_F16) ts::selftest_silu_kernel<LMOE_F16><<<256, 256, 0, st>>>(mismatches);
  else return LMOE_ERR_INVALID;
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

int launch_down_ts(const GemmLaunch& L, cudaStream_t st) {
  if (L.mode != kWeighted || L.tiles == nullptr || L.rweight == nullptr || L.ksplit > 1) return LMOE_ERR_INVALID;
  if (L.K % kGroup || L.K <= 0 || L.N % 128 || L.N <= 0) return LMOE_ERR_INVALID;
  return launch_ts<true>(L, st);
}

}  // namespace lmoe

extern "C" int lmoe_selftest_silu(int dtype, int* mismatches, void* stream) {
  return lmoe::selftest_silu(dtype, mismatches, (cudaStream_t)stream);
}

// ============================================================================
// Dense W8A16 linear on the TMEM-operand kernel (the down kernel's geometry with no
// routing weight): y[m, n] = sum_k x[m, k] * round(q[n, k] * s[n, k/128]), the MMA's M
// side 128 weight rows, its N side up to 128 of the m rows, so that small m still
// streams the weights at full width.  When the (row tile, 128-column block) units are
// fewer than the SMs, K is split: each split stores fp32 sums to the workspace and
// dense_reduce_kernel adds the splits in order and rounds once.
namespace lmoe {
namespace {
// The split that minimises an estimate of the call's time: rounds of units on the busiest
// SM x (stages per unit + about one stage of per-unit fill and epilogue) x ~0.45 us per
// 128-K stage, plus the fp32 partial sums written and read back (8 bytes per output per
// split) at ~6 TB/s.  Every split is non-empty.
int dense_ksplit(int64_t m, int64_t n, int64_t k) {
  const int64_t units = ((m + kTileRoutes - 1) / kTileRoutes) * (n / 128);
  const int G = (int)(k / kGroup);
  const int64_t sms = sm_count();
  const double stage_us = 0.45, part_us_per_byte = 1.0 / 6.0e6;
  int best = 1;
  double best_cost = (double)((units + sms - 1) / sms) * (G + 1) * stage_us;
  for (int want = 2; want <= G; ++want) {
    const int gs = (G + want - 1) / want;
    const int S = (G + gs - 1) / gs;
    const double cost = (double)((units * S + sms - 1) / sms) * (gs + 1) * stage_us +
                        (double)S * (double)m * (double)n * 8.0 * part_us_per_byte;
    if (cost < best_cost) {
      best_cost = cost;
      best = S;
    }
  }
  return best;
}

template <int DT>
__global__ void __launch_bounds__(256) dense_reduce_kernel(const float* __restrict__ part, typename Act<DT>::T* y,
                                                           int64_t total, int splits) {
  grid_dep_wait();
  const int64_t i4 = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) * 4;
  if (i4 >= total) return;
  if (i4 + 4 <= total) {
    float4 acc = __ldcg(reinterpret_cast<const float4*>(part + i4));
    for (int s = 1; s < splits; ++s) {
      const float4 v = __ldcg(reinterpret_cast<const float4*>(part + (int64_t)s * total + i4));
      acc.x = __fadd_rn(acc.x, v.x);
      acc.y = __fadd_rn(acc.y, v.y);
      acc.z = __fadd_rn(acc.z, v.z);
      acc.w = __fadd_rn(acc.w, v.w);
    }
    uint2 o;
    o.x = Act<DT>::pack(acc.x, acc.y);
    o.y = Act<DT>::pack(acc.z, acc.w);
    *reinterpret_cast<uint2*>(y + i4) = o;
  } else {
    for (int64_t i = i4; i < total; ++i) {
      float acc = part[i];
      for (int s = 1; s < splits; ++s) acc = __fadd_rn(acc, part[(int64_t)s * total + i]);
      y[i] = Act<DT>::from_f(acc);
    }
  }
}
}  // namespace

bool dense_ts_ok(int64_t m, int64_t n, int64_t k) { return m >= 1 && n % 128 == 0 && n > 0 && k % kGroup == 0 && k > 0; }

int64_t dense_ts_workspace(int64_t m, int64_t n, int64_t k) {
  if (!dense_ts_ok(m, n, k)) return 0;
  const int S = dense_ksplit(m, n, k);
  return S > 1 ? (int64_t)S * m * n * 4 : 0;
}

int launch_dense_ts(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n, int64_t k,
                    int dtype, void* ws, int64_t ws_bytes, int* err, cudaStream_t st) {
  if (!dense_ts_ok(m, n, k) || (((uintptr_t)x) & 15) || (((uintptr_t)y) & 15) || (n % 8)) return LMOE_ERR_INVALID;
  int S = dense_ksplit(m, n, k);
  if (S > 1 && (ws == nullptr || ws_bytes < (int64_t)S * m * n * 4 || (((uintptr_t)ws) & 15))) S = 1;
  GemmLaunch L = {};
  L.x = x;
  L.x_rows = m;
  L.K = k;
  L.grid_tiles = (m + kTileRoutes - 1) / kTileRoutes;
  L.dense_rows = m;
  L.q_bank = q;
  L.s_bank = scale;
  L.experts = 1;
  L.N = n;
  L.y = y;
  L.ldy = n;
  L.mode = kWeighted;
  L.dtype = dtype;
  L.err = err;
  L.ksplit = S;
  L.partial = S > 1 ? (float*)ws : nullptr;
  int rc = launch_ts<true>(L, st);
  if (rc || S == 1) return rc;
  const int64_t total = m * n;
  const unsigned blocks = (unsigned)((total / 4 + 255) / 256 + 1);
  if (dtype == LMOE_BF16) {
    LMOE_CUDA_CHECK(launch_pdl(dense_reduce_kernel<LMOE_BF16>, dim3(blocks), dim3(256), 0, st, (const float*)ws,
                               (__nv_bfloat16*)y, total, S));
  } else {
    LMOE_CUDA_CHECK(launch_pdl(dense_reduce_kernel<LMOE_F16>, dim3(blocks), dim3(256), 0, st, (const float*)ws,
                               (__half*)y, total, S));
  }
  return LMOE_OK;
}
}  // namespace lmoe
