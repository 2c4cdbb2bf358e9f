// Tensor-core (tcgen05) W8A16 grouped GEMM for the routed experts, the shared
// expert and the dense INT8 linears.
//
// Replaces prefill._routed / gpu_routes._nonempty (qwen35_deploy/runtime/
// prefill.py:12-34, gpu_routes.py:39-44) and the large-M int8._linear
// (operators/int8.py:9-37).  Arithmetic follows the reference: every weight
// is dequantised as round_dtype(float(q) * scale) (int8.py:19-21, prefill.py:24-25)
// and multiplied into an fp32 accumulator; the output is stored in the
// activation dtype.
//
// Layout: the MMA's M side is a tile of 128 routes (token rows, already in
// route order after permute_rows_kernel), its N side is 128 weight rows of one
// expert, K streams in 64-wide MMA stages:
//   W  int8 [128 x 128] TMA -> 128B-swizzled smem ring (one scale group per
//                       stage: 128 contiguous bytes per weight row per request,
//                       which HBM streams near its peak)
//      bf16 [128 x 64]  dequant warps -> 128B-swizzled K-major smem (4 slots,
//                       filled in pairs: one int8 stage = two MMA stages); the
//                       MMA's B operand
//   X  bf16 [128 x 128] per stage, two 64-column chunks of 32-row TMA boxes
//                       covering the tile's routes, on one barrier (a warp's
//                       bulk copies stream at about one barrier stage per 0.4 us
//                       whatever their size) -> same layout (the MMA's A operand)
//   D  fp32 [128 token lanes x 128 weight columns] in tensor memory, 4 buffers
// so an epilogue thread owns one route row and finds that row's output
// columns contiguous in its tensor-memory lane: it stores 16-byte vectors,
// with no shuffles or shared-memory transposes.
// The kernel is persistent: one CTA per SM walks the (tile, column-block)
// work units in a fixed stride, so the epilogue of one unit overlaps the main
// loop of the next ones.
// Warp roles (512 threads): w0 + w3 weight TMA (alternate stages), w1 TMEM
// owner + MMA issuer, w2 activation TMA, w4-11 dequantisers, w12-15 epilogue.
// Epilogue modes: PLAIN (y = round(acc)), SWIGLU (gate columns 0-63 and up
// columns 64-127 of the unit give hidden = round(round(silu(g)) * u), the
// reference's gpu_routes.py:74-75), WEIGHTED (v = round(round(acc) * w_route),
// the per-route product of prefill._reduce, prefill.py:45).
// Every wait is bounded (LMOE_WAIT_NS); a timeout raises the CTA abort flag
// and the caller's error word, every role drains and the CTA exits.
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "routes.cuh"

namespace lmoe {

constexpr int kBM = 128;
constexpr int kBK = 64;    // MMA stage: one 128-byte swizzle atom of 16-bit K values
constexpr int kBK8 = 128;  // int8 stage: one scale group
constexpr int kNS8 = 4;    // int8 weight stages
constexpr int kNA = 4;     // bf16 weight slots (two pairs)
constexpr int kNS = 3;     // activation stages (one per int8 stage: K 128)
constexpr int kGemmThreads = 512;
constexpr int kDeqWarp0 = 4, kDeqWarps = 8;
constexpr int kEpiWarp0 = 12;
constexpr int kA8Bytes = kBM * kBK8;
constexpr int kA16Bytes = kBM * kBK * 2;
constexpr int kBBytes = kTileRoutes * kBK * 2;    // one 64-column chunk
constexpr int kBChunks = kBK8 / kBK;              // chunks per activation stage
constexpr int kBStage = kBChunks * kBBytes;
constexpr int kXBoxRows = 32;  // activation TMA box rows: a tile loads only the boxes covering its routes
constexpr int kTmemBufs = 4;                 // accumulator buffers
constexpr int kTmemCols = kTmemBufs * kBM;   // 4 x 128 fp32 columns
static_assert(kTileRoutes == 128, "the MMA M extent is the route tile");

struct GemmParams {
  int64_t K;
  const Tile* tiles;     // nullptr: dense mode
  const int32_t* hdr;    // tiles mode: hdr[kHdrNumTiles]
  int64_t dense_rows;    // dense mode: M
  int64_t N;             // rows of one expert's weight (PLAIN/WEIGHTED output width; SWIGLU: 2I)
  int64_t inter;         // SWIGLU: I
  int64_t rows_bank;     // E * N (rows in the bank tensor map)
  int64_t rows_lo, rows_hi;
  const float* s_bank;   // [E*N, G]
  const float* s_lo;     // shared expert: gate (SWIGLU) or the whole matrix (PLAIN)
  const float* s_hi;     // shared expert: up (SWIGLU)
  int experts;           // tiles with expert == experts read the shared tensors
  void* y;
  int64_t ldy;
  const float* rweight;  // WEIGHTED: weight of each route row
  int mode;
  int* err;
};

struct GemmSmem {
  static constexpr int a8 = 0;
  static constexpr int a16 = a8 + kNS8 * kA8Bytes;
  static constexpr int b = a16 + kNA * kA16Bytes;
  static constexpr int bars = b + kNS * kBStage;
  // full8, empty8 (kNS8 each); fullA, emptyA (one per slot pair); fullB, emptyB (kNS each);
  // tfull, tempty (kTmemBufs each); drain
  static constexpr int nbars = 2 * kNS8 + 2 * (kNA / 2) + 2 * kNS + 2 * kTmemBufs + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int bytes = misc + 64;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};
static_assert(GemmSmem::alloc <= 232448, "shared memory per block");
static_assert(kNS8 % 2 == 0, "two weight producers own alternate stages");

// A work unit: one tile of routes of one expert x one block of output columns.
struct Unit {
  int expert, start, count, nb;
  bool shared;
};

__device__ __forceinline__ bool get_unit(const GemmParams& p, int u, int nblocks, Unit& o) {
  const int t = u / nblocks;
  o.nb = u - t * nblocks;
  if (p.tiles != nullptr) {
    if (t >= p.hdr[kHdrNumTiles]) return false;
    const Tile tl = p.tiles[t];
    o.expert = tl.expert;
    o.start = tl.start;
    o.count = tl.count;
    o.shared = tl.expert == p.experts;
  } else {
    o.expert = 0;
    o.start = t * kTileRoutes;
    const int64_t left = p.dense_rows - o.start;
    if (left <= 0) return false;
    o.count = left < kTileRoutes ? (int)left : kTileRoutes;
    o.shared = false;
  }
  return o.count > 0;
}

// rows (tensor-map coordinates) of the unit's two 64-row halves
__device__ __forceinline__ void unit_rows(const GemmParams& p, const Unit& u, int64_t& lo, int64_t& hi) {
  const bool sw = p.mode == kSwiGLU;
  const int64_t ebase = u.shared ? 0 : (int64_t)u.expert * p.N;
  const int64_t col0 = (int64_t)u.nb * (sw ? 64 : kBM);
  lo = ebase + col0;
  hi = sw ? ((u.shared ? 0 : ebase + p.inter) + col0) : lo + 64;
}

// bounded wait by lane 0, result broadcast: keeps the warp's control flow uniform
__device__ __forceinline__ bool warp_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err) {
  int ok = 1;
  if (lane_id() == 0) ok = mbar_wait(bar, parity, abort, err) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

template <int DT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tm_bank, const __grid_constant__ CUtensorMap tm_lo,
                              const __grid_constant__ CUtensorMap tm_hi, const __grid_constant__ CUtensorMap tm_x,
                              const __grid_constant__ CUtensorMap tm_x128, const GemmParams p) {
  using A = Act<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sA8 = s_base + GemmSmem::a8;
  const uint32_t sA16 = s_base + GemmSmem::a16;
  const uint32_t sB = s_base + GemmSmem::b;
  const uint32_t bar0 = s_base + GemmSmem::bars;
  uint32_t* sTmem = (uint32_t*)(smem + GemmSmem::misc);
  volatile int* sAbort = (volatile int*)(smem + GemmSmem::misc + 8);

  constexpr int kPairs = kNA / 2;
  auto full8 = [&](int s) { return bar0 + 8u * s; };
  auto empty8 = [&](int s) { return bar0 + 8u * (kNS8 + s); };
  auto fullA = [&](int q) { return bar0 + 8u * (2 * kNS8 + q); };
  auto emptyA = [&](int q) { return bar0 + 8u * (2 * kNS8 + kPairs + q); };
  auto fullB = [&](int s) { return bar0 + 8u * (2 * kNS8 + 2 * kPairs + s); };
  auto emptyB = [&](int s) { return bar0 + 8u * (2 * kNS8 + 2 * kPairs + kNS + s); };
  auto tfull = [&](int b) { return bar0 + 8u * (2 * kNS8 + 2 * kPairs + 2 * kNS + b); };
  auto tempty = [&](int b) { return bar0 + 8u * (2 * kNS8 + 2 * kPairs + 2 * kNS + kTmemBufs + b); };
  const uint32_t drain = bar0 + 8u * (2 * kNS8 + 2 * kPairs + 2 * kNS + 2 * kTmemBufs);

  const bool swiglu = p.mode == kSwiGLU;
  const int64_t out_w = swiglu ? p.inter : p.N;
  const int cols_per_unit = swiglu ? 64 : kBM;
  const int nblocks = (int)((out_w + cols_per_unit - 1) / cols_per_unit);
  const int KB = (int)(p.K / kBK);    // MMA stages per unit
  const int KB8 = (int)(p.K / kBK8);  // int8 stages per unit (== scale groups)
  const int G = KB8;
  const int warp = warp_id(), lane = lane_id();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS8; ++s) {
      mbar_init(full8(s), 1);
      mbar_init(empty8(s), kDeqWarps);
    }
    for (int q = 0; q < kPairs; ++q) {
      mbar_init(fullA(q), kDeqWarps);
      mbar_init(emptyA(q), 1);
    }
    for (int s = 0; s < kNS; ++s) {
      mbar_init(fullB(s), 1);
      mbar_init(emptyB(s), 1);
    }
    for (int b = 0; b < kTmemBufs; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), 4);
    }
    mbar_init(drain, 1);
    *sAbort = 0;
    fence_mbar_init();
  }
  if ((warp == 0 || warp == 3) && lane == 0) {
    prefetch_tmap(&tm_bank);
    prefetch_tmap(&tm_lo);
    prefetch_tmap(&tm_hi);
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
  const uint32_t tmem = *sTmem;
  const int stride = gridDim.x;

  if (warp == 0 || warp == 3) {
    // ------------------------------------------------------------ weight TMA
    // two producer warps take alternate stages (one warp's bulk copies on
    // different barriers complete one after another); stage s always belongs
    // to warp (s & 1) since kNS8 is even
    if (lane == 0) {
      const int mine = warp == 3 ? 1 : 0;
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok; u += stride) {
        Unit un;
        if (!get_unit(p, u, nblocks, un)) break;
        int64_t rlo, rhi;
        unit_rows(p, un, rlo, rhi);
        const CUtensorMap* mlo = un.shared ? &tm_lo : &tm_bank;
        const CUtensorMap* mhi = un.shared ? (swiglu ? &tm_hi : &tm_lo) : &tm_bank;
        for (int kb = 0; kb < KB8; ++kb, ++it) {
          if ((it & 1) != mine) continue;
          const int s8 = it % kNS8;
          if (!mbar_wait(empty8(s8), ((it / kNS8) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(full8(s8), kA8Bytes);
          tma_load_2d(sA8 + s8 * kA8Bytes, mlo, full8(s8), kb * kBK8, (int)rlo);
          tma_load_2d(sA8 + s8 * kA8Bytes + kA8Bytes / 2, mhi, full8(s8), kb * kBK8, (int)rhi);
        }
      }
      // never leave a bulk copy in flight into shared memory that is about to be released
      for (int k = max(0, it - kNS8); k < it; ++k)
        if ((k & 1) == mine) mbar_wait_drain(full8(k % kNS8), (k / kNS8) & 1, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int it = 0, ia = 0, ui = 0;
      bool ok = true, issued = false;
      for (int u = blockIdx.x; ok; u += stride, ++ui) {
        Unit un;
        if (!get_unit(p, u, nblocks, un)) break;
        const uint32_t idesc = idesc_f16(DT == LMOE_BF16 ? 1 : 0, kTileRoutes, kBM);
        const int b = ui % kTmemBufs;
        if (!mbar_wait(tempty(b), ((ui / kTmemBufs) & 1) ^ 1, sAbort, p.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(b * kBM);
        for (int kb = 0; kb < KB && ok; kb += 2, ++ia) {
          // one int8 stage = the A slot pair (2q, 2q + 1) = MMA stages kb and kb + 1
          const int q = ia % kPairs;
          if (!mbar_wait(fullA(q), (ia / kPairs) & 1, sAbort, p.err)) { ok = false; break; }
          const int s = it % kNS;
          if (!mbar_wait(fullB(s), (it / kNS) & 1, sAbort, p.err)) { ok = false; break; }
          ++it;
          tc_fence_after();
#pragma unroll
          for (int h = 0; h < kBChunks; ++h) {
            // A = the route rows (activations), B = the dequantised weight rows
            const uint64_t wd = sdesc_k_sw128(sA16 + (2 * q + h) * kA16Bytes);
            const uint64_t xd = sdesc_k_sw128(sB + s * kBStage + h * kBBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_f16(dt, xd + (uint64_t)(kk * 2), wd + (uint64_t)(kk * 2), idesc, ((kb + h) | kk) != 0);
          }
          mma_commit(emptyB(s));
          mma_commit(emptyA(q));
          issued = true;
        }
        // also after an abort, so the epilogue's wait ends (a commit with no
        // MMA issued before it is not relied on to arrive)
        if (issued) mma_commit(tfull(b));
      }
      // every MMA issued by this thread completes before TMEM is released
      if (issued) {
        mma_commit(drain);
        mbar_wait_drain(drain, 0, p.err);
      }
    }
    __syncwarp();
  } else if (warp == 2) {
    // ------------------------------------------------------------ activation TMA
    if (lane == 0) {
      int it = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok; u += stride) {
        Unit un;
        if (!get_unit(p, u, nblocks, un)) break;
        for (int kb8 = 0; kb8 < KB8; ++kb8, ++it) {
          const int s = it % kNS;
          if (!mbar_wait(emptyB(s), ((it / kNS) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          // boxes of 32 route rows covering the tile: a small tile does not load 128
          // rows.  Rows of the MMA tile past those boxes keep older data and rows past
          // the tile belong to other tiles (or read as zeros past the tensor); none of
          // them is ever stored.  A nearly full tile takes one 128-row box per chunk
          // instead of four: a warp's bulk copies cost about the same per copy
          // whatever their size.
          const bool big = un.count > 3 * kXBoxRows;
          const int nbox = big ? 1 : (un.count + kXBoxRows - 1) / kXBoxRows;
          const uint32_t chunk_bytes = big ? (uint32_t)kBBytes : (uint32_t)(nbox * kXBoxRows * kBK * 2);
          mbar_arrive_expect_tx(fullB(s), kBChunks * chunk_bytes);
          for (int h = 0; h < kBChunks; ++h) {
            const uint32_t dst = sB + s * kBStage + h * kBBytes;
            const int kx = (kb8 * kBChunks + h) * kBK;
            if (big) {
              tma_load_2d(dst, &tm_x128, fullB(s), kx, un.start);
            } else {
              for (int i = 0; i < nbox; ++i)
                tma_load_2d(dst + i * (kXBoxRows * kBK * 2), &tm_x, fullB(s), kx, un.start + kXBoxRows * i);
            }
          }
        }
      }
      for (int k = max(0, it - kNS); k < it; ++k) mbar_wait_drain(fullB(k % kNS), (k / kNS) & 1, p.err);
    }
    __syncwarp();
  } else if (warp >= kDeqWarp0 && warp < kDeqWarp0 + kDeqWarps) {
    // ------------------------------------------------------------ dequantise
    // Thread (w, lane) converts 16-byte chunk c8 = lane & 7 (K values 16*c8 .. +15
    // of the stage) of rows rb + 4i (i = 0..3), rb = 16w + (lane >> 3).  Eight
    // lanes of a shared-memory phase read one whole 128-byte row: no bank
    // conflicts under the 128-byte swizzle.  Chunks 0-3 go to the pair's first
    // A slot (K 0..63), chunks 4-7 to the second; the two halves write their
    // 16-byte pieces in opposite order, so a phase's stores never share banks.
    const int w = warp - kDeqWarp0;
    const int c8 = lane & 7;
    const int hh = c8 >> 2, cc = c8 & 3;
    const int rb = w * 16 + (lane >> 3);
    int it8 = 0, ia = 0;
    bool ok = true;
    for (int u = blockIdx.x; ok; u += stride) {
      Unit un;
      if (!get_unit(p, u, nblocks, un)) break;
      int64_t rlo, rhi;
      unit_rows(p, un, rlo, rhi);
      // the thread's 16 rows lie in one 64-row half (one source tensor)
      const bool hi_half = rb >= 64;
      const float* sp = hi_half ? (un.shared ? (swiglu ? p.s_hi : p.s_lo) : p.s_bank) : (un.shared ? p.s_lo : p.s_bank);
      const int64_t rmax = hi_half ? (un.shared ? (swiglu ? p.rows_hi : p.rows_lo) : p.rows_bank)
                                   : (un.shared ? p.rows_lo : p.rows_bank);
      const int64_t g0 = hi_half ? rhi + (rb - 64) : rlo + rb;
      const float* ps[4];
      bool vr[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        vr[i] = g0 + 4 * i < rmax;
        ps[i] = sp + (g0 + 4 * i) * G;
      }
      // group scales, fetched two stages ahead of use
      float sc[4], sn[4], sm[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        sc[i] = vr[i] ? __ldg(ps[i]) : 0.f;
        sn[i] = (G > 1 && vr[i]) ? __ldg(ps[i] + 1) : 0.f;
        sm[i] = (G > 2 && vr[i]) ? __ldg(ps[i] + 2) : 0.f;
      }
      for (int g = 0; g < G; ++g, ++it8, ++ia) {
        if (g > 0) {
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            sc[i] = sn[i];
            sn[i] = sm[i];
            sm[i] = (g + 2 < G && vr[i]) ? __ldg(ps[i] + g + 2) : 0.f;
          }
        }
        const int s8 = it8 % kNS8;
        const int q = ia % kPairs;
        if (!warp_wait(full8(s8), (it8 / kNS8) & 1, sAbort, p.err)) { ok = false; break; }
        const uint32_t a8 = sA8 + s8 * kA8Bytes;
        uint4 v[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = rb + 4 * i;
          v[i] = lds128(a8 + (uint32_t)(r * 128 + ((c8 ^ (r & 7)) << 4)));
        }

        if (!warp_wait(emptyA(q), ((ia / kPairs) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
        const uint32_t a16 = sA16 + (uint32_t)((2 * q + hh) * kA16Bytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = rb + 4 * i;
          const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          uint32_t o[8];
          const uint64_t sc2 = splat2(sc[i]);
#pragma unroll
          for (int j = 0; j < 4; ++j) deq4<DT>(wv[j], sc2, o[2 * j], o[2 * j + 1]);
          const uint4 lo = make_uint4(o[0], o[1], o[2], o[3]), hi = make_uint4(o[4], o[5], o[6], o[7]);
          const uint32_t d0 = a16 + sw128_off(r, 2 * cc), d1 = a16 + sw128_off(r, 2 * cc + 1);
          // selects, not a branch: a divergent branch would issue each store twice
          // with half the lanes and double the shared-memory wavefronts
          sts128(hh ? d1 : d0, hh ? hi : lo);
          sts128(hh ? d0 : d1, hh ? lo : hi);
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(fullA(q));
        // The int8 slot is handed back only now, after the converted weights
        // were published.  Handing it back right after the loads (even with
        // the arrive made data-dependent on every loaded value) gave
        // run-to-run differences confined to weight-row pairs of single
        // dequantiser half-warps; this ordering gave none in repeated runs.
        if (lane == 0) mbar_arrive(empty8(s8));
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    // Thread (q, lane) owns TMEM lane tok = route row start + tok of the unit;
    // its columns are the unit's output columns col0 .. col0 + 127 (SWIGLU:
    // gate 0-63, up 64-127 for hidden columns col0 .. col0 + 63).
    const int q = warp - kEpiWarp0;  // TMEM lane quadrant (== warp % 4)
    const int tok = q * 32 + lane;
    typename A::T* y = (typename A::T*)p.y;
    const bool vec_ok = ((p.ldy & 7) == 0) && ((((uintptr_t)p.y) & 15) == 0);
    int ui = 0;
    for (int u = blockIdx.x;; u += stride, ++ui) {
      Unit un;
      if (!get_unit(p, u, nblocks, un)) break;
      const int b = ui % kTmemBufs;
      int okw = 1;
      if (lane == 0) okw = mbar_wait_drain(tfull(b), (ui / kTmemBufs) & 1, p.err) ? 1 : 0;
      const bool have = __shfl_sync(0xffffffffu, okw, 0) != 0;
      tc_fence_after();
      const uint32_t taddr = tmem + (uint32_t)(b * kBM) + ((uint32_t)(q * 32) << 16);
      const int64_t col0 = (int64_t)un.nb * cols_per_unit;
      const int valid_cols = (out_w - col0) < cols_per_unit ? (int)(out_w - col0) : cols_per_unit;
      const bool live = have && tok < un.count;
      typename A::T* yrow = y + (int64_t)(un.start + tok) * p.ldy + col0;
      const int nchunks = swiglu ? 2 : kBM / 32;
      float wt = 1.f;
      if (live && p.mode == kWeighted && !un.shared) wt = __ldg(p.rweight + un.start + tok);
      for (int c = 0; c < nchunks; ++c) {
        const int c0 = c * 32;
        uint32_t h[16];  // 32 output values, packed pairs
        if (swiglu) {
          uint32_t g[32], uu[32];
          tmem_ld32(taddr + c0, g);
          tmem_ld32(taddr + 64 + c0, uu);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float o[2];
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const float gv = A::round(__uint_as_float(g[2 * j + t]));
              const float up = A::round(__uint_as_float(uu[2 * j + t]));
              const float sl = A::round(__fdividef(gv, 1.0f + __expf(-gv)));
              o[t] = __fmul_rn(sl, up);
            }
            h[j] = A::pack(o[0], o[1]);
          }
        } else {
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            float o0 = A::round(__uint_as_float(r[2 * j])), o1 = A::round(__uint_as_float(r[2 * j + 1]));
            if (p.mode == kWeighted) {
              o0 = __fmul_rn(o0, wt);
              o1 = __fmul_rn(o1, wt);
            }
            h[j] = A::pack(o0, o1);
          }
        }
        if (c == nchunks - 1) {  // last TMEM read of this unit: hand the buffer back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty(b));
        }
        if (!live || c0 >= valid_cols) continue;
        if (vec_ok && c0 + 32 <= valid_cols) {
          uint4* dst = reinterpret_cast<uint4*>(yrow + c0);
#pragma unroll
          for (int v = 0; v < 4; ++v) dst[v] = make_uint4(h[4 * v], h[4 * v + 1], h[4 * v + 2], h[4 * v + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if (c0 + j < valid_cols)
              reinterpret_cast<uint16_t*>(yrow)[c0 + j] = (uint16_t)((h[j >> 1] >> (16 * (j & 1))) & 0xffffu);
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

// ============================================================================ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = (EncodeTiledFn)f;
  });
  return fn;
}

// int8 [rows, K] row-major, box = 64 rows x 128 bytes (one scale group), 128-byte swizzle
int make_int8_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 16) || rows <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {(cuuint32_t)kBK8, 64};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)base, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

// int8 [rows, K] with a 128-row x 128-byte, 128B-swizzled box (the W8A8 GEMM's tiles)
int make_i8_tile_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 128) || rows <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {128, 128};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)base, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

// gate_up bank [E, 2I, K] int8 viewed as [2E][I][K]: box 2 x 64 rows x 128 bytes, 128-byte
// swizzle -- the 64 gate rows and the matching 64 up rows of one output block in one copy
int make_int8_pair_map(CUtensorMap* m, const int8_t* base, int64_t experts, int64_t inter, int64_t K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 16) || experts <= 0 || inter <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)inter, (cuuint64_t)(2 * experts)};
  cuuint64_t strides[2] = {(cuuint64_t)K, (cuuint64_t)(inter * K)};
  cuuint32_t box[3] = {(cuuint32_t)kBK8, 64, 2};
  cuuint32_t es[3] = {1, 1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 3, (void*)base, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

// activations [rows, K] 16-bit, box of 64 rows x 64 elements (8 KB) with the
// 128-byte swizzle: the B operand's K-major UMMA layout
int make_act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int dtype, int box_rows) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 64) || rows <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)box_rows};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dtype == LMOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  (void*)base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

int launch_grouped_gemm(const GemmLaunch& L, cudaStream_t st) {
  if (L.K % kGroup || L.K <= 0) return LMOE_ERR_INVALID;
  if (L.grid_tiles <= 0) return LMOE_OK;
  CUtensorMap tb, tl, th, tx, tx128;
  int rc = make_int8_map(&tb, L.q_bank, L.experts * L.N, L.K);
  if (rc) return rc;
  tl = tb;
  th = tb;
  if (L.q_lo && (rc = make_int8_map(&tl, L.q_lo, L.rows_lo, L.K))) return rc;
  if (L.q_hi && (rc = make_int8_map(&th, L.q_hi, L.rows_hi, L.K))) return rc;
  if ((rc = make_act_map(&tx, L.x, L.x_rows, L.K, L.dtype, kXBoxRows))) return rc;
  if ((rc = make_act_map(&tx128, L.x, L.x_rows, L.K, L.dtype, kTileRoutes))) return rc;
  GemmParams p = {};
  p.K = L.K;
  p.tiles = L.tiles;
  p.hdr = L.hdr;
  p.dense_rows = L.dense_rows;
  p.N = L.N;
  p.inter = L.inter;
  p.rows_bank = L.experts * L.N;
  p.rows_lo = L.rows_lo;
  p.rows_hi = L.rows_hi;
  p.s_bank = L.s_bank;
  p.s_lo = L.s_lo;
  p.s_hi = L.s_hi;
  p.experts = (int)L.experts;
  p.y = L.y;
  p.ldy = L.ldy;
  p.rweight = L.rweight;
  p.mode = L.mode;
  p.err = L.err;
  const int64_t out_w = L.mode == kSwiGLU ? L.inter : L.N;
  const int per = L.mode == kSwiGLU ? 64 : kBM;
  const int64_t units = ((out_w + per - 1) / per) * L.grid_tiles;
  const int64_t sms = sm_count();
  const int64_t ctas = units < sms ? units : sms;
  const size_t smem = GemmSmem::alloc;
  if (L.dtype == LMOE_BF16) {
    auto k = grouped_gemm_w8a16_kernel<LMOE_BF16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<(unsigned)ctas, kGemmThreads, smem, st>>>(tb, tl, th, tx, tx128, p);
  } else if (L.dtype == LMOE_F16) {
    auto k = grouped_gemm_w8a16_kernel<LMOE_F16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<(unsigned)ctas, kGemmThreads, smem, st>>>(tb, tl, th, tx, tx128, p);
  } else {
    return LMOE_ERR_INVALID;
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

}  // namespace lmoe

using namespace lmoe;

int lmoe_dense_gemv_w8a16(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                          int64_t k, int dtype, cudaStream_t st);

extern "C" int lmoe_linear_w8a16(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                                 int64_t k, int dtype, int* err, void* stream) {
  if (!x || !q || !scale || !y || m < 0 || n <= 0 || k <= 0 || k % kGroup) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  if (m == 0) return LMOE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  // one row: the HBM-streaming GEMV; more rows: the TMEM-operand tensor-core kernel (weights
  // on the MMA's M side, the rows on its N side), else (n not a multiple of 128) the GEMV up
  // to 16 rows and the shared-memory-operand GEMM above
  if (m >= 2 && dense_ts_ok(m, n, k) && (((uintptr_t)x) & 15) == 0 && (((uintptr_t)y) & 15) == 0)
    return launch_dense_ts(x, q, scale, y, m, n, k, dtype, nullptr, 0, err, st);
  if (m <= 16) return lmoe_dense_gemv_w8a16(x, q, scale, y, m, n, k, dtype, st);
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
  L.mode = kPlain;
  L.dtype = dtype;
  L.err = err;
  return launch_grouped_gemm(L, st);
}

extern "C" int64_t lmoe_linear_w8a16_workspace_size(int64_t m, int64_t n, int64_t k) {
  if (m < 2 || n <= 0 || k <= 0) return 0;
  return dense_ts_workspace(m, n, k);
}

extern "C" int lmoe_linear_w8a16_ws(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                                    int64_t k, int dtype, void* ws, int64_t ws_bytes, int* err, void* stream) {
  if (!x || !q || !scale || !y || m < 0 || n <= 0 || k <= 0 || k % kGroup || ws_bytes < 0) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  if (m >= 2 && dense_ts_ok(m, n, k) && (((uintptr_t)x) & 15) == 0 && (((uintptr_t)y) & 15) == 0)
    return launch_dense_ts(x, q, scale, y, m, n, k, dtype, ws, ws_bytes, err, (cudaStream_t)stream);
  return lmoe_linear_w8a16(x, q, scale, y, m, n, k, dtype, err, stream);
}

extern "C" int64_t lmoe_routed_linear_workspace_size(int64_t tokens, int64_t top, int64_t k) {
  return MetaLayout::align(tokens * top * k * 2);
}

extern "C" int lmoe_routed_linear(const void* x, const int8_t* q, const float* scale, int64_t experts, int64_t n,
                                  int64_t k, const void* meta, int64_t tokens, int64_t top, int gather, void* y,
                                  int dtype, void* ws, int* err, void* stream) {
  if (!x || !q || !scale || !meta || !y || experts <= 0 || n <= 0 || k <= 0 || k % kGroup) return LMOE_ERR_INVALID;
  if (gather && !ws) return LMOE_ERR_INVALID;
  const MetaLayout ML(tokens, top, experts);
  const char* m = (const char*)meta;
  cudaStream_t st = (cudaStream_t)stream;
  const void* rows = x;
  if (gather) {  // route-order copy of the token rows, then a plain tiled GEMM
    int rc = launch_permute_rows(x, (const int32_t*)(m + ML.off_pos), ws, tokens * top, k, st);
    if (rc) return rc;
    rows = ws;
  }
  GemmLaunch L = {};
  L.x = rows;
  L.x_rows = tokens * top;
  L.K = k;
  L.tiles = (const Tile*)(m + ML.off_tiles);
  L.hdr = (const int32_t*)(m + ML.off_hdr);
  L.grid_tiles = ML.max_tiles;
  L.q_bank = q;
  L.s_bank = scale;
  L.experts = experts;
  L.N = n;
  L.y = y;
  L.ldy = n;
  L.mode = kPlain;
  L.dtype = dtype;
  L.err = err;
  return launch_grouped_gemm(L, st);
}
