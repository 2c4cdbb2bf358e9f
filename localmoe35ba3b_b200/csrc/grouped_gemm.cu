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
// Layout ("swap AB"): the MMA's M side is 128 weight rows, its N side is a
// tile's routes (16..256, a multiple of 16), K streams in 64-wide MMA stages.
//   A  int8 [128 x 128] TMA -> 128B-swizzled smem ring (3 stages of one scale
//                       group each: 128 contiguous bytes per weight row per
//                       request, which HBM streams near its peak; 64-byte
//                       pieces reach well under half of it)
//      bf16 [128 x 64]  dequant warps -> 128B-swizzled K-major smem (4 slots,
//                       filled in pairs: one int8 stage = two MMA stages)
//   B  bf16 [NT x 64]   TMA tiles of 64 consecutive rows -> same layout (3 stages);
//                       routed rows are consecutive because the activations are
//                       permuted into route order first (permute_rows_kernel)
//   D  fp32 [128 lanes x 256 cols] in tensor memory, two buffers
// The kernel is persistent: one CTA per SM walks the (tile, column-block)
// work units in a fixed stride, so the epilogue of one unit overlaps the
// main loop of the next (the MMA issuer alternates TMEM buffers).
// Warp roles (512 threads): w0 weight TMA, w1 TMEM owner + MMA issuer,
// w2 activation TMA, w3 idle, w4-11 dequantisers, w12-15 epilogue.
// Activations: row r of a unit is x[start + r] (no gather inside the GEMM).
// Epilogue modes: PLAIN (y = round(acc)), SWIGLU (gate rows 0-63 and up rows
// 64-127 of the unit give hidden = round(round(silu(g)) * u), the reference's
// gpu_routes.py:74-75), WEIGHTED (v = round(round(acc) * w_route), the
// per-route product of prefill._reduce, prefill.py:45).
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
constexpr int kNS8 = 3;    // int8 stages
constexpr int kNA = 4;     // bf16 A slots (two pairs)
constexpr int kNS = 3;     // activation stages
constexpr int kGemmThreads = 512;
constexpr int kDeqWarp0 = 4, kDeqWarps = 8;
constexpr int kEpiWarp0 = 12;
constexpr int kA8Bytes = kBM * kBK8;
constexpr int kA16Bytes = kBM * kBK * 2;
constexpr int kBBytes = kTileRoutes * kBK * 2;
constexpr int kTmemCols = 512;   // two 256-column accumulators
constexpr int kStageTok = 32;    // epilogue chunk (tokens)
constexpr int kStgBytes = kStageTok * kBM * 2;

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
  static constexpr int stg = b + kNS * kBBytes;
  static constexpr int bars = stg + 2 * kStgBytes;
  // full8, empty8 (kNS8 each); fullA, emptyA (one per slot pair); fullB, emptyB (kNS each);
  // tfull, tempty (2 each); drain
  static constexpr int nbars = 2 * kNS8 + 2 * (kNA / 2) + 2 * kNS + 4 + 1;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int bytes = misc + 64;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};
static_assert(GemmSmem::alloc <= 232448, "shared memory per block");

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
                              const GemmParams p) {
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
  auto tempty = [&](int b) { return bar0 + 8u * (2 * kNS8 + 2 * kPairs + 2 * kNS + 2 + b); };
  const uint32_t drain = bar0 + 8u * (2 * kNS8 + 2 * kPairs + 2 * kNS + 4);

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
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), 4);
    }
    mbar_init(drain, 1);
    *sAbort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_bank);
    prefetch_tmap(&tm_lo);
    prefetch_tmap(&tm_hi);
  }
  if (warp == 2 && lane == 0) prefetch_tmap(&tm_x);
  if (warp == 1) {
    tmem_alloc(smem_u32(sTmem), kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;
  const int stride = gridDim.x;

  if (warp == 0) {
    // ------------------------------------------------------------ weight TMA
    if (lane == 0) {
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
          const int s8 = it % kNS8;
          if (!mbar_wait(empty8(s8), ((it / kNS8) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(full8(s8), kA8Bytes);
          tma_load_2d(sA8 + s8 * kA8Bytes, mlo, full8(s8), kb * kBK8, (int)rlo);
          tma_load_2d(sA8 + s8 * kA8Bytes + kA8Bytes / 2, mhi, full8(s8), kb * kBK8, (int)rhi);
        }
      }
      // never leave a bulk copy in flight into shared memory that is about to be released
      for (int k = max(0, it - kNS8); k < it; ++k) mbar_wait_drain(full8(k % kNS8), (k / kNS8) & 1, p.err);
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
        const int NT = (un.count + 15) & ~15;
        const uint32_t idesc = idesc_f16(DT == LMOE_BF16 ? 1 : 0, kBM, NT);
        const int b = ui & 1;
        if (!mbar_wait(tempty(b), ((ui >> 1) & 1) ^ 1, sAbort, p.err)) break;
        tc_fence_after();
        const uint32_t dt = tmem + (uint32_t)(b * 256);
        for (int kb = 0; kb < KB && ok; kb += 2, ++ia) {
          // one int8 stage = the A slot pair (2q, 2q + 1) = MMA stages kb and kb + 1
          const int q = ia % kPairs;
          if (!mbar_wait(fullA(q), (ia / kPairs) & 1, sAbort, p.err)) { ok = false; break; }
          for (int h = 0; h < 2; ++h, ++it) {
            const int s = it % kNS;
            if (!mbar_wait(fullB(s), (it / kNS) & 1, sAbort, p.err)) { ok = false; break; }
            tc_fence_after();
            const uint64_t ad = sdesc_k_sw128(sA16 + (2 * q + h) * kA16Bytes);
            const uint64_t bd = sdesc_k_sw128(sB + s * kBBytes);
#pragma unroll
            for (int kk = 0; kk < kBK / 16; ++kk)
              mma_f16(dt, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, ((kb + h) | kk) != 0);
            mma_commit(emptyB(s));
            issued = true;
          }
          if (ok) mma_commit(emptyA(q));
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
        const int nbox = (un.count + 63) / 64;  // 64-row boxes covering the unit's NT rows
        for (int kb = 0; kb < KB; ++kb, ++it) {
          const int s = it % kNS;
          if (!mbar_wait(emptyB(s), ((it / kNS) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(fullB(s), (uint32_t)nbox * 8192u);
          const uint32_t dst = sB + s * kBBytes;
          for (int i = 0; i < nbox; ++i) tma_load_2d(dst + i * 8192, &tm_x, fullB(s), kb * kBK, un.start + 64 * i);
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
        __syncwarp();
        if (lane == 0) mbar_arrive(empty8(s8));
        if (!warp_wait(emptyA(q), ((ia / kPairs) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
        const uint32_t a16 = sA16 + (uint32_t)((2 * q + hh) * kA16Bytes);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = rb + 4 * i;
          const uint32_t wv[4] = {v[i].x, v[i].y, v[i].z, v[i].w};
          uint32_t o[8];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float f0, f1, f2, f3;
            i8x4_to_f32(wv[j], f0, f1, f2, f3);
            o[2 * j] = A::pack(__fmul_rn(f0, sc[i]), __fmul_rn(f1, sc[i]));
            o[2 * j + 1] = A::pack(__fmul_rn(f2, sc[i]), __fmul_rn(f3, sc[i]));
          }
          const uint4 lo = make_uint4(o[0], o[1], o[2], o[3]), hi = make_uint4(o[4], o[5], o[6], o[7]);
          const uint32_t d0 = a16 + sw128_off(r, 2 * cc), d1 = a16 + sw128_off(r, 2 * cc + 1);
          if (hh == 0) {
            sts128(d0, lo);
            sts128(d1, hi);
          } else {
            sts128(d1, hi);
            sts128(d0, lo);
          }
        }
        fence_proxy_async_smem();
        __syncwarp();
        if (lane == 0) mbar_arrive(fullA(q));
      }
    }
  } else if (warp >= kEpiWarp0) {
    // ------------------------------------------------------------ epilogue
    const int q = warp - kEpiWarp0;              // TMEM lane quadrant (== warp % 4)
    const int e = threadIdx.x - kEpiWarp0 * 32;  // 0..127
    const int row = q * 32 + lane;               // weight row of this thread in the unit
    typename A::T* y = (typename A::T*)p.y;
    uint16_t* stg0 = (uint16_t*)(smem + GemmSmem::stg);
    volatile uint32_t* sHave = (volatile uint32_t*)(sTmem + 1);
    int ui = 0, chunk_ctr = 0;
    for (int u = blockIdx.x;; u += stride, ++ui) {
      Unit un;
      if (!get_unit(p, u, nblocks, un)) break;
      const int b = ui & 1;
      // one thread waits (bounded); the group follows through a named barrier,
      // so all 128 threads take the same path
      if (e == 0) *sHave = mbar_wait_drain(tfull(b), (ui >> 1) & 1, p.err) ? 1u : 0u;
      named_barrier(1, 128);
      const bool have = *sHave != 0;
      named_barrier(1, 128);
      tc_fence_after();
      const int NT = (un.count + 15) & ~15;
      const int64_t col0 = (int64_t)un.nb * cols_per_unit;
      const int valid_cols = (out_w - col0) < cols_per_unit ? (int)(out_w - col0) : cols_per_unit;
      const uint32_t taddr = tmem + (uint32_t)(b * 256) + ((uint32_t)(q * 32) << 16);
      const bool weigh = (p.mode == kWeighted) && !un.shared;
      for (int c0 = 0; c0 < NT; c0 += kStageTok, ++chunk_ctr) {
        uint16_t* stg = stg0 + (chunk_ctr & 1) * (kStgBytes / 2);
        uint32_t r[32];
        tmem_ld32(taddr + c0, r);
        tmem_ld_wait();
        if (c0 + kStageTok >= NT) {  // last TMEM read of this unit: hand the buffer back
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive(tempty(b));
        }
        if (have) {
          float wl = 1.f;
          if (weigh && c0 + lane < un.count) wl = __ldg(p.rweight + un.start + c0 + lane);
          // stage [token][row] in the activation dtype
#pragma unroll
          for (int jj = 0; jj < kStageTok; ++jj) {
            float v = A::round(__uint_as_float(r[jj]));
            if (weigh) v = A::round(__fmul_rn(v, __shfl_sync(0xffffffffu, wl, jj)));
            stg[jj * kBM + row] = A::bits(v);
          }
        }
        // the next chunk uses the other staging buffer, and the barrier of the
        // chunk after that orders its writes behind these reads
        named_barrier(1, 128);
        if (have) {
          const int ntok = min(kStageTok, un.count - c0);
          if (!swiglu) {
            // 4 threads per token row, 32 columns (64 B) each
            const int j = e >> 2, cb = (e & 3) * 32;
            if (j < ntok) {
              typename A::T* dst = y + (int64_t)(un.start + c0 + j) * p.ldy + col0 + cb;
              const uint16_t* src = stg + j * kBM + cb;
              if (valid_cols == kBM && (p.ldy % 8) == 0) {
#pragma unroll
                for (int v = 0; v < 4; ++v)
                  reinterpret_cast<uint4*>(dst)[v] = reinterpret_cast<const uint4*>(src)[v];
              } else {
                for (int v = 0; v < 32; ++v)
                  if (cb + v < valid_cols) reinterpret_cast<uint16_t*>(dst)[v] = src[v];
              }
            }
          } else {
            // hidden = round(round(silu(gate)) * up): 4 threads per token, 16 columns each
            const int j = e >> 2, cb = (e & 3) * 16;
            if (j < ntok) {
              uint32_t hv[8];
#pragma unroll
              for (int v = 0; v < 8; ++v) {
                float h2[2];
#pragma unroll
                for (int t = 0; t < 2; ++t) {
                  const int col = cb + 2 * v + t;
                  const float g = A::lo_f((uint32_t)stg[j * kBM + col]);
                  const float up = A::lo_f((uint32_t)stg[j * kBM + 64 + col]);
                  const float sl = A::round(__fdividef(g, 1.0f + __expf(-g)));
                  h2[t] = __fmul_rn(sl, up);
                }
                hv[v] = A::pack(h2[0], h2[1]);
              }
              typename A::T* dst = y + (int64_t)(un.start + c0 + j) * p.ldy + col0 + cb;
              if (valid_cols == 64 && (p.ldy % 8) == 0) {
                reinterpret_cast<uint4*>(dst)[0] = make_uint4(hv[0], hv[1], hv[2], hv[3]);
                reinterpret_cast<uint4*>(dst)[1] = make_uint4(hv[4], hv[5], hv[6], hv[7]);
              } else {
                for (int v = 0; v < 16; ++v)
                  if (cb + v < valid_cols)
                    reinterpret_cast<uint16_t*>(dst)[v] = (uint16_t)((hv[v >> 1] >> (16 * (v & 1))) & 0xffffu);
              }
            }
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

// ============================================================================ host
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

static EncodeTiledFn encode_fn() {
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
static int make_int8_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K) {
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

// activations [rows, K] 16-bit, box of 64 rows x 64 elements (8 KB) with the
// 128-byte swizzle: the B operand's K-major UMMA layout
static int make_act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int dtype) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 64) || rows <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K * 2};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, dtype == LMOE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2,
                  (void*)base, dims, strides, box, es, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_128B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

static int sm_count() {
  int dev = 0, n = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 148;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) return 148;
  return n;
}

int launch_grouped_gemm(const GemmLaunch& L, cudaStream_t st) {
  if (L.K % kGroup || L.K <= 0) return LMOE_ERR_INVALID;
  if (L.grid_tiles <= 0) return LMOE_OK;
  CUtensorMap tb, tl, th, tx;
  int rc = make_int8_map(&tb, L.q_bank, L.experts * L.N, L.K);
  if (rc) return rc;
  tl = tb;
  th = tb;
  if (L.q_lo && (rc = make_int8_map(&tl, L.q_lo, L.rows_lo, L.K))) return rc;
  if (L.q_hi && (rc = make_int8_map(&th, L.q_hi, L.rows_hi, L.K))) return rc;
  if ((rc = make_act_map(&tx, L.x, L.x_rows, L.K, L.dtype))) return rc;
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
    k<<<(unsigned)ctas, kGemmThreads, smem, st>>>(tb, tl, th, tx, p);
  } else if (L.dtype == LMOE_F16) {
    auto k = grouped_gemm_w8a16_kernel<LMOE_F16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<(unsigned)ctas, kGemmThreads, smem, st>>>(tb, tl, th, tx, p);
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
