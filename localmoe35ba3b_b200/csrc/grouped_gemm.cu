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
// Layout ("swap AB"): the MMA's M side is 128 weight rows, its N side is the
// tile's routes (16..256, a multiple of 16), K streams in 64-wide stages.
//   A  int8 [128 x 64]  TMA  -> smem (4 stages)
//      bf16 [128 x 64]  dequant warps -> 128B-swizzled K-major smem (3 stages)
//   B  bf16 [256 x 64]  cp.async row gather x[pos[r]] -> same layout (3 stages)
//   D  fp32 [128 lanes x 256 columns] in tensor memory
// Warp roles (256 threads): w0 TMA producer, w1 TMEM owner + MMA issuer,
// w2-3 activation gather, w4-7 dequantisers and then the epilogue.
// Epilogue modes: PLAIN (y = round(acc)), SWIGLU (gate rows 0-63 and up
// rows 64-127 of the tile give hidden = round(round(silu(g)) * u), the
// reference's gpu_routes.py:74-75), WEIGHTED (v = round(round(acc) * w_route),
// the per-route product of prefill._reduce, prefill.py:45).
#include <mutex>

#include "common.cuh"
#include "gemm.cuh"
#include "routes.cuh"

namespace lmoe {

constexpr int kBM = 128;
constexpr int kBK = 64;
constexpr int kNS8 = 4;
constexpr int kNS = 3;
constexpr int kGemmThreads = 256;
constexpr int kMaxGroups = 32;  // K <= 4096
constexpr int kA8Bytes = kBM * kBK;
constexpr int kA16Bytes = kBM * kBK * 2;
constexpr int kBBytes = kTileRoutes * kBK * 2;
constexpr int kTmemCols = 256;

struct GemmParams {
  const void* x;         // activations [rows, K]
  int64_t K;
  const int32_t* pos;    // per route row: x row to read (nullptr: the route row itself)
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
  static constexpr int b = a16 + kNS * kA16Bytes;
  static constexpr int scale = b + kNS * kBBytes;
  static constexpr int pos = scale + kBM * kMaxGroups * 4;
  static constexpr int bars = pos + kTileRoutes * 4;
  static constexpr int nbars = 2 * kNS8 + 3 * kNS + 3;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int bytes = misc + 64;
  static constexpr int alloc = bytes + 1024;  // slack for 1024-byte alignment
};

template <int DT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    grouped_gemm_w8a16_kernel(const __grid_constant__ CUtensorMap tm_bank, const __grid_constant__ CUtensorMap tm_lo,
                              const __grid_constant__ CUtensorMap tm_hi, const GemmParams p) {
  using A = Act<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t s_base = smem_u32(smem);
  const uint32_t sA8 = s_base + GemmSmem::a8;
  const uint32_t sA16 = s_base + GemmSmem::a16;
  const uint32_t sB = s_base + GemmSmem::b;
  float* sScale = (float*)(smem + GemmSmem::scale);
  int32_t* sPos = (int32_t*)(smem + GemmSmem::pos);
  const uint32_t bar0 = s_base + GemmSmem::bars;
  uint32_t* sTmem = (uint32_t*)(smem + GemmSmem::misc);
  volatile int* sAbort = (volatile int*)(smem + GemmSmem::misc + 8);

  auto full8 = [&](int s) { return bar0 + 8u * s; };
  auto empty8 = [&](int s) { return bar0 + 8u * (kNS8 + s); };
  auto full16 = [&](int s) { return bar0 + 8u * (2 * kNS8 + s); };
  auto fullB = [&](int s) { return bar0 + 8u * (2 * kNS8 + kNS + s); };
  auto emptyAB = [&](int s) { return bar0 + 8u * (2 * kNS8 + 2 * kNS + s); };
  const uint32_t tmem_full = bar0 + 8u * (2 * kNS8 + 3 * kNS);
  const uint32_t epi_bar0 = tmem_full + 8u;  // epilogue rendezvous (128 threads, used once each)
  const uint32_t epi_bar1 = tmem_full + 16u;

  // ---------------------------------------------------------------- tile
  int expert = 0, start, count;
  if (p.tiles != nullptr) {
    if ((int)blockIdx.y >= p.hdr[kHdrNumTiles]) return;
    const Tile t = p.tiles[blockIdx.y];
    expert = t.expert;
    start = t.start;
    count = t.count;
  } else {
    start = (int)blockIdx.y * kTileRoutes;
    const int64_t left = p.dense_rows - start;
    count = left < kTileRoutes ? (int)left : kTileRoutes;
  }
  if (count <= 0) return;
  const bool shared = (p.tiles != nullptr) && expert == p.experts;
  const int nb = blockIdx.x;
  const bool swiglu = p.mode == kSwiGLU;
  const int64_t out_w = swiglu ? p.inter : p.N;      // output columns of one expert
  const int rows_per_block = swiglu ? 64 : kBM;        // output columns per CTA
  const int64_t col0 = (int64_t)nb * rows_per_block;
  if (col0 >= out_w) return;
  const int valid_cols = (out_w - col0) < rows_per_block ? (int)(out_w - col0) : rows_per_block;
  const int NT = (count + 15) & ~15;
  const int KB = (int)(p.K / kBK);
  const int G = (int)(p.K / kGroup);

  // A rows (tensor-map coordinates) and their scale rows
  const CUtensorMap* map_lo = shared ? &tm_lo : &tm_bank;
  const CUtensorMap* map_hi = shared ? (swiglu ? &tm_hi : &tm_lo) : &tm_bank;
  const float* scl_lo = shared ? p.s_lo : p.s_bank;
  const float* scl_hi = shared ? (swiglu ? p.s_hi : p.s_lo) : p.s_bank;
  const int64_t rmax_lo = shared ? p.rows_lo : p.rows_bank;
  const int64_t rmax_hi = shared ? (swiglu ? p.rows_hi : p.rows_lo) : p.rows_bank;
  const int64_t ebase = shared ? 0 : (int64_t)expert * p.N;
  int64_t row_lo, row_hi;
  if (swiglu) {
    row_lo = ebase + col0;
    row_hi = (shared ? 0 : ebase + p.inter) + col0;
  } else {
    row_lo = ebase + col0;
    row_hi = row_lo + 64;
  }

  const int warp = warp_id(), lane = lane_id();
  if (threadIdx.x == 0) {
    for (int s = 0; s < kNS8; ++s) {
      mbar_init(full8(s), 1);
      mbar_init(empty8(s), 128);
    }
    for (int s = 0; s < kNS; ++s) {
      mbar_init(full16(s), 128);
      mbar_init(fullB(s), 64);
      mbar_init(emptyAB(s), 1);
    }
    mbar_init(tmem_full, 1);
    mbar_init(epi_bar0, 128);
    mbar_init(epi_bar1, 128);
    *sAbort = 0;
    fence_mbar_init();
    prefetch_tmap(map_lo);
    prefetch_tmap(map_hi);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sTmem), kTmemCols);
    tmem_relinquish();
    tc_fence_before();
  }
  if (warp >= 4) {  // scales of this CTA's 128 weight rows
    const int r = threadIdx.x - 128;
    const int64_t gr = (r < 64) ? row_lo + r : row_hi + (r - 64);
    const float* sp = (r < 64) ? scl_lo : scl_hi;
    const int64_t rmax = (r < 64) ? rmax_lo : rmax_hi;
    for (int g = 0; g < G; ++g) sScale[r * kMaxGroups + g] = (gr < rmax) ? __ldg(sp + gr * G + g) : 0.f;
  } else if (warp >= 2) {  // gather rows of this tile
    for (int j = threadIdx.x - 64; j < NT; j += 64) {
      int src = 0;
      if (j < count) src = p.pos ? __ldg(p.pos + start + j) : start + j;
      sPos[j] = src;
    }
  }
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *sTmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      int issued = 0;
      for (int kb = 0; kb < KB; ++kb) {
        const int s8 = kb % kNS8;
        if (!mbar_wait(empty8(s8), ((kb / kNS8) & 1) ^ 1, sAbort, p.err)) break;
        mbar_arrive_expect_tx(full8(s8), kA8Bytes);
        tma_load_2d(sA8 + s8 * kA8Bytes, map_lo, full8(s8), kb * kBK, (int)row_lo);
        tma_load_2d(sA8 + s8 * kA8Bytes + kA8Bytes / 2, map_hi, full8(s8), kb * kBK, (int)row_hi);
        issued = kb + 1;
      }
      // never leave a bulk copy in flight into shared memory we are about to release
      for (int kb = max(0, issued - kNS8); kb < issued; ++kb) mbar_wait_drain(full8(kb % kNS8), (kb / kNS8) & 1, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(DT == LMOE_BF16 ? 1 : 0, kBM, NT);
      for (int kb = 0; kb < KB; ++kb) {
        const int s = kb % kNS;
        const uint32_t ph = (kb / kNS) & 1;
        if (!mbar_wait(full16(s), ph, sAbort, p.err)) break;
        if (!mbar_wait(fullB(s), ph, sAbort, p.err)) break;
        tc_fence_after();
        const uint64_t ad = sdesc_k_sw128(sA16 + s * kA16Bytes);
        const uint64_t bd = sdesc_k_sw128(sB + s * kBBytes);
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_f16(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (kb | kk) != 0);
        mma_commit(emptyAB(s));
      }
      mma_commit(tmem_full);
    }
    __syncwarp();
  } else if (warp < 4) {
    // ------------------------------------------------------------ activation gather
    const int b = threadIdx.x - 64;
    const int c = b & 7;
    const int r0 = b >> 3;
    const char* xb = (const char*)p.x;
    int done = 0;
    for (int kb = 0; kb < KB; ++kb) {
      const int s = kb % kNS;
      if (!mbar_wait(emptyAB(s), ((kb / kNS) & 1) ^ 1, sAbort, p.err)) break;
      const uint32_t dst = sB + s * kBBytes;
      for (int j = r0; j < NT; j += 8) {
        const bool v = j < count;
        const char* src = xb + ((int64_t)sPos[j] * p.K + (int64_t)kb * kBK + c * 8) * 2;
        cp_async16(dst + sw128_off(j, c), src, v ? 16u : 0u);
      }
      cp_async_commit();
      if (kb > 0) {
        cp_async_wait<1>();
        fence_proxy_async_smem();
        mbar_arrive(fullB((kb - 1) % kNS));
      }
      done = kb + 1;
    }
    cp_async_wait<0>();
    fence_proxy_async_smem();
    if (done > 0) mbar_arrive(fullB((done - 1) % kNS));
  } else {
    // ------------------------------------------------------------ dequantise
    const int d = threadIdx.x - 128;
    const int w = d >> 5;
    bool ok = true;
    for (int kb = 0; kb < KB && ok; ++kb) {
      const int s8 = kb % kNS8;
      const int s = kb % kNS;
      if (!mbar_wait(full8(s8), (kb / kNS8) & 1, sAbort, p.err)) { ok = false; break; }
      if (!mbar_wait(emptyAB(s), ((kb / kNS) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
      const int g = kb >> 1;
      const uint8_t* a8 = smem + GemmSmem::a8 + s8 * kA8Bytes;
      uint8_t* a16 = smem + GemmSmem::a16 + s * kA16Bytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int row = w * 32 + i * 8 + (lane >> 2);
        const int c = lane & 3;
        const uint4 v = *reinterpret_cast<const uint4*>(a8 + row * 64 + c * 16);
        const float sc = sScale[row * kMaxGroups + g];
        const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
        uint32_t o[8];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          float f0, f1, f2, f3;
          i8x4_to_f32(wv[j], f0, f1, f2, f3);
          o[2 * j] = A::pack(__fmul_rn(f0, sc), __fmul_rn(f1, sc));
          o[2 * j + 1] = A::pack(__fmul_rn(f2, sc), __fmul_rn(f3, sc));
        }
        *reinterpret_cast<uint4*>(a16 + sw128_off(row, 2 * c)) = make_uint4(o[0], o[1], o[2], o[3]);
        *reinterpret_cast<uint4*>(a16 + sw128_off(row, 2 * c + 1)) = make_uint4(o[4], o[5], o[6], o[7]);
      }
      mbar_arrive(empty8(s8));
      fence_proxy_async_smem();
      mbar_arrive(full16(s));
    }

    // ------------------------------------------------------------ epilogue
    // every epilogue thread takes the same path: the waits below ignore the
    // abort flag and are bounded, and the rendezvous are mbarriers, not bar.sync
    const bool have = mbar_wait_drain(tmem_full, 0, p.err);
    tc_fence_after();
    if (have) {
      const int q = w;  // TMEM lane quadrant of this warp (warps 4..7)
      const int row = q * 32 + lane;
      const uint32_t taddr = tmem + ((uint32_t)(q * 32) << 16);
      uint16_t* stg = (uint16_t*)(smem + GemmSmem::b);  // B stages are idle now
      typename A::T* y = (typename A::T*)p.y;
      if (!swiglu) {
        const bool weigh = (p.mode == kWeighted) && !shared;
        for (int c0 = 0; c0 < NT; c0 += 32) {
          uint32_t r[32];
          tmem_ld32(taddr + c0, r);
          tmem_ld_wait();
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int j = c0 + jj;
            if (j < count) {
              float v = A::round(__uint_as_float(r[jj]));
              if (weigh) v = A::round(__fmul_rn(v, __ldg(p.rweight + start + j)));
              stg[j * kBM + row] = A::bits(v);
            }
          }
        }
        mbar_arrive(epi_bar0);
        mbar_wait_drain(epi_bar0, 0, p.err);
        const bool vec = (valid_cols == kBM) && (p.ldy % 8 == 0) && (col0 % 8 == 0);
        for (int j = d >> 4; j < count; j += 8) {
          const int c8 = (d & 15) * 8;
          typename A::T* dst = y + (int64_t)(start + j) * p.ldy + col0 + c8;
          const uint16_t* src = stg + j * kBM + c8;
          if (vec) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
            for (int u = 0; u < 8; ++u)
              if (c8 + u < valid_cols) reinterpret_cast<uint16_t*>(dst)[u] = src[u];
          }
        }
      } else {
        uint16_t* stg_u = stg;                       // [NT][64] up values
        uint16_t* stg_h = stg + kTileRoutes * 64;    // [NT][64] hidden values
        if (q >= 2) {
          for (int c0 = 0; c0 < NT; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int j = c0 + jj;
              if (j < count) stg_u[j * 64 + (row - 64)] = A::bits(__uint_as_float(r[jj]));
            }
          }
        }
        mbar_arrive(epi_bar0);
        mbar_wait_drain(epi_bar0, 0, p.err);
        if (q < 2) {
          for (int c0 = 0; c0 < NT; c0 += 32) {
            uint32_t r[32];
            tmem_ld32(taddr + c0, r);
            tmem_ld_wait();
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int j = c0 + jj;
              if (j < count) {
                const float gt = A::round(__uint_as_float(r[jj]));
                const float up = A::lo_f((uint32_t)stg_u[j * 64 + row]);
                const float sl = A::round(__fdiv_rn(gt, __fadd_rn(1.0f, expf(-gt))));
                stg_h[j * 64 + row] = A::bits(__fmul_rn(sl, up));
              }
            }
          }
        }
        mbar_arrive(epi_bar1);
        mbar_wait_drain(epi_bar1, 0, p.err);
        const bool vec = (valid_cols == 64) && (p.ldy % 8 == 0) && (col0 % 8 == 0);
        for (int j = d >> 3; j < count; j += 16) {
          const int c8 = (d & 7) * 8;
          typename A::T* dst = y + (int64_t)(start + j) * p.ldy + col0 + c8;
          const uint16_t* src = stg_h + j * 64 + c8;
          if (vec) {
            *reinterpret_cast<uint4*>(dst) = *reinterpret_cast<const uint4*>(src);
          } else {
            for (int u = 0; u < 8; ++u)
              if (c8 + u < valid_cols) reinterpret_cast<uint16_t*>(dst)[u] = src[u];
          }
        }
      }
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

// int8 [rows, K] row-major, box = 64 rows x 64 bytes, no swizzle
static int make_int8_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K) {
  EncodeTiledFn fn = encode_fn();
  if (!fn) return LMOE_ERR_CUDA;
  if (((uintptr_t)base & 15) || (K % 16) || rows <= 0) return LMOE_ERR_INVALID;
  cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)K};
  cuuint32_t box[2] = {64, 64};
  cuuint32_t es[2] = {1, 1};
  CUresult r = fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, (void*)base, dims, strides, box, es,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? LMOE_OK : LMOE_ERR_CUDA;
}

int launch_grouped_gemm(const GemmLaunch& L, cudaStream_t st) {
  if (L.K % kGroup || L.K / kGroup > kMaxGroups || L.K <= 0) return LMOE_ERR_INVALID;
  if (L.grid_tiles <= 0) return LMOE_OK;
  CUtensorMap tb, tl, th;
  int rc = make_int8_map(&tb, L.q_bank, L.experts * L.N, L.K);
  if (rc) return rc;
  tl = tb;
  th = tb;
  if (L.q_lo) {
    if ((rc = make_int8_map(&tl, L.q_lo, L.rows_lo, L.K))) return rc;
  }
  if (L.q_hi) {
    if ((rc = make_int8_map(&th, L.q_hi, L.rows_hi, L.K))) return rc;
  }
  GemmParams p = {};
  p.x = L.x;
  p.K = L.K;
  p.pos = L.pos;
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
  const dim3 grid((unsigned)((out_w + per - 1) / per), (unsigned)L.grid_tiles);
  const size_t smem = GemmSmem::alloc;
  if (L.dtype == LMOE_BF16) {
    auto k = grouped_gemm_w8a16_kernel<LMOE_BF16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<grid, kGemmThreads, smem, st>>>(tb, tl, th, p);
  } else if (L.dtype == LMOE_F16) {
    auto k = grouped_gemm_w8a16_kernel<LMOE_F16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    k<<<grid, kGemmThreads, smem, st>>>(tb, tl, th, p);
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
  if (k / kGroup > kMaxGroups) return LMOE_ERR_UNSUPPORTED;
  GemmLaunch L = {};
  L.x = x;
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

extern "C" int lmoe_routed_linear(const void* x, const int8_t* q, const float* scale, int64_t experts, int64_t n,
                                  int64_t k, const void* meta, int64_t tokens, int64_t top, int gather, void* y,
                                  int dtype, int* err, void* stream) {
  if (!x || !q || !scale || !meta || !y || experts <= 0 || n <= 0 || k <= 0 || k % kGroup) return LMOE_ERR_INVALID;
  if (k / kGroup > kMaxGroups) return LMOE_ERR_UNSUPPORTED;
  const MetaLayout ML(tokens, top, experts);
  const char* m = (const char*)meta;
  GemmLaunch L = {};
  L.x = x;
  L.K = k;
  L.pos = gather ? (const int32_t*)(m + ML.off_pos) : nullptr;
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
  return launch_grouped_gemm(L, (cudaStream_t)stream);
}
