// The sparse-MoE block's router in one kernel: the logits GEMM on tcgen05 tensor cores
// and the router tail on the logits while they are still on chip.
//
// Replaces the HF Qwen3_5MoeTopKRouter.forward (transformers/models/qwen3_5_moe/
// modeling_qwen3_5_moe.py:762-770) that the reference keeps around its experts
// (qwen35_deploy/model.py:57-68): logits = F.linear(x, gate.weight) in the activation
// dtype (fp32 accumulation, rounded once), then softmax / top-k / renormalise
// (router_tail_row, the arithmetic of lmoe_router_topk).  For the prefill block the
// kernel also writes each 128-token tile's per-expert route counts, the first step of
// the routing metadata (meta_count_kernel's output), when a tile is exactly one
// metadata chunk (top * 128 == kMetaChunk).
//
// Two launches.  router_partial_kernel: per 128-token tile, kSplit CTAs each sum a
// quarter of K on tcgen05 (w0 TMA producer: the x tile [128 x 64] and the router weight
// [E x 64] per 64-wide K stage, 128B-swizzled, 4 stages; w1 TMEM owner and MMA issuer,
// M = 128 tokens, N = E experts, fp32 accumulators in E TMEM columns; w2-5 store each
// token's E fp32 sums to the workspace).  router_tail_kernel: per tile, the splits added
// in split order and rounded once (the logits), then the tail, 4 threads per token, and
// the tile's route counts.  Every wait is bounded.
#include "common.cuh"
#include "gemm.cuh"
#include "router_tail.cuh"
#include "routes.cuh"

namespace lmoe {
namespace rg {

constexpr int kGemmThreads = 192;   // w0 TMA, w1 TMEM + MMA, w2-5 epilogue
constexpr int kTailWarps = 4;       // tokens per CTA of the tail kernel, one warp each
constexpr int kStages = 4;
constexpr int kBK = 64;             // K per stage: one 128-byte swizzle atom of 16-bit values
constexpr int kTile = 128;          // tokens per tile: the MMA M extent
constexpr int kSplit = 4;           // K splits: CTAs per tile in the GEMM

template <int E>
struct Smem {
  static constexpr int a_bytes = kTile * kBK * 2;  // 16 KB
  static constexpr int b_bytes = E * kBK * 2;      // 32 KB at E = 256
  static constexpr int stage = a_bytes + b_bytes;
  static constexpr int data = kStages * stage;
  static constexpr int bars = data;                // full[kStages], empty[kStages], tfull
  static constexpr int misc = bars + (2 * kStages + 1) * 8;
  static constexpr int bytes = misc + 16;
  static constexpr int alloc = bytes + 1024;       // slack for 1024-byte alignment
};

struct Args {
  int64_t T, K;
  int top;
  float* part;      // [tiles][kSplit][kTile][E] fp32 partial sums (workspace)
  float* weights;
  int64_t* ids;
  float* probs;     // nullable: [T, E] fp32 softmax
  void* logits;     // nullable: [T, E] in the activation dtype
  int32_t* counts;  // nullable: per tile, E + 1 route counts (the last, invalid ids, is 0)
  int* err;
};

// CTA (tile, ks): the fp32 sums of x[tile] . w^T over K stages [ks * n, (ks + 1) * n).
template <int DT, int VPL>
__global__ void __launch_bounds__(kGemmThreads, 1)
    router_partial_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                          const Args p) {
  using S = Smem<VPL * 32>;
  constexpr int E = VPL * 32;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar0 = sb + S::bars;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (kStages + s); };
  const uint32_t tfull = bar0 + 8u * (2 * kStages);
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + S::misc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + S::misc + 4);
  const int warp = warp_id(), lane = lane_id();
  const int tile = blockIdx.x / kSplit, ks = blockIdx.x % kSplit;
  const int KS = (int)(p.K / kBK), per = (KS + kSplit - 1) / kSplit;
  const int g0 = ks * per, g1 = min(KS, g0 + per);
  const int64_t t0 = (int64_t)tile * kTile;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    mbar_init(tfull, 1);
    *sAbort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
  }
  if (p.counts != nullptr && ks == 0 && warp >= 2) {
    // the tile's route counts start at zero (the tail kernel adds to them); the previous
    // kernel may still read the metadata scratch they live in
    grid_dep_wait();
    for (int i = threadIdx.x - 64; i <= E; i += kGemmThreads - 64) p.counts[(int64_t)tile * (E + 1) + i] = 0;
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sTmem), E);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = *sTmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // x is the previous kernel's output, and the partial sums the previous call's tail
    // kernel read are about to be rewritten: wait for the previous kernel first
    grid_dep_wait();
    if (lane == 0) {
      int n = 0;
      for (int g = g0; g < g1; ++g, ++n) {
        const int s = n % kStages;
        if (!mbar_wait(empty(s), ((n / kStages) & 1) ^ 1, sAbort, p.err)) break;
        mbar_arrive_expect_tx(full(s), S::stage);
        const uint32_t dst = sb + (uint32_t)(s * S::stage);
        tma_load_2d(dst, &tm_x, full(s), g * kBK, (int)t0);
        tma_load_2d(dst + S::a_bytes, &tm_w, full(s), g * kBK, 0);
      }
      // never leave a load in flight when the CTA may exit (after an abort the MMAs may not
      // have consumed the last stages)
      for (int k = max(0, n - kStages); k < n; ++k) mbar_wait_drain(full(k % kStages), (k / kStages) & 1, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_f16(DT == LMOE_BF16 ? 1 : 0, kTile, E);
      bool issued = false;
      int n = 0;
      for (int g = g0; g < g1; ++g, ++n) {
        const int s = n % kStages;
        if (!mbar_wait(full(s), (n / kStages) & 1, sAbort, p.err)) break;
        tc_fence_after();
        const uint64_t ad = sdesc_k_sw128(sb + (uint32_t)(s * S::stage));
        const uint64_t bd = sdesc_k_sw128(sb + (uint32_t)(s * S::stage + S::a_bytes));
#pragma unroll
        for (int kk = 0; kk < kBK / 16; ++kk)
          mma_f16(tmem, ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, (n | kk) != 0);
        mma_commit(empty(s));
        issued = true;
      }
      // also after an abort, so that the epilogue's wait ends
      if (issued) mma_commit(tfull);
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // each thread: its token's (TMEM lane's) E fp32 sums to the workspace
    const int q = warp & 3;
    const int row = q * 32 + lane;
    int have = 1;
    if (lane == 0) have = mbar_wait_drain(tfull, 0, p.err) ? 1 : 0;
    have = __shfl_sync(0xffffffffu, have, 0);
    tc_fence_after();
    float* dst = p.part + (((int64_t)tile * kSplit + ks) * kTile + row) * E;
#pragma unroll 1
    for (int c = 0; c < E / 32; ++c) {
      uint32_t acc[32];
      tmem_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(c * 32), acc);
      tmem_ld_wait();
      if (have) {
#pragma unroll
        for (int j = 0; j < 8; ++j)
          reinterpret_cast<uint4*>(dst + c * 32)[j] = make_uint4(acc[4 * j], acc[4 * j + 1], acc[4 * j + 2], acc[4 * j + 3]);
      }
    }
    tc_fence_before();
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, E);
  }
}

// One warp per token (4 tokens per CTA): the token's kSplit partial sums added in split
// order and rounded to the activation dtype (its logits), then router_tail_row on them --
// lmoe_router_topk's tail, the same code -- and one route count per selected expert added
// to its tile's counts (zeroed by the tile's first GEMM CTA).
template <int DT, int VPL>
__global__ void __launch_bounds__(kTailWarps * 32) router_tail_kernel(const Args p) {
  using A = Act<DT>;
  constexpr int E = VPL * 32;
  __shared__ typename A::T s_row[kTailWarps][E];
  const int warp = warp_id(), lane = lane_id();
  const int64_t t = (int64_t)blockIdx.x * kTailWarps + warp;
  grid_dep_wait();  // the partial sums (and the zeroed counts) of router_partial_kernel
  grid_dep_launch();
  if (t >= p.T) return;  // whole warps leave together
  const int64_t tile = t / kTile, row = t % kTile;
  const float* base = p.part + ((tile * kSplit) * kTile + row) * E;
  typename A::T* gl = reinterpret_cast<typename A::T*>(p.logits);
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    const int e = i * 32 + lane;
    float acc = __ldcg(base + e);
#pragma unroll
    for (int k = 1; k < kSplit; ++k) acc = __fadd_rn(acc, __ldcg(base + (int64_t)k * kTile * E + e));
    const typename A::T v = A::from_f(acc);
    s_row[warp][e] = v;
    if (gl != nullptr) gl[t * E + e] = v;
  }
  __syncwarp();
  const int sel = router_tail_row<DT, VPL>(s_row[warp], p.top, t, p.weights, p.ids, p.probs);
  if (p.counts != nullptr && sel >= 0) atomicAdd(&p.counts[tile * (E + 1) + sel], 1);
}

}  // namespace rg

int64_t router_gemm_workspace(int64_t tokens, int64_t experts) {
  const int64_t tiles = (tokens + rg::kTile - 1) / rg::kTile;
  return tiles * rg::kSplit * rg::kTile * experts * 4;
}

bool router_gemm_ok(int64_t tokens, int64_t hidden, int64_t experts, int64_t top) {
  return tokens > 0 && hidden > 0 && hidden % rg::kBK == 0 && (experts == 64 || experts == 128 || experts == 256) &&
         top >= 1 && top <= 32 && top <= experts;
}

template <int DT, int VPL>
static int launch_router_gemm(const CUtensorMap& tx, const CUtensorMap& tw, const rg::Args& a, cudaStream_t st) {
  auto kg = rg::router_partial_kernel<DT, VPL>;
  auto kt = rg::router_tail_kernel<DT, VPL>;
  const int sg = rg::Smem<VPL * 32>::alloc;
  LMOE_CUDA_CHECK(cudaFuncSetAttribute(kg, cudaFuncAttributeMaxDynamicSharedMemorySize, sg));
  const unsigned tiles = (unsigned)((a.T + rg::kTile - 1) / rg::kTile);
  LMOE_CUDA_CHECK(launch_pdl(kg, dim3(tiles * rg::kSplit), dim3(rg::kGemmThreads), (size_t)sg, st, tx, tw, a));
  LMOE_CUDA_CHECK(launch_pdl(kt, dim3((unsigned)((a.T + rg::kTailWarps - 1) / rg::kTailWarps)),
                             dim3(rg::kTailWarps * 32), 0, st, a));
  return LMOE_OK;
}

int launch_router_gemm_topk(const void* x, const void* w, int64_t tokens, int64_t hidden, int64_t experts,
                            int64_t top, float* weights, int64_t* ids, float* probs, void* logits, int32_t* counts,
                            void* ws, int dtype, int* err, cudaStream_t st) {
  if (!x || !w || !weights || !ids || !ws || !router_gemm_ok(tokens, hidden, experts, top)) return LMOE_ERR_INVALID;
  if (((uintptr_t)ws) & 15) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  if ((((uintptr_t)x) & 15) || (((uintptr_t)w) & 15) || (logits && (((uintptr_t)logits) & 15)))
    return LMOE_ERR_INVALID;
  CUtensorMap tx, tw;
  int rc;
  if ((rc = make_act_map(&tx, x, tokens, hidden, dtype, rg::kTile))) return rc;
  if ((rc = make_act_map(&tw, w, experts, hidden, dtype, (int)experts))) return rc;
  rg::Args a = {};
  a.T = tokens;
  a.K = hidden;
  a.top = (int)top;
  a.part = (float*)ws;
  a.weights = weights;
  a.ids = ids;
  a.probs = probs;
  a.logits = logits;
  a.counts = counts;
  a.err = err;
#define LMOE_RG_CASE(DT)                                                      \
  switch (experts) {                                                          \
    case 64: return launch_router_gemm<DT, 2>(tx, tw, a, st);                 \
    case 128: return launch_router_gemm<DT, 4>(tx, tw, a, st);                \
    default: return launch_router_gemm<DT, 8>(tx, tw, a, st);                 \
  }
  if (dtype == LMOE_BF16) {
    LMOE_RG_CASE(LMOE_BF16)
  }
  LMOE_RG_CASE(LMOE_F16)
#undef LMOE_RG_CASE
}

}  // namespace lmoe

using namespace lmoe;

extern "C" int64_t lmoe_router_gemm_workspace_size(int64_t tokens, int64_t experts) {
  if (tokens <= 0 || experts <= 0) return 0;
  return router_gemm_workspace(tokens, experts);
}

extern "C" int lmoe_router_gemm_topk(const void* x, const void* router_w, int64_t tokens, int64_t hidden,
                                     int64_t experts, int64_t top, float* weights, int64_t* ids, float* probs,
                                     void* logits, void* ws, int dtype, int* err, void* stream) {
  return launch_router_gemm_topk(x, router_w, tokens, hidden, experts, top, weights, ids, probs, logits, nullptr, ws,
                                 dtype, err, (cudaStream_t)stream);
}
