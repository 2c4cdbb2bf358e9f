// Router tail of the sparse-MoE block on the device: fp32 softmax over the
// expert logits, top-k, renormalisation.
//
// Restates the HF Qwen3_5MoeTopKRouter.forward tail that the reference drives
// (transformers/models/qwen3_5_moe/modeling_qwen3_5_moe.py:765-769 -- the
// reference replaces only the experts and the linears, qwen35_deploy/model.py:57-68):
//   p = softmax(float(logits)); (v, i) = topk(p, k); w = v / sum(v)   (fp32)
// The logits themselves are the block's bf16 `F.linear(x, gate.weight)`, a plain
// library GEMM computed by the caller.
//
// One warp per token; the tail's arithmetic is router_tail_row (router_tail.cuh), which
// the fused logits + tail kernel (router_gemm.cu) runs too.
#include "common.cuh"
#include "router_tail.cuh"

namespace lmoe {

constexpr int kRouterWarps = 4;

template <int DT, int VPL>
__global__ void __launch_bounds__(kRouterWarps * 32)
    router_topk_kernel(const typename Act<DT>::T* __restrict__ logits, int64_t tokens, int top,
                       float* __restrict__ weights, int64_t* __restrict__ ids, float* __restrict__ probs) {
  constexpr int E = VPL * 32;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  if (t >= tokens) return;  // whole warps leave together
  router_tail_row<DT, VPL>(logits + t * E, top, t, weights, ids, probs);
}

template <int DT, int VPL>
static void launch_router(const void* logits, int64_t tokens, int top, float* w, int64_t* ids, float* probs,
                          cudaStream_t st) {
  const unsigned blocks = (unsigned)((tokens + kRouterWarps - 1) / kRouterWarps);
  router_topk_kernel<DT, VPL><<<blocks, kRouterWarps * 32, 0, st>>>((const typename Act<DT>::T*)logits, tokens, top, w,
                                                                    ids, probs);
}

template <int DT>
static int dispatch_router(const void* logits, int64_t tokens, int64_t experts, int top, float* w, int64_t* ids,
                           float* probs, cudaStream_t st) {
  switch (experts / 32) {
    case 1: launch_router<DT, 1>(logits, tokens, top, w, ids, probs, st); break;
    case 2: launch_router<DT, 2>(logits, tokens, top, w, ids, probs, st); break;
    case 4: launch_router<DT, 4>(logits, tokens, top, w, ids, probs, st); break;
    case 8: launch_router<DT, 8>(logits, tokens, top, w, ids, probs, st); break;
    case 16: launch_router<DT, 16>(logits, tokens, top, w, ids, probs, st); break;
    default: return LMOE_ERR_UNSUPPORTED;
  }
  return LMOE_OK;
}

}  // namespace lmoe

using namespace lmoe;

extern "C" int lmoe_router_topk(const void* logits, int64_t tokens, int64_t experts, int64_t top, float* weights,
                                int64_t* ids, float* probs, int dtype, void* stream) {
  if (!logits || !weights || !ids || tokens < 0 || experts <= 0 || top <= 0 || top > 32 || top > experts)
    return LMOE_ERR_INVALID;
  if (experts % 32) return LMOE_ERR_UNSUPPORTED;
  if (tokens == 0) return LMOE_OK;
  cudaStream_t st = (cudaStream_t)stream;
  int rc;
  if (dtype == LMOE_BF16)
    rc = dispatch_router<LMOE_BF16>(logits, tokens, experts, (int)top, weights, ids, probs, st);
  else if (dtype == LMOE_F16)
    rc = dispatch_router<LMOE_F16>(logits, tokens, experts, (int)top, weights, ids, probs, st);
  else
    return LMOE_ERR_INVALID;
  if (rc) return rc;
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}
