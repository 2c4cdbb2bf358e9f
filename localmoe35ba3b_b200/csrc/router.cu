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
// One warp per token: lane j holds experts j, j + 32, ...; the max and the sum
// are butterfly reductions (every lane ends with the same value); top-k runs k
// warp-wide argmax rounds, ties going to the lower expert id.  The fp32 sum
// order differs from torch's reduction, so probabilities and weights may differ
// in the last ulp; equal logits give equal probabilities either way, so the
// selected expert set does not depend on it.  A NaN probability ranks below
// every number (it is selected only when nothing else is left).
#include "common.cuh"

namespace lmoe {

constexpr int kRouterWarps = 4;

template <int DT, int VPL>
__global__ void __launch_bounds__(kRouterWarps * 32)
    router_topk_kernel(const typename Act<DT>::T* __restrict__ logits, int64_t tokens, int top,
                       float* __restrict__ weights, int64_t* __restrict__ ids, float* __restrict__ probs) {
  constexpr int E = VPL * 32;
  const int64_t t = (int64_t)blockIdx.x * kRouterWarps + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (t >= tokens) return;  // whole warps leave together
  const typename Act<DT>::T* row = logits + t * E;
  float v[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) v[i] = Act<DT>::to_f(row[i * 32 + lane]);
  float m = v[0];
#pragma unroll
  for (int i = 1; i < VPL; ++i) m = fmaxf(m, v[i]);
#pragma unroll
  for (int o = 16; o; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
  float e[VPL], s = 0.f;
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    e[i] = expf(__fsub_rn(v[i], m));
    s = __fadd_rn(s, e[i]);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) s = __fadd_rn(s, __shfl_xor_sync(0xffffffffu, s, o));
  float p[VPL];
#pragma unroll
  for (int i = 0; i < VPL; ++i) {
    p[i] = __fdiv_rn(e[i], s);
    if (probs) probs[t * E + i * 32 + lane] = p[i];
    if (p[i] != p[i]) p[i] = -1.f;  // NaN ranks below every probability
  }
  float mine_v = 0.f, total = 0.f;
  int mine_i = 0;
  for (int r = 0; r < top; ++r) {
    float bv = -3.f;  // below NaN (-1) and taken (-2) entries
    int bi = E;
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (p[i] > bv) {  // ascending i: the lower id wins a tie inside the lane
        bv = p[i];
        bi = i * 32 + lane;
      }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
#pragma unroll
    for (int i = 0; i < VPL; ++i)
      if (bi == i * 32 + lane) p[i] = -2.f;  // taken
    if (lane == r) {
      mine_v = bv;
      mine_i = bi;
    }
    total = __fadd_rn(total, bv);
  }
  if (lane < top) {
    weights[t * top + lane] = __fdiv_rn(mine_v, total);
    ids[t * top + lane] = mine_i;
  }
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
