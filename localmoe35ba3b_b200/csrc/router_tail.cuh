// The router tail of the sparse-MoE block for one token, shared by the router kernels:
// fp32 softmax over the expert logits, top-k, renormalisation, restating the HF
// Qwen3_5MoeTopKRouter.forward tail (transformers/models/qwen3_5_moe/
// modeling_qwen3_5_moe.py:765-769):
//   p = softmax(float(logits)); (v, i) = topk(p, k); w = v / sum(v)   (fp32)
// One warp per token: lane j holds experts j, j + 32, ...; the max and the sum are
// butterfly reductions (every lane ends with the same value); top-k runs k warp-wide
// argmax rounds, ties going to the lower expert id.  The fp32 sum order differs from
// torch's reduction, so probabilities and weights may differ in the last ulp; equal
// logits give equal probabilities either way, so the selected expert set does not
// depend on it.  A NaN probability ranks below every number (it is selected only when
// nothing else is left).
#pragma once
#include "common.cuh"

namespace lmoe {

// row: the token's E = 32 * VPL logits (global or shared memory); writes weights[t, :top],
// ids[t, :top] and, when probs, probs[t, :]; returns the expert chosen in round `lane`
// (lanes < top), -1 on the other lanes.
template <int DT, int VPL>
__device__ __forceinline__ int router_tail_row(const typename Act<DT>::T* row, int top, int64_t t,
                                               float* __restrict__ weights, int64_t* __restrict__ ids,
                                               float* __restrict__ probs) {
  constexpr int E = VPL * 32;
  const int lane = threadIdx.x & 31;
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
  return lane < top ? mine_i : -1;
}

}  // namespace lmoe
