// Route-order permutation of activation rows: out[r] = x[pos[r]].
//
// The prefill gate_up GEMM reads its B operand as TMA tiles of consecutive
// rows, so the per-route gather of the reference's _routed kernel
// (x[POS[row]], qwen35_deploy/runtime/prefill.py:20-23) is done once here:
// one warp per output row, 16-byte loads and stores.  The source x (T rows)
// is small and read top-k times, so most reads hit L2.
#include "common.cuh"
#include "gemm.cuh"

namespace lmoe {

constexpr int kPermWarps = 8;

__global__ void __launch_bounds__(kPermWarps * 32) permute_rows_kernel(const uint4* __restrict__ x,
                                                                      const int32_t* __restrict__ pos,
                                                                      uint4* __restrict__ out, int64_t rows,
                                                                      int64_t vec_per_row) {
  grid_dep_wait();    // pos is the previous kernel's output
  grid_dep_launch();  // the gate_up kernel may take SMs as this kernel's blocks leave them
  const int64_t r = (int64_t)blockIdx.x * kPermWarps + warp_id();
  if (r >= rows) return;
  const int64_t src = pos[r];
  const uint4* s = x + src * vec_per_row;
  uint4* d = out + r * vec_per_row;
  for (int64_t i = lane_id(); i < vec_per_row; i += 32) d[i] = __ldg(s + i);
}

int launch_permute_rows(const void* x, const int32_t* pos, void* out, int64_t rows, int64_t k, cudaStream_t st) {
  if (rows <= 0) return LMOE_OK;
  if (k % 8 || ((uintptr_t)x & 15) || ((uintptr_t)out & 15)) return LMOE_ERR_INVALID;
  const unsigned blocks = (unsigned)((rows + kPermWarps - 1) / kPermWarps);
  LMOE_CUDA_CHECK(launch_pdl(permute_rows_kernel, dim3(blocks), dim3(kPermWarps * 32), 0, st, (const uint4*)x, pos,
                             (uint4*)out, rows, k / 8));
  return LMOE_OK;
}

}  // namespace lmoe
