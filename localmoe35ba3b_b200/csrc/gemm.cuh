// Host-side launch description of the tcgen05 grouped GEMM (grouped_gemm.cu).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "routes.cuh"

namespace lmoe {

enum GemmMode { kPlain = 0, kSwiGLU = 1, kWeighted = 2 };

struct GemmLaunch {
  const void* x;          // activations [x_rows, K]
  int64_t x_rows;
  int64_t K;
  const Tile* tiles;      // nullptr: dense mode over dense_rows rows
  const int32_t* hdr;     // tiles mode: metadata header (tile count)
  int64_t grid_tiles;     // grid.y: max tiles (tiles mode) or ceil(M/256) (dense)
  int64_t dense_rows;
  const int8_t* q_bank;   // routed bank [experts*N, K]
  const float* s_bank;
  int64_t experts, N, inter;
  const int8_t* q_lo;     // shared expert: gate (SwiGLU) or whole matrix (plain/weighted)
  const float* s_lo;
  const int8_t* q_hi;     // shared expert: up (SwiGLU)
  const float* s_hi;
  int64_t rows_lo, rows_hi;
  void* y;
  int64_t ldy;
  const float* rweight;   // weighted mode: per-route weight
  int mode;
  int dtype;
  int* err;
  int ksplit;             // TS down kernel, dense mode: K splits (fp32 sums to partial)
  float* partial;
};

int launch_grouped_gemm(const GemmLaunch& L, cudaStream_t st);
// gate_up with the SwiGLU epilogue / down with the routing-weight epilogue on the
// TMEM-operand kernel (gemm_ts.cu)
int launch_swiglu_ts(const GemmLaunch& L, cudaStream_t st);
int launch_down_ts(const GemmLaunch& L, cudaStream_t st);
// the SwiGLU epilogue's SiLU against the exact division over every 16-bit gate value
int selftest_silu(int dtype, int* mismatches, cudaStream_t st);
// dense W8A16 linear on the TS kernel (gemm_ts.cu): n % 128 == 0, k % 128 == 0; K split over
// dense_ts_workspace bytes of ws when the units would not fill the SMs (ws == nullptr: no split)
bool dense_ts_ok(int64_t m, int64_t n, int64_t k);
int64_t dense_ts_workspace(int64_t m, int64_t n, int64_t k);
int launch_dense_ts(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n, int64_t k,
                    int dtype, void* ws, int64_t ws_bytes, int* err, cudaStream_t st);

// tensor maps (grouped_gemm.cu): int8 [rows, K] with a 64-row x 128-byte, 128B-swizzled box;
// 16-bit activations [rows, K] with a box_rows x 64-element, 128B-swizzled box
int make_int8_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K);
int make_int8_pair_map(CUtensorMap* m, const int8_t* base, int64_t experts, int64_t inter, int64_t K);
int make_act_map(CUtensorMap* m, const void* base, int64_t rows, int64_t K, int dtype, int box_rows);
int make_i8_tile_map(CUtensorMap* m, const int8_t* base, int64_t rows, int64_t K);
int sm_count();

// out[r] = x[pos[r]] for r < rows; rows of k 16-bit elements (permute.cu)
int launch_permute_rows(const void* x, const int32_t* pos, void* out, int64_t rows, int64_t k, cudaStream_t st);

}  // namespace lmoe
