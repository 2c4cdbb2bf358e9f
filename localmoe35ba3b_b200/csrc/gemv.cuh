// Warp-level GEMV building blocks shared by the table-driven grouped GEMV
// (gemv.cu) and the fused one-token decode kernels (decode.cu), so both run the
// same arithmetic in the same order.
#pragma once
#include "common.cuh"

namespace lmoe {

constexpr int kMaxChunksPerLane = 8;  // K <= 4096: 16-byte chunks per lane

constexpr float kInv127 = 1.0f / 127.0f;  // fp32(1/127), the reference's (1./127.)

__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ int dp4a(uint32_t a, uint32_t b, int c) { return __dp4a((int)a, (int)b, c); }

// ----------------------------------------------------------------------------
// Activation quantisation of one (row, 128-group) by one warp.
template <int DT>
__device__ __forceinline__ void quant_group(const typename Act<DT>::T* xg, int8_t* qg, float* sg, int lane) {
  // 4 consecutive elements per lane
  float v[4];
  const uint2 raw = *reinterpret_cast<const uint2*>(xg + lane * 4);
  v[0] = Act<DT>::lo_f(raw.x);
  v[1] = Act<DT>::hi_f(raw.x);
  v[2] = Act<DT>::lo_f(raw.y);
  v[3] = Act<DT>::hi_f(raw.y);
  float a = fmaxf(fmaxf(fabsf(v[0]), fabsf(v[1])), fmaxf(fabsf(v[2]), fabsf(v[3])));
#pragma unroll
  for (int o = 16; o; o >>= 1) a = fmaxf(a, __shfl_xor_sync(0xffffffffu, a, o));
  const float s = __fmul_rn(fmaxf(a, 1e-10f), kInv127);
  uint32_t packed = 0;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const int qi = __float2int_rn(__fdiv_rn(v[j], s));  // IEEE divide, round half to even
    packed |= ((uint32_t)(qi & 0xff)) << (8 * j);
  }
  *reinterpret_cast<uint32_t*>(qg + lane * 4) = packed;
  if (lane == 0) *sg = s;
}

// One weight row (K int8 bytes) as 16-byte chunks, chunk lane + 32 i in w[i]; every
// load is issued before the first use.
template <int MAXI>
__device__ __forceinline__ void row_load(const int8_t* wrow, int chunks, int lane, uint4 (&w)[MAXI]) {
#pragma unroll
  for (int i = 0; i < MAXI; ++i)
    if (lane + 32 * i < chunks) w[i] = ldg_stream(wrow + (lane + 32 * i) * 16);
}

// W8A8 (w8a8._linear, operators/w8a8.py:25-41): exact int32 dot per 128-group, then
// acc = acc + (float(dot) * xs[g]) * ws[g] in group order.  xq / xs: the quantised
// activation row and its group scales; srow: the weight row's scales (global or
// shared memory).  Every lane returns acc.
template <int MAXI>
__device__ __forceinline__ float row_dot_w8a8(const uint4 (&w)[MAXI], const float* srow, const int8_t* xq,
                                              const float* xs, int chunks, int lane) {
  const int iters = (chunks + 31) / 32;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    if (i >= iters) break;
    const int c = lane + 32 * i;
    int d = 0;
    if (c < chunks) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xq + c * 16);
      d = dp4a(w[i].x, xv.x, d);
      d = dp4a(w[i].y, xv.y, d);
      d = dp4a(w[i].z, xv.z, d);
      d = dp4a(w[i].w, xv.w, d);
    }
    d += __shfl_xor_sync(0xffffffffu, d, 1);
    d += __shfl_xor_sync(0xffffffffu, d, 2);
    d += __shfl_xor_sync(0xffffffffu, d, 4);
    const int g = c >> 3;  // group of this lane's chunk
    float t = 0.f;
    if (c < chunks) t = __fmul_rn(__fmul_rn((float)d, xs[g]), srow[g]);
    // lanes 0, 8, 16, 24 hold groups 4i .. 4i+3; add them in order
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float tj = __shfl_sync(0xffffffffu, t, 8 * j);
      if (32 * i + 8 * j < chunks) acc = __fadd_rn(acc, tj);
    }
  }
  return acc;
}

// W8A16 (int8._linear arithmetic, operators/int8.py:19-21): w = round_dtype(q * s), fp32
// products summed in lane partials, then a butterfly tree.  xv: the activation row.
// Every lane returns the sum.
template <int DT, int MAXI>
__device__ __forceinline__ float row_dot_w16(const uint4 (&w)[MAXI], const float* srow,
                                             const typename Act<DT>::T* xv, int chunks, int lane) {
  const int iters = (chunks + 31) / 32;
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    if (i >= iters) break;
    const int c = lane + 32 * i;
    if (c >= chunks) continue;
    const float sc = srow[c >> 3];
    const uint4 xa = *reinterpret_cast<const uint4*>(xv + c * 16);
    const uint4 xb = *reinterpret_cast<const uint4*>(xv + c * 16 + 8);
    const uint32_t wv[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float f0, f1, f2, f3;
      i8x4_to_f32(wv[j], f0, f1, f2, f3);
      const float w0 = Act<DT>::round(__fmul_rn(f0, sc)), w1 = Act<DT>::round(__fmul_rn(f1, sc));
      const float w2 = Act<DT>::round(__fmul_rn(f2, sc)), w3 = Act<DT>::round(__fmul_rn(f3, sc));
      acc = fmaf(Act<DT>::lo_f(xw[2 * j]), w0, acc);
      acc = fmaf(Act<DT>::hi_f(xw[2 * j]), w1, acc);
      acc = fmaf(Act<DT>::lo_f(xw[2 * j + 1]), w2, acc);
      acc = fmaf(Act<DT>::hi_f(xw[2 * j + 1]), w3, acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace lmoe
