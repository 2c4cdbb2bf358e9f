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
// Activation quantisation of one (row, 128-group) by one warp: v = the lane's 4
// consecutive elements of the group (lane * 4 .. lane * 4 + 3).
__device__ __forceinline__ void quant_vals(const float (&v)[4], int8_t* qg, float* sg, int lane) {
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

template <int DT>
__device__ __forceinline__ void quant_group(const typename Act<DT>::T* xg, int8_t* qg, float* sg, int lane) {
  float v[4];
  const uint2 raw = *reinterpret_cast<const uint2*>(xg + lane * 4);
  v[0] = Act<DT>::lo_f(raw.x);
  v[1] = Act<DT>::hi_f(raw.x);
  v[2] = Act<DT>::lo_f(raw.y);
  v[3] = Act<DT>::hi_f(raw.y);
  quant_vals(v, qg, sg, lane);
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

// The same W8A8 row dot as row_dot_w8a8 -- bit for bit: the exact int32 group dots,
// t_g = (float(dot_g) * xs[g]) * ws[g], acc = acc + t_g in group order from 0 -- with
// the chunk partial sums of all of the lane's groups reduced together (independent
// shuffles), then gathered in group order.  w: the row's chunks as in row_dot_w8a8
// (chunk lane + 32 i; a group = 8 consecutive chunks).
template <int MAXI>
__device__ __forceinline__ float row_dot_w8a8_ilp(const uint4 (&w)[MAXI], const float* srow, const int8_t* xq,
                                                  const float* xs, int chunks, int lane) {
  int d[MAXI];
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    d[i] = 0;
    if (lane + 32 * i < chunks) {
      const uint4 xv = *reinterpret_cast<const uint4*>(xq + (lane + 32 * i) * 16);
      d[i] = dp4a(w[i].x, xv.x, d[i]);
      d[i] = dp4a(w[i].y, xv.y, d[i]);
      d[i] = dp4a(w[i].z, xv.z, d[i]);
      d[i] = dp4a(w[i].w, xv.w, d[i]);
    }
  }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1)
#pragma unroll
    for (int i = 0; i < MAXI; ++i) d[i] += __shfl_xor_sync(0xffffffffu, d[i], o);
  float t[MAXI];
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    const int c = lane + 32 * i;
    t[i] = c < chunks ? __fmul_rn(__fmul_rn((float)d[i], xs[c >> 3]), srow[c >> 3]) : 0.f;
  }
  float acc = 0.f;
#pragma unroll
  for (int i = 0; i < MAXI; ++i) {
    float tj[4];
#pragma unroll
    for (int j = 0; j < 4; ++j) tj[j] = __shfl_sync(0xffffffffu, t[i], 8 * j);
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (32 * i + 8 * j < chunks) acc = __fadd_rn(acc, tj[j]);
  }
  return acc;
}

// NR W8A8 row dots at once (row_dot_w8a8's arithmetic for each row, bit for bit),
// their shuffles interleaved: w[r] = row r's chunks, srow[r] its group scales, xq[r] /
// xs[r] its quantised activation row and scales.
template <int MAXI, int NR>
__device__ __forceinline__ void rows_dot_w8a8_ilp(const uint4 (&w)[NR][MAXI], const float* const (&srow)[NR],
                                                  const int8_t* const (&xq)[NR], const float* const (&xs)[NR],
                                                  int chunks, int lane, float (&out)[NR]) {
  int d[NR][MAXI];
#pragma unroll
  for (int r = 0; r < NR; ++r)
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
      d[r][i] = 0;
      if (lane + 32 * i < chunks) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xq[r] + (lane + 32 * i) * 16);
        d[r][i] = dp4a(w[r][i].x, xv.x, d[r][i]);
        d[r][i] = dp4a(w[r][i].y, xv.y, d[r][i]);
        d[r][i] = dp4a(w[r][i].z, xv.z, d[r][i]);
        d[r][i] = dp4a(w[r][i].w, xv.w, d[r][i]);
      }
    }
#pragma unroll
  for (int o = 1; o < 8; o <<= 1)
#pragma unroll
    for (int r = 0; r < NR; ++r)
#pragma unroll
      for (int i = 0; i < MAXI; ++i) d[r][i] += __shfl_xor_sync(0xffffffffu, d[r][i], o);
#pragma unroll
  for (int r = 0; r < NR; ++r) {
    float t[MAXI];
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
      const int c = lane + 32 * i;
      t[i] = c < chunks ? __fmul_rn(__fmul_rn((float)d[r][i], xs[r][c >> 3]), srow[r][c >> 3]) : 0.f;
    }
    float acc = 0.f;
#pragma unroll
    for (int i = 0; i < MAXI; ++i) {
      float tj[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) tj[j] = __shfl_sync(0xffffffffu, t[i], 8 * j);
#pragma unroll
      for (int j = 0; j < 4; ++j)
        if (32 * i + 8 * j < chunks) acc = __fadd_rn(acc, tj[j]);
    }
    out[r] = acc;
  }
}

// W8A16 (int8._linear arithmetic, operators/int8.py:19-21): w = round_dtype(q * s), fp32
// products summed in lane partials, then a butterfly tree.  xv: the activation row
// (read through L2 only when CG, for rows that other CTAs of the same launch wrote).
// Every lane returns the sum.
template <int DT, int MAXI, bool CG = false>
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
    const uint4* xp = reinterpret_cast<const uint4*>(xv + c * 16);
    const uint4 xa = CG ? __ldcg(xp) : xp[0];
    const uint4 xb = CG ? __ldcg(xp + 1) : xp[1];
    const uint32_t wv[4] = {w[i].x, w[i].y, w[i].z, w[i].w};
    const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
    const uint64_t sc2 = splat2(sc);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      // round_dtype(q * s) for the word's 4 weights, two to a register (deq4: packed
      // f32x2 products, the same bits as one product and one rounding per weight)
      uint32_t lo, hi;
      deq4<DT>(wv[j], sc2, lo, hi);
      acc = fmaf(Act<DT>::lo_f(xw[2 * j]), Act<DT>::lo_f(lo), acc);
      acc = fmaf(Act<DT>::hi_f(xw[2 * j]), Act<DT>::hi_f(lo), acc);
      acc = fmaf(Act<DT>::lo_f(xw[2 * j + 1]), Act<DT>::lo_f(hi), acc);
      acc = fmaf(Act<DT>::hi_f(xw[2 * j + 1]), Act<DT>::hi_f(hi), acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  return acc;
}

}  // namespace lmoe
