// Dense W8A8 linear on tcgen05 integer tensor cores (kind::i8, int32 accumulation).
//
// The reference's W8A8 arithmetic (qwen35_deploy/operators/w8a8.py:8-41: _quant, then
// _linear) for any number of activation rows m: each row quantised per 128-wide K group
// (q = rint(x / s), s = max(absmax, 1e-10) * (1/127)), then per output (row, n)
//   acc = 0;  for g in order: acc = acc + (float(dot_g) * xs[row, g]) * ws[n, g]
// with dot_g the exact int32 dot of the group and no fused multiply-add, rounded once to
// the activation dtype.  The reference runs it as a one-row GEMV per expert (decode);
// this kernel runs it for the dense sweep's m rows, bit for bit the same arithmetic.
//
// Unit = (128-row tile of the activations, 128 weight rows), persistent CTAs.  Per 128-K
// group g: w0 (TMA) brings the int8 activation tile [128 x 128 B] and the weight tile
// [128 x 128 B] (128B-swizzled) into stage g % 4; w1 (TMEM owner, MMA issuer) issues 4
// MMAs (M = 128 rows, N = 128 weight rows, K = 32) into int32 accumulator buffer g % 2,
// fresh for the group, and commits; 8 epilogue warps (2 per TMEM lane quadrant, 64 columns
// each) read the group's int32 dots, hand the buffer back, and fold them into fp32
// accumulators held in registers for the whole unit: t = (float(dot) * xs) * ws, acc += t
// (float(dot) exactly: |dot| <= 128^3 < 2^22, via the 1.5 * 2^23 bias).  The weight
// scales of the unit (128 rows x K/128 fp32) arrive by one bulk copy per unit.  Every wait
// is bounded (LMOE_WAIT_NS); a timeout raises the abort flag and the caller's error word.
#include "common.cuh"
#include "gemm.cuh"

namespace lmoe {
namespace w8 {

constexpr int kTile = 128;                 // activation rows per unit: the MMA M extent
constexpr int kBN = 128;                   // weight rows per unit: the MMA N extent
constexpr int kStages = 4;
constexpr int kEpiWarps = 8;
constexpr int kThreads = (2 + kEpiWarps) * 32;
constexpr int kMaxGroups = 64;             // K <= 8192
constexpr int kStageBytes = (kTile + kBN) * 128;  // 32 KB: the activation and weight group tiles
constexpr int kWsBytes = kBN * kMaxGroups * 4;    // the unit's weight scales (fp32)

struct Smem {
  static constexpr int stages = 0;
  static constexpr int ws = kStages * kStageBytes;  // two buffers of weight scales [128][G], as copied
  static constexpr int wst = ws + 2 * kWsBytes;     // the unit's scales transposed, [G][128]
  static constexpr int bars = wst + kWsBytes;
  // full, empty (kStages each); tfull, tempty (2 each); wfull, wempty (2 each)
  static constexpr int nbars = 2 * kStages + 8;
  static constexpr int misc = bars + nbars * 8;
  static constexpr int bytes = misc + 16;
  static constexpr int alloc = bytes + 1024;
};
static_assert(Smem::alloc <= 232448, "shared memory per block");

struct Params {
  int64_t M, N, K;
  const float* xs;   // [M, K/128] activation scales
  const float* ws;   // [N, K/128] weight scales
  void* y;           // [M, N]
  int* err;
};

// Two group terms at once: float(d) for |d| < 2^22 as the int bits of 1.5 * 2^23 + d minus
// 1.5 * 2^23 (exact), then t = (float(d) * xs) * ws with packed f32x2 multiplies (each lane the
// IEEE round-to-nearest product), and acc = acc + t as two scalar add.rn.f32. The add stays
// scalar on purpose: ptxas contracts a packed mul.rn.f32x2 feeding a packed add.rn.f32x2 into
// one fused multiply-add (measured: the outputs then equal fma(float(d) * xs, ws, acc) in every
// element), which is not the reference's rounding; scalar add.rn.f32 is never contracted.
__device__ __forceinline__ void fold2(float& acc0, float& acc1, uint32_t d0, uint32_t d1, uint64_t xs2, float w0,
                                      float w1) {
  uint64_t v, w;
  asm("mov.b64 %0, {%1, %2};" : "=l"(v) : "r"(0x4B400000u + d0), "r"(0x4B400000u + d1));
  asm("sub.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(0x4B4000004B400000ull));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(xs2));
  asm("mov.b64 %0, {%1, %2};" : "=l"(w) : "f"(w0), "f"(w1));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(v) : "l"(w));
  float t0, t1;
  asm("mov.b64 {%0, %1}, %2;" : "=f"(t0), "=f"(t1) : "l"(v));
  acc0 = __fadd_rn(acc0, t0);
  acc1 = __fadd_rn(acc1, t1);
}

template <int DT>
__global__ void __launch_bounds__(kThreads, 1)
    w8a8_gemm_kernel(const __grid_constant__ CUtensorMap tm_x, const __grid_constant__ CUtensorMap tm_w,
                     const Params p) {
  using A = Act<DT>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = (uint8_t*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sb = smem_u32(smem);
  const uint32_t bar0 = sb + Smem::bars;
  auto full = [&](int s) { return bar0 + 8u * s; };
  auto empty = [&](int s) { return bar0 + 8u * (kStages + s); };
  auto tfull = [&](int b) { return bar0 + 8u * (2 * kStages + b); };
  auto tempty = [&](int b) { return bar0 + 8u * (2 * kStages + 2 + b); };
  auto wfull = [&](int b) { return bar0 + 8u * (2 * kStages + 4 + b); };
  auto wempty = [&](int b) { return bar0 + 8u * (2 * kStages + 6 + b); };
  uint32_t* sTmem = reinterpret_cast<uint32_t*>(smem + Smem::misc);
  volatile int* sAbort = reinterpret_cast<volatile int*>(smem + Smem::misc + 4);
  const int warp = warp_id(), lane = lane_id();
  const int G = (int)(p.K / 128);
  const int nblk = (int)(p.N / kBN);
  const int64_t units = ((p.M + kTile - 1) / kTile) * nblk;
  const int stride = gridDim.x;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(full(s), 1);
      mbar_init(empty(s), 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(tfull(b), 1);
      mbar_init(tempty(b), kEpiWarps);
      mbar_init(wfull(b), 1);
      mbar_init(wempty(b), kEpiWarps);
    }
    *sAbort = 0;
    fence_mbar_init();
  }
  if (warp == 0 && lane == 0) {
    prefetch_tmap(&tm_x);
    prefetch_tmap(&tm_w);
  }
  if (warp == 1) {
    tmem_alloc(smem_u32(sTmem), 2 * kBN);
    tmem_relinquish();
    tc_fence_before();
  }
  __syncthreads();
  tc_fence_after();
  grid_dep_launch();
  const uint32_t tmem = *sTmem;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    // the quantised activations are the previous kernel's output
    grid_dep_wait();
    if (lane == 0) {
      int it = 0, ui = 0, nw = 0;
      bool ok = true;
      for (int64_t u = blockIdx.x; u < units && ok; u += stride, ++ui) {
        const int64_t t0 = (u / nblk) * kTile, n0 = (u % nblk) * kBN;
        // the unit's weight scales: rows n0 .. n0 + 127, contiguous
        const int wb = ui & 1;
        if (!mbar_wait(wempty(wb), ((ui >> 1) & 1) ^ 1, sAbort, p.err)) break;
        ++nw;
        mbar_arrive_expect_tx(wfull(wb), (uint32_t)(kBN * G * 4));
        bulk_g2s(sb + (uint32_t)(Smem::ws + wb * kWsBytes), p.ws + n0 * G, (uint32_t)(kBN * G * 4), wfull(wb));
        for (int g = 0; g < G; ++g, ++it) {
          const int s = it % kStages;
          if (!mbar_wait(empty(s), ((it / kStages) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          mbar_arrive_expect_tx(full(s), kStageBytes);
          const uint32_t dst = sb + (uint32_t)(s * kStageBytes);
          tma_load_2d(dst, &tm_x, full(s), g * 128, (int)t0);
          tma_load_2d(dst + kTile * 128, &tm_w, full(s), g * 128, (int)n0);
        }
      }
      // never leave a copy in flight into shared memory when the CTA may exit
      for (int k = max(0, it - kStages); k < it; ++k) mbar_wait_drain(full(k % kStages), (k / kStages) & 1, p.err);
      for (int k = max(0, nw - 2); k < nw; ++k) mbar_wait_drain(wfull(k & 1), (k >> 1) & 1, p.err);
    }
    __syncwarp();
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = idesc_i8(kTile, kBN);
      int it = 0, gi = 0;
      bool ok = true, issued = false;
      for (int64_t u = blockIdx.x; u < units && ok; u += stride) {
        for (int g = 0; g < G; ++g, ++it, ++gi) {
          const int b = gi & 1;  // one int32 accumulator buffer per group, alternating
          if (!mbar_wait(tempty(b), ((gi >> 1) & 1) ^ 1, sAbort, p.err)) { ok = false; break; }
          const int s = it % kStages;
          if (!mbar_wait(full(s), (it / kStages) & 1, sAbort, p.err)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = sdesc_k_sw128(sb + (uint32_t)(s * kStageBytes));
          const uint64_t bd = sdesc_k_sw128(sb + (uint32_t)(s * kStageBytes + kTile * 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            mma_i8(tmem + (uint32_t)(b * kBN), ad + (uint64_t)(kk * 2), bd + (uint64_t)(kk * 2), idesc, kk != 0);
          mma_commit(empty(s));
          mma_commit(tfull(b));
          issued = true;
        }
      }
      // (after an abort the epilogue's waits end on the abort flag)
      (void)issued;
    }
    __syncwarp();
  } else {
    // ------------------------------------------------------------ epilogue
    // warp w: TMEM lane quadrant w % 4 (its 32 activation rows), columns h * 64 .. + 63
    const int q = warp & 3, h = (warp - 2) >> 2;
    const int row = q * 32 + lane;
    typename A::T* y = (typename A::T*)p.y;
    int gi = 0, ui = 0;
    bool ok = true;
    // the activation scales read below are the previous kernel's (the quantiser's) output
    grid_dep_wait();
    // every epilogue warp walks every unit and reaches both named barriers of each, also
    // after an abort (then skipping the work), so that none can wait at a barrier for good
    for (int64_t u = blockIdx.x; u < units; u += stride, ++ui) {
      const int64_t t0 = (u / nblk) * kTile, n0 = (u % nblk) * kBN;
      const int64_t t = t0 + row;
      const int wb = ui & 1;
      int have = 0;
      if (lane == 0 && ok) have = mbar_wait(wfull(wb), (ui >> 1) & 1, sAbort, p.err) ? 1 : 0;
      have = __shfl_sync(0xffffffffu, have, 0);
      ok = ok && have;
      // the unit's scales transposed to [G][128] by all the epilogue warps (the previous
      // unit's reads of the transposed copy ended at its second barrier)
      named_barrier(1, kEpiWarps * 32);
      if (ok) {
        const float* src = reinterpret_cast<const float*>(smem + Smem::ws + wb * kWsBytes);
        float* dst = reinterpret_cast<float*>(smem + Smem::wst);
        for (int i = threadIdx.x - 64; i < kBN * G; i += kEpiWarps * 32) dst[(i % G) * kBN + i / G] = src[i];
      }
      named_barrier(1, kEpiWarps * 32);
      __syncwarp();
      if (lane == 0) mbar_arrive(wempty(wb));  // the copied buffer is free again
      const float* swt = reinterpret_cast<const float*>(smem + Smem::wst);
      const float* xsr = p.xs + (t < p.M ? t : 0) * G;
      float acc[64];
#pragma unroll
      for (int j = 0; j < 64; ++j) acc[j] = 0.f;
      for (int g = 0; g < G && ok; ++g, ++gi) {
        const int b = gi & 1;
        const float xsg = xsr[g];
        if (lane == 0) have = mbar_wait(tfull(b), (gi >> 1) & 1, sAbort, p.err) ? 1 : 0;
        if (!__shfl_sync(0xffffffffu, have, 0)) {
          ok = false;
          break;
        }
        tc_fence_after();
        uint32_t d0[32], d1[32];
        const uint32_t ta = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(b * kBN + h * 64);
        tmem_ld32(ta, d0);
        tmem_ld32(ta + 32, d1);
        tmem_ld_wait();
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(tempty(b));
        // t = (float(dot) * xs[row, g]) * ws[n, g]; acc = acc + t (in group order); this
        // group's 64 weight scales are one broadcast row of the transposed copy
        const uint64_t xs2 = splat2(xsg);
        const uint32_t wrow = smem_u32(swt + g * kBN + h * 64);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const uint4 wa = lds128(wrow + j * 4), wc = lds128(wrow + 128 + j * 4);
          fold2(acc[j], acc[j + 1], d0[j], d0[j + 1], xs2, __uint_as_float(wa.x), __uint_as_float(wa.y));
          fold2(acc[j + 2], acc[j + 3], d0[j + 2], d0[j + 3], xs2, __uint_as_float(wa.z), __uint_as_float(wa.w));
          fold2(acc[32 + j], acc[33 + j], d1[j], d1[j + 1], xs2, __uint_as_float(wc.x), __uint_as_float(wc.y));
          fold2(acc[34 + j], acc[35 + j], d1[j + 2], d1[j + 3], xs2, __uint_as_float(wc.z), __uint_as_float(wc.w));
        }
      }
      if (ok && t < p.M) {
        typename A::T* dst = y + t * p.N + n0 + h * 64;
#pragma unroll
        for (int j = 0; j < 8; ++j)
          reinterpret_cast<uint4*>(dst)[j] =
              make_uint4(A::pack(acc[8 * j], acc[8 * j + 1]), A::pack(acc[8 * j + 2], acc[8 * j + 3]),
                         A::pack(acc[8 * j + 4], acc[8 * j + 5]), A::pack(acc[8 * j + 6], acc[8 * j + 7]));
      }
    }
  }

  // ---------------------------------------------------------------- teardown
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 2 * kBN);
  }
}

}  // namespace w8

bool w8a8_gemm_ok(int64_t m, int64_t n, int64_t k) {
  return m >= 1 && n > 0 && n % w8::kBN == 0 && k > 0 && k % 128 == 0 && k / 128 <= w8::kMaxGroups;
}

int64_t w8a8_gemm_workspace(int64_t m, int64_t k) {
  const int64_t q = (m * k + 255) & ~int64_t(255);
  return q + m * (k / 128) * 4;
}

int launch_w8a8_gemm(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n, int64_t k,
                     int dtype, void* ws, int* err, cudaStream_t st) {
  if (!x || !q || !scale || !y || !ws || !w8a8_gemm_ok(m, n, k)) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  if ((((uintptr_t)q) & 15) || (((uintptr_t)ws) & 255) || (((uintptr_t)y) & 15) || (((uintptr_t)scale) & 15))
    return LMOE_ERR_INVALID;
  int8_t* xq = (int8_t*)ws;
  float* xs = (float*)((char*)ws + ((m * k + 255) & ~int64_t(255)));
  int rc = lmoe_quantize_rows(x, xq, xs, m, k, dtype, (void*)st);
  if (rc) return rc;
  CUtensorMap tx, tw;
  if ((rc = make_i8_tile_map(&tx, xq, m, k))) return rc;
  if ((rc = make_i8_tile_map(&tw, q, n, k))) return rc;
  w8::Params p = {};
  p.M = m;
  p.N = n;
  p.K = k;
  p.xs = xs;
  p.ws = scale;
  p.y = y;
  p.err = err;
  const int64_t units = ((m + w8::kTile - 1) / w8::kTile) * (n / w8::kBN);
  const int64_t sms = sm_count();
  const unsigned grid = (unsigned)(units < sms ? units : sms);
  const size_t smem = w8::Smem::alloc;
  if (dtype == LMOE_BF16) {
    auto kf = w8::w8a8_gemm_kernel<LMOE_BF16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(launch_pdl(kf, dim3(grid), dim3(w8::kThreads), smem, st, tx, tw, p));
  } else {
    auto kf = w8::w8a8_gemm_kernel<LMOE_F16>;
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(kf, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
    LMOE_CUDA_CHECK(launch_pdl(kf, dim3(grid), dim3(w8::kThreads), smem, st, tx, tw, p));
  }
  return LMOE_OK;
}

}  // namespace lmoe

using namespace lmoe;

extern "C" int64_t lmoe_linear_w8a8_workspace_size(int64_t m, int64_t k) {
  if (m <= 0 || k <= 0 || k % 128) return 0;
  return w8a8_gemm_workspace(m, k);
}

extern "C" int lmoe_linear_w8a8(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                                int64_t k, int dtype, void* ws, int* err, void* stream) {
  if (m == 0) return LMOE_OK;
  return launch_w8a8_gemm(x, q, scale, y, m, n, k, dtype, ws, err, (cudaStream_t)stream);
}
