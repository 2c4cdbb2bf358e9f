// Shared device helpers for the sm_100a INT8 group-128 MoE kernels.
//
// Every spin-wait here is bounded: after LMOE_WAIT_NS nanoseconds (read from
// %globaltimer) a wait gives up, raises the CTA's abort flag and the global
// error word, and returns false so the caller can drain and exit.  No kernel
// in this library traps or asserts on the device.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/localmoe_b200.h"

#ifndef LMOE_WAIT_NS
#define LMOE_WAIT_NS 2000000000ull  // 2 s
#endif

namespace lmoe {

constexpr int kGroup = 128;  // quantisation group along K

// ---------------------------------------------------------------- dtypes
template <int DT> struct Act;
template <> struct Act<LMOE_BF16> {
  using T = __nv_bfloat16;
  using T2 = __nv_bfloat162;
  static __device__ __forceinline__ float to_f(T v) { return __bfloat162float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2bfloat16_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
  // two fp32 -> packed pair, round to nearest even (lo in the low half)
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  static __device__ __forceinline__ float lo_f(uint32_t u) { return __uint_as_float(u << 16); }
  static __device__ __forceinline__ float hi_f(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
  static __device__ __forceinline__ uint16_t bits(float v) { return __bfloat16_as_ushort(__float2bfloat16_rn(v)); }
};
template <> struct Act<LMOE_F16> {
  using T = __half;
  using T2 = __half2;
  static __device__ __forceinline__ float to_f(T v) { return __half2float(v); }
  static __device__ __forceinline__ T from_f(float v) { return __float2half_rn(v); }
  static __device__ __forceinline__ float round(float v) { return __half2float(__float2half_rn(v)); }
  static __device__ __forceinline__ uint32_t pack(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.f16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
  }
  static __device__ __forceinline__ float lo_f(uint32_t u) {
    return __half2float(__ushort_as_half((unsigned short)(u & 0xffffu)));
  }
  static __device__ __forceinline__ float hi_f(uint32_t u) {
    return __half2float(__ushort_as_half((unsigned short)(u >> 16)));
  }
  static __device__ __forceinline__ uint16_t bits(float v) { return __half_as_ushort(__float2half_rn(v)); }
};

// int8 lane j (0..3) of a 32-bit word, as fp32 (exact)
__device__ __forceinline__ float i8f(uint32_t w, int j) {
  return (float)(int)(int8_t)((w >> (8 * j)) & 0xffu);
}

// Exact int8 -> fp32 for all four bytes of a word using the 2^23 magic:
// as_float(0x4B000000 | (b ^ 0x80)) = 2^23 + b + 128, minus (2^23 + 128) = b.
__device__ __forceinline__ void i8x4_to_f32(uint32_t w, float& f0, float& f1, float& f2, float& f3) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t m0, m1, m2, m3;
  // selector 0x765k: result byte0 = u.byte_k, bytes 1..3 = 0x00, 0x00, 0x4B from the constant
  asm("prmt.b32 %0, %1, %2, 0x7650;" : "=r"(m0) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7651;" : "=r"(m1) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7652;" : "=r"(m2) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7653;" : "=r"(m3) : "r"(u), "r"(0x4B000000u));
  const float magic = 8388736.0f;  // 2^23 + 128
  f0 = __uint_as_float(m0) - magic;
  f1 = __uint_as_float(m1) - magic;
  f2 = __uint_as_float(m2) - magic;
  f3 = __uint_as_float(m3) - magic;
}

// Dequantise one int8 word with packed f32x2 arithmetic: lo / hi = the packed
// 16-bit pairs round_dtype(float(q_j) * s) for bytes j = 0,1 / 2,3.  Each lane of
// sub.rn.f32x2 and mul.rn.f32x2 is the IEEE round-to-nearest operation of the
// scalar path (i8x4_to_f32, __fmul_rn, Act::pack), so the results are the same bit
// for bit with half the floating-point instructions.  s2 = splat2(scale).
__device__ __forceinline__ uint64_t splat2(float s) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %1};" : "=l"(r) : "r"(__float_as_uint(s)));
  return r;
}
template <int DT>
__device__ __forceinline__ void deq4(uint32_t w, uint64_t s2, uint32_t& lo, uint32_t& hi) {
  const uint32_t u = w ^ 0x80808080u;
  uint32_t m0, m1, m2, m3;
  asm("prmt.b32 %0, %1, %2, 0x7650;" : "=r"(m0) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7651;" : "=r"(m1) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7652;" : "=r"(m2) : "r"(u), "r"(0x4B000000u));
  asm("prmt.b32 %0, %1, %2, 0x7653;" : "=r"(m3) : "r"(u), "r"(0x4B000000u));
  uint64_t a, b;
  asm("mov.b64 %0, {%1, %2};" : "=l"(a) : "r"(m0), "r"(m1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(b) : "r"(m2), "r"(m3));
  const uint64_t magic2 = 0x4B0000804B000080ull;  // (2^23 + 128) in both lanes
  asm("sub.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(magic2));
  asm("sub.rn.f32x2 %0, %0, %1;" : "+l"(b) : "l"(magic2));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(a) : "l"(s2));
  asm("mul.rn.f32x2 %0, %0, %1;" : "+l"(b) : "l"(s2));
  uint32_t a0, a1, b0, b1;
  asm("mov.b64 {%0, %1}, %2;" : "=r"(a0), "=r"(a1) : "l"(a));
  asm("mov.b64 {%0, %1}, %2;" : "=r"(b0), "=r"(b1) : "l"(b));
  lo = Act<DT>::pack(__uint_as_float(a0), __uint_as_float(a1));
  hi = Act<DT>::pack(__uint_as_float(b0), __uint_as_float(b1));
}

// ---------------------------------------------------------------- timing
__device__ __forceinline__ uint64_t gtime_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void raise_error(int* err, int code) {
  if (err) atomicOr(err, code);
}

// ---------------------------------------------------------------- smem / mbarrier
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(bar), "r"(bytes)
               : "memory");
}
// One potentially-suspending test of the phase with the given parity.  The
// suspend-time hint lets the hardware park the thread (no issue slots used)
// until the phase completes or the hint elapses; without it a waiter spins and
// steals issue slots from the producer and MMA threads on its SM sub-partition.
constexpr uint32_t kSuspendHintNs = 20000;
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
// Bounded wait for the phase with the given parity.  Returns false (and sets
// *abort and *err) when the wait gives up or another thread already aborted.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, volatile int* abort, int* err) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime_ns();
  for (;;) {
    if (mbar_try(bar, parity)) return true;
    if (*abort) return false;
    if (gtime_ns() - t0 > LMOE_WAIT_NS) {
      *abort = 1;
      raise_error(err, LMOE_ERR_TIMEOUT);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag (used to drain in-flight copies and
// for the epilogue's own rendezvous).
__device__ __forceinline__ bool mbar_wait_drain(uint32_t bar, uint32_t parity, int* err) {
  if (mbar_try(bar, parity)) return true;
  const uint64_t t0 = gtime_ns();
  while (!mbar_try(bar, parity)) {
    if (gtime_ns() - t0 > LMOE_WAIT_NS) {
      raise_error(err, LMOE_ERR_TIMEOUT);
      return false;
    }
  }
  return true;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ---------------------------------------------------------------- programmatic dependent launch
// A kernel launched with cudaLaunchAttributeProgrammaticStreamSerialization may start
// before the previous kernel in its stream has finished: grid_dep_wait blocks until
// that kernel has completed and its writes are visible (a no-op for a normal
// launch); grid_dep_launch lets this kernel's own dependent start early.  Only reads
// of the previous kernel's output must come after grid_dep_wait: data written by
// earlier work is complete, since the previous kernel itself started after it.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Host: launch `kernel` so that it may start before the previous kernel in `st` ends
// (the kernel calls grid_dep_wait before reading that kernel's output).
template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                              Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

// ---------------------------------------------------------------- TMA / cp.async
__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, uint32_t bar, int c0, int c1, int c2) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(dst),
      "l"((uint64_t)map), "r"(bar), "r"(c0), "r"(c1), "r"(c2)
      : "memory");
}
// One bulk global->shared copy (no tensor map, no multicast): dst and src 16-byte
// aligned, bytes a multiple of 16; completes `bytes` of the barrier's transaction count.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
// bring `bytes` (a multiple of 16, 16-byte aligned source) of global memory into L2 (no
// shared memory, no completion to wait for)
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}
// pull the 128-byte line holding p into L1 (no register written, no wait)
__device__ __forceinline__ void prefetch_l1(const void* p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"((uint64_t)map) : "memory");
}
// 16-byte global->shared copy; src_bytes = 0 writes zeros
__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(src_bytes) : "memory");
}
// 4-byte global->shared copy through L1
__device__ __forceinline__ void cp_async4(uint32_t dst, const void* src) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, kind::f16 (bf16 or f16 inputs, f32 accumulate)
__device__ __forceinline__ void mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// kind::i8 (s8 x s8 -> s32)
__device__ __forceinline__ void mma_i8(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc]^T, kind::f16 with the A operand in tensor memory
// (A: 128 lanes = rows, 8 consecutive 32-bit columns = 16 packed 16-bit K values)
__device__ __forceinline__ void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                           uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p; }" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(acc)
      : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns from registers: thread i writes lane (base_lane + i)
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]),
      "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]),
      "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31])
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// shared-memory vector access by 32-bit shared address
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ void sts128(uint32_t a, uint4 v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(a), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w) : "memory");
}

// arrive on an mbarrier once all previously issued tcgen05 ops of this thread complete
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// 32 lanes x 32 consecutive 32-bit columns: thread i gets lane (base_lane + i)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes grouped 8 at a time (1024-byte swizzle atoms stacked along M/N).
__device__ __forceinline__ uint64_t sdesc_k_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFFu) >> 4);  // start address >> 4, bits [0,14)
  d |= (uint64_t)1 << 16;                     // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;           // stride byte offset: next 8-row group
  d |= (uint64_t)1 << 46;                     // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                     // layout: SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: D=f32, A/B = bf16 (fmt 1) or f16 (fmt 0), both K-major.
__device__ __forceinline__ uint32_t idesc_f16(int ab_fmt, int m, int n) {
  return (1u << 4) | ((uint32_t)ab_fmt << 7) | ((uint32_t)ab_fmt << 10) | ((uint32_t)(n >> 3) << 17) |
         ((uint32_t)(m >> 4) << 24);
}
// Instruction descriptor, kind::i8: D=s32, A/B signed int8, both K-major.
__device__ __forceinline__ uint32_t idesc_i8(int m, int n) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// byte offset of 16-byte chunk c of row r inside a 128B-swizzled K-major tile
__device__ __forceinline__ uint32_t sw128_off(int r, int c) {
  return (uint32_t)(r * 128 + ((c ^ (r & 7)) << 4));
}

__device__ __forceinline__ int warp_id() { return threadIdx.x >> 5; }
__device__ __forceinline__ int lane_id() { return threadIdx.x & 31; }

__device__ __forceinline__ void named_barrier(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

}  // namespace lmoe

// host-side helper
#define LMOE_CUDA_CHECK(expr)                     \
  do {                                            \
    cudaError_t _e = (expr);                      \
    if (_e != cudaSuccess) return LMOE_ERR_CUDA;  \
  } while (0)
