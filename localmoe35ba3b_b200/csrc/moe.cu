// Prefill MoE expert block: routing metadata -> gate_up GEMM (+SwiGLU) ->
// down GEMM (+routing weight) -> ordered combine (+ gated shared expert,
// + optional residual).
//
// Replaces gpu_routes.routed_moe (qwen35_deploy/runtime/gpu_routes.py:66-82)
// and, with the shared-expert arguments, the expert part of the HF
// Qwen3_5MoeSparseMoeBlock.forward (transformers qwen3_5_moe/
// modeling_qwen3_5_moe.py:781-792).  Rounding sequence kept from the
// reference: per route v = round(round(acc) * w) (prefill.py:45), per token
// acc = round(acc + v) over routes in ascending expert order (prefill.py:46),
// then round(acc + round(round(sigmoid(round(x . g))) * shared)) (HF :787-790).
#include "common.cuh"
#include "gemm.cuh"
#include "routes.cuh"

namespace lmoe {



constexpr int kCombineThreads = 256;

template <int DT>
__global__ void __launch_bounds__(kCombineThreads) moe_combine_kernel(
    const typename Act<DT>::T* __restrict__ down, const int32_t* __restrict__ ordered,
    const int32_t* __restrict__ hdr, int top, int64_t H, int64_t R,
    const typename Act<DT>::T* __restrict__ x, const typename Act<DT>::T* __restrict__ gate_w, int with_shared,
    const typename Act<DT>::T* __restrict__ residual, typename Act<DT>::T* __restrict__ out) {
  using A = Act<DT>;
  __shared__ float red[kCombineThreads / 32];
  const int64_t t = blockIdx.x;
  float sig = 1.f;
  if (with_shared && gate_w != nullptr) {
    float part = 0.f;
    for (int64_t c = threadIdx.x * 8; c < H; c += kCombineThreads * 8) {
      const uint4 xv = *reinterpret_cast<const uint4*>(x + t * H + c);
      const uint4 gv = *reinterpret_cast<const uint4*>(gate_w + c);
      const uint32_t xa[4] = {xv.x, xv.y, xv.z, xv.w}, ga[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        part = fmaf(A::lo_f(xa[j]), A::lo_f(ga[j]), part);
        part = fmaf(A::hi_f(xa[j]), A::hi_f(ga[j]), part);
      }
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) part += __shfl_xor_sync(0xffffffffu, part, o);
    if (lane_id() == 0) red[warp_id()] = part;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineThreads / 32; ++w) tot += red[w];
    const float logit = A::round(tot);
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-logit))));
  }
  // the shared gate above reads only the block's input; the rows below are the down
  // kernel's output
  grid_dep_wait();
  grid_dep_launch();
  // routes at sorted positions >= valid have id -1 ("no route"): never computed, skipped
  const int64_t valid = hdr[kHdrValid];
  for (int64_t c = threadIdx.x * 8; c < H; c += kCombineThreads * 8) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int i = 0; i < top; ++i) {
      const int64_t r = ordered[t * top + i];
      if (r >= valid) continue;
      const uint4 v = *reinterpret_cast<const uint4*>(down + r * H + c);
      const uint32_t va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = A::round(__fadd_rn(acc[2 * j], A::lo_f(va[j])));
        acc[2 * j + 1] = A::round(__fadd_rn(acc[2 * j + 1], A::hi_f(va[j])));
      }
    }
    if (with_shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(down + (R + t) * H + c);
      const uint32_t va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float s0 = gate_w ? A::round(__fmul_rn(sig, A::lo_f(va[j]))) : A::lo_f(va[j]);
        const float s1 = gate_w ? A::round(__fmul_rn(sig, A::hi_f(va[j]))) : A::hi_f(va[j]);
        acc[2 * j] = A::round(__fadd_rn(acc[2 * j], s0));
        acc[2 * j + 1] = A::round(__fadd_rn(acc[2 * j + 1], s1));
      }
    }
    if (residual != nullptr) {
      const uint4 v = *reinterpret_cast<const uint4*>(residual + t * H + c);
      const uint32_t va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = A::round(__fadd_rn(A::lo_f(va[j]), acc[2 * j]));
        acc[2 * j + 1] = A::round(__fadd_rn(A::hi_f(va[j]), acc[2 * j + 1]));
      }
    }
    uint4 o;
    o.x = A::pack(acc[0], acc[1]);
    o.y = A::pack(acc[2], acc[3]);
    o.z = A::pack(acc[4], acc[5]);
    o.w = A::pack(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + t * H + c) = o;
  }
}

struct MoeWs {
  int64_t off_meta, off_xs, off_hidden, off_down, bytes;
  MoeWs(int64_t T, int64_t top, int64_t E, int64_t H, int64_t I) {
    const int64_t R = T * top;
    const MetaLayout L(T, top, E);
    off_meta = 0;
    off_xs = MetaLayout::align(L.bytes);  // token rows in route order (+ the shared segment)
    off_hidden = MetaLayout::align(off_xs + (R + T) * H * 2);
    off_down = MetaLayout::align(off_hidden + (R + T) * I * 2);
    bytes = MetaLayout::align(off_down + (R + T) * H * 2);
  }
};

}  // namespace lmoe

using namespace lmoe;

int lmoe_route_meta_impl(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                         int with_shared, void* meta, int* err, cudaStream_t st);

extern "C" int64_t lmoe_moe_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t hidden,
                                           int64_t inter) {
  return MoeWs(tokens, top, experts, hidden, inter).bytes;
}

int lmoe_route_meta_after_counts(const int64_t* ids, const float* weights, int64_t tokens, int64_t top,
                                 int64_t experts, int with_shared, void* meta, int* err, cudaStream_t st);
namespace lmoe {
bool router_gemm_ok(int64_t tokens, int64_t hidden, int64_t experts, int64_t top);
int launch_router_gemm_topk(const void* x, const void* w, int64_t tokens, int64_t hidden, int64_t experts,
                            int64_t top, float* weights, int64_t* ids, float* probs, void* logits, int32_t* counts,
                            void* ws, int dtype, int* err, cudaStream_t st);
int64_t router_gemm_workspace(int64_t tokens, int64_t experts);
}  // namespace lmoe

// The block after the routing: metadata (router_counts: the per-chunk expert counts are
// already in the metadata's scratch), permute, gate_up, down, combine.
static int moe_block_body(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                          const int8_t* qg, const float* sg, const int8_t* qd, const float* sd, int64_t experts,
                          int64_t hidden, int64_t inter, const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu,
                          const float* sh_su, const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w,
                          const void* residual, void* out, int dtype, void* ws, int* err, void** stage_events,
                          cudaStream_t st, bool router_counts);

extern "C" int lmoe_routed_moe(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                               const int8_t* qg, const float* sg, const int8_t* qd, const float* sd, int64_t experts,
                               int64_t hidden, int64_t inter, const int8_t* sh_qg, const float* sh_sg,
                               const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd, const float* sh_sd,
                               const void* sh_gate_w, const void* residual, void* out, int dtype, void* ws, int* err,
                               void** stage_events, void* stream) {
  return moe_block_body(x, weights, ids, tokens, top, qg, sg, qd, sd, experts, hidden, inter, sh_qg, sh_sg, sh_qu,
                        sh_su, sh_qd, sh_sd, sh_gate_w, residual, out, dtype, ws, err, stage_events,
                        (cudaStream_t)stream, false);
}

extern "C" int lmoe_moe_block_router(const void* x, const void* router_w, int64_t tokens, int64_t top,
                                     const int8_t* qg, const float* sg, const int8_t* qd, const float* sd,
                                     int64_t experts, int64_t hidden, int64_t inter, const int8_t* sh_qg,
                                     const float* sh_sg, const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd,
                                     const float* sh_sd, const void* sh_gate_w, const void* residual, void* out,
                                     float* weights, int64_t* ids, int dtype, void* ws, int* err, void* stream) {
  if (!x || !router_w || !weights || !ids || !ws || top <= 0) return LMOE_ERR_INVALID;
  if (!router_gemm_ok(tokens, hidden, experts, top)) return LMOE_ERR_UNSUPPORTED;
  cudaStream_t st = (cudaStream_t)stream;
  const MoeWs W(tokens, top, experts, hidden, inter);
  const MetaLayout ML(tokens, top, experts);
  // a 128-token tile is one metadata chunk when top * 128 == kMetaChunk: the router kernel
  // then writes the chunk's expert counts itself
  const bool fused_counts = top * 128 == kMetaChunk;
  int32_t* cc = fused_counts ? (int32_t*)((char*)ws + W.off_meta + ML.off_scratch) : nullptr;
  // the router's fp32 partial sums go to the down rows' region, which the down GEMM only
  // writes later in the call
  if (router_gemm_workspace(tokens, experts) > W.bytes - W.off_down) return LMOE_ERR_UNSUPPORTED;
  int rc = launch_router_gemm_topk(x, router_w, tokens, hidden, experts, top, weights, ids, nullptr, nullptr, cc,
                                   (char*)ws + W.off_down, dtype, err, st);
  if (rc) return rc;
  return moe_block_body(x, weights, ids, tokens, top, qg, sg, qd, sd, experts, hidden, inter, sh_qg, sh_sg, sh_qu,
                        sh_su, sh_qd, sh_sd, sh_gate_w, residual, out, dtype, ws, err, nullptr, st, fused_counts);
}

static int moe_block_body(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                          const int8_t* qg, const float* sg, const int8_t* qd, const float* sd, int64_t experts,
                          int64_t hidden, int64_t inter, const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu,
                          const float* sh_su, const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w,
                          const void* residual, void* out, int dtype, void* ws, int* err, void** stage_events,
                          cudaStream_t st, bool router_counts) {
  // top == 0 (no routed experts, the gated shared expert alone) is accepted when a shared
  // expert is given: expert-parallel callers compute their own tokens' shared expert this way
  const bool shared_only = top == 0 && sh_qg != nullptr;
  if (!x || (!shared_only && (!weights || !ids)) || !qg || !sg || !qd || !sd || !out || !ws) return LMOE_ERR_INVALID;
  if (tokens <= 0 || top < 0 || (top == 0 && !shared_only) || experts <= 0 || hidden <= 0 || inter <= 0)
    return LMOE_ERR_INVALID;
  if (hidden % kGroup || inter % kGroup || hidden % 8) return LMOE_ERR_INVALID;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return LMOE_ERR_INVALID;
  const bool with_shared = sh_qg != nullptr;
  if (with_shared && (!sh_sg || !sh_qu || !sh_su || !sh_qd || !sh_sd)) return LMOE_ERR_INVALID;
  const MoeWs W(tokens, top, experts, hidden, inter);
  const MetaLayout ML(tokens, top, experts);
  char* w = (char*)ws;
  char* meta = w + W.off_meta;
  void* xs = w + W.off_xs;
  void* hid = w + W.off_hidden;
  void* dn = w + W.off_down;
  const int64_t R = tokens * top;

  // optional stage timing: events[0..4] bracket metadata, gate_up, down, combine
  auto mark = [&](int i) -> int {
    if (stage_events && stage_events[i]) LMOE_CUDA_CHECK(cudaEventRecord((cudaEvent_t)stage_events[i], st));
    return LMOE_OK;
  };
  int rc = mark(0);
  if (rc) return rc;
  if ((rc = router_counts ? lmoe_route_meta_after_counts(ids, weights, tokens, top, experts, with_shared ? 1 : 0, meta,
                                                         err, st)
                          : lmoe_route_meta_impl(ids, weights, tokens, top, experts, with_shared ? 1 : 0, meta, err,
                                                 st)))
    return rc;
  if ((rc = mark(1))) return rc;

  const int64_t rows = R + (with_shared ? tokens : 0);
  if ((rc = launch_permute_rows(x, (const int32_t*)(meta + ML.off_pos), xs, rows, hidden, st))) return rc;

  GemmLaunch g = {};
  g.x = xs;
  g.x_rows = rows;
  g.K = hidden;
  g.tiles = (const Tile*)(meta + ML.off_tiles);
  g.hdr = (const int32_t*)(meta + ML.off_hdr);
  g.grid_tiles = ML.max_tiles;
  g.q_bank = qg;
  g.s_bank = sg;
  g.experts = experts;
  g.N = 2 * inter;
  g.inter = inter;
  if (with_shared) {
    g.q_lo = sh_qg;
    g.s_lo = sh_sg;
    g.q_hi = sh_qu;
    g.s_hi = sh_su;
    g.rows_lo = inter;
    g.rows_hi = inter;
  }
  g.y = hid;
  g.ldy = inter;
  g.mode = kSwiGLU;
  g.dtype = dtype;
  g.err = err;
  if ((rc = launch_swiglu_ts(g, st))) return rc;
  if ((rc = mark(2))) return rc;

  GemmLaunch d = g;
  d.x = hid;
  d.x_rows = rows;
  d.K = inter;
  d.q_bank = qd;
  d.s_bank = sd;
  d.N = hidden;
  d.inter = 0;
  d.q_lo = with_shared ? sh_qd : nullptr;
  d.s_lo = with_shared ? sh_sd : nullptr;
  d.q_hi = nullptr;
  d.s_hi = nullptr;
  d.rows_lo = with_shared ? hidden : 0;
  d.rows_hi = 0;
  d.y = dn;
  d.ldy = hidden;
  d.rweight = (const float*)(meta + ML.off_rweight);
  d.mode = kWeighted;
  if ((rc = launch_down_ts(d, st))) return rc;
  if ((rc = mark(3))) return rc;

  const int32_t* ordered = (const int32_t*)(meta + ML.off_ordered);
  const int32_t* hdr = (const int32_t*)(meta + ML.off_hdr);
  if (dtype == LMOE_BF16)
    LMOE_CUDA_CHECK(launch_pdl(moe_combine_kernel<LMOE_BF16>, dim3((unsigned)tokens), dim3(kCombineThreads), 0, st,
                               (const __nv_bfloat16*)dn, ordered, hdr, (int)top, hidden, R, (const __nv_bfloat16*)x,
                               (const __nv_bfloat16*)sh_gate_w, with_shared ? 1 : 0,
                               (const __nv_bfloat16*)residual, (__nv_bfloat16*)out));
  else
    LMOE_CUDA_CHECK(launch_pdl(moe_combine_kernel<LMOE_F16>, dim3((unsigned)tokens), dim3(kCombineThreads), 0, st,
                               (const __half*)dn, ordered, hdr, (int)top, hidden, R, (const __half*)x,
                               (const __half*)sh_gate_w, with_shared ? 1 : 0, (const __half*)residual,
                               (__half*)out));
  return mark(4);
}

// ============================================================================
// Allocation-free variant of lmoe_routed_moe.
//
// Some callers cannot allocate device memory at the point where they run the
// MoE block: host runtimes that hand out device memory only from a fixed,
// pre-sized arena they do not expose to plug-ins, and C/FFI hosts that link
// this library without any device allocator of their own.  For them the
// scratch space lives in a file-scope __device__ array of a fixed size,
// kNoAllocScratchBytes, which every GPU that loads this library keeps for
// the life of the process.
namespace lmoe {
constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // 16 MiB per device
constexpr int64_t kNoAllocMaxDim = int64_t(1) << 20;        // hidden, inter: keeps the size products in range
static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];
}  // namespace lmoe

#include <mutex>

// Device address of the scratch array in the calling thread's current CUDA
// context.  Host code cannot use the array's name as a pointer (it is a
// host-side stand-in), so the address is looked up with cudaGetSymbolAddress,
// with the caller's device current, the first time a context calls, and cached
// per (context, device).  That first lookup may load the module on the device:
// make the first call on each device (or context) before any stream capture.
typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
static CUcontext current_context() {
  static CtxGetCurrentFn fn = []() -> CtxGetCurrentFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (CtxGetCurrentFn)f;
    return nullptr;
  }();
  CUcontext c = nullptr;
  if (fn == nullptr || fn(&c) != CUDA_SUCCESS) return nullptr;
  return c;
}

static void* noalloc_scratch() {
  struct Entry {
    CUcontext ctx;
    int dev;
    void* ptr;
  };
  static std::mutex mu;
  static Entry cache[64] = {};
  static int next = 0;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0) return nullptr;
  // cudaSetDevice makes the device's primary context current when the thread has none yet
  CUcontext ctx = current_context();
  if (ctx == nullptr) {
    if (cudaSetDevice(dev) != cudaSuccess) return nullptr;
    ctx = current_context();
  }
  std::lock_guard<std::mutex> lock(mu);
  for (const Entry& e : cache)
    if (e.ptr != nullptr && e.ctx == ctx && e.dev == dev) return e.ptr;
  void* p = nullptr;
  if (cudaGetSymbolAddress(&p, lmoe::g_noalloc_scratch) != cudaSuccess || p == nullptr) return nullptr;
  cache[next] = Entry{ctx, dev, p};
  next = (next + 1) % 64;
  return p;
}

extern "C" int64_t lmoe_routed_moe_noalloc_limit(void) { return lmoe::kNoAllocScratchBytes; }

extern "C" int lmoe_routed_moe_noalloc(const void* x, const float* weights, const int64_t* ids, int64_t tokens,
                                       int64_t top, const int8_t* qg, const float* sg, const int8_t* qd,
                                       const float* sd, int64_t experts, int64_t hidden, int64_t inter,
                                       const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu,
                                       const float* sh_su, const int8_t* sh_qd, const float* sh_sd,
                                       const void* sh_gate_w, const void* residual, void* out, int dtype, int* err,
                                       void* stream) {
  if (tokens <= 0 || top < 0 || (top == 0 && sh_qg == nullptr) || experts <= 0 || hidden <= 0 || inter <= 0)
    return LMOE_ERR_INVALID;
  if (tokens > (int64_t(1) << 30) || top > 64 || experts > (int64_t(1) << 20) || hidden > lmoe::kNoAllocMaxDim ||
      inter > lmoe::kNoAllocMaxDim)
    return LMOE_ERR_INVALID;
  // every byte of the scratch that a call reads is written earlier in the same
  // call, so nothing needs clearing between calls
  if (lmoe_moe_workspace_size(tokens, top, experts, hidden, inter) > lmoe::kNoAllocScratchBytes)
    return LMOE_ERR_UNSUPPORTED;
  void* ws = noalloc_scratch();
  if (ws == nullptr) return LMOE_ERR_CUDA;
  return lmoe_routed_moe(x, weights, ids, tokens, top, qg, sg, qd, sd, experts, hidden, inter, sh_qg, sh_sg, sh_qu,
                         sh_su, sh_qd, sh_sd, sh_gate_w, residual, out, dtype, ws, err, nullptr, stream);
}
