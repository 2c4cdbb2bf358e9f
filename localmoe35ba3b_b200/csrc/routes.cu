// GPU routing metadata: one single-CTA kernel replaces the torch stable sort,
// searchsorted, cumsum, argsort and scatter of gpu_routes.plan and the
// reference's _table kernel (qwen35_deploy/runtime/gpu_routes.py:17-63).
//
// Algorithm: a stable counting sort of the flat route ids.  The flat array is
// cut into 32 contiguous segments, one per warp.  Pass 1 counts ids per
// (warp, expert) in shared memory; a scan over experts, then over warps,
// gives every (warp, expert) its first sorted slot; pass 2 walks each
// segment in order, 32 routes at a time, ranking equal ids inside the warp
// with __match_any_sync -- so routes of one expert keep their flat order, as
// torch.sort(stable=True) does.  The per-token ascending-expert order
// (argsort(dim=1, stable=True)) comes from each route's rank among its own
// token's top-k ids (smaller id, or equal id and earlier slot), computed in
// the same pass, so `ordered`/`slots` need no second pass over `inverse`.
#include "common.cuh"
#include "routes.cuh"
#include "routes_dev.cuh"

namespace lmoe {

constexpr int kMaxTop = 32;
constexpr int kBatch = 16;  // ids held per lane per batch

__device__ __forceinline__ int clamp_id(int64_t v, int E, int* err) {
  if (v < 0 || v >= E) {
    raise_error(err, 2);
    return E;
  }
  return (int)v;
}

// Fused-path bucket of a route id: -1 is "no route" (a padded slot: an
// expert-parallel owner's received row lists only the routes to its own
// experts); it sorts into bucket E after every expert, like an out-of-range
// id, so it gets no GEMM tile and the combine skips it.  Any other id outside
// [0, E) is flagged.
__device__ __forceinline__ int route_bucket(int64_t v, int E, int* err) {
  if (v < 0 || v >= E) {
    if (v != -1) raise_error(err, 2);
    return E;
  }
  return (int)v;
}

struct RouteArgs {
  const int64_t* ids;
  const float* weights;  // nullable: [T, top] fp32 routing weights
  int T, top, E, with_shared;
  // fused-path outputs (nullable block: hdr == nullptr)
  int32_t* hdr;
  int32_t* offsets;
  Tile* tiles;
  int32_t* pos32;
  float* rweight;
  int32_t* ordered32;
  int32_t* inverse;  // optional [R]: sorted position of each flat route
  // reference-format outputs (nullable)
  int64_t* pos64;
  int64_t* table64;
  int64_t* ordered64;
  int64_t* slots64;
  int bm;
  int max_tiles_ref;
  int* err;
};

__global__ void __launch_bounds__(kRouteThreads) route_kernel(RouteArgs a) {
  extern __shared__ int cw[];  // [kRouteWarps][E+1] counts, then first slots
  __shared__ int warp_tot[32];
  const int R = a.T * a.top;
  const int E = a.E;
  const int Es = E + (a.with_shared ? 1 : 0);  // ranked experts incl. shared
  const int lane = lane_id(), warp = warp_id();
  const int L = (R + kRouteWarps - 1) / kRouteWarps;
  const int seg_lo = warp * L;
  const int seg_hi = min(R, seg_lo + L);

  for (int i = threadIdx.x; i < kRouteWarps * (E + 1); i += blockDim.x) cw[i] = 0;
  __syncthreads();
  // pass 1: per-warp counts (out-of-range ids are counted in bucket E and
  // flagged).  Ids are fetched kBatch per lane at a time so the loads overlap.
  for (int base = seg_lo; base < seg_hi; base += 32 * kBatch) {
    int idv[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int f = base + i * 32 + lane;
      idv[i] = (f < seg_hi) ? clamp_id(a.ids[f], E, a.err) : -1;
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i)
      if (idv[i] >= 0) atomicAdd(&cw[warp * (E + 1) + idv[i]], 1);
  }
  __syncthreads();
  // per expert: exclusive over warps, then exclusive over experts
  int count = 0;
  const int e = threadIdx.x;
  if (e <= E) {
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = cw[w * (E + 1) + e];
      cw[w * (E + 1) + e] = count;
      count += c;
    }
  }
  // E + 1 <= kRouteThreads is checked on the host
  const int incl = block_incl_scan(e <= E ? count : 0, warp_tot);
  const int first = incl - (e <= E ? count : 0);
  if (e <= E) {
    for (int w = 0; w < kRouteWarps; ++w) cw[w * (E + 1) + e] += first;
    if (a.offsets != nullptr && e < E) a.offsets[e] = first;
  }
  if (a.offsets != nullptr && e == 0) {
    a.offsets[E] = R;
    a.offsets[E + 1] = R + (a.with_shared ? a.T : 0);
  }
  __syncthreads();

  // pass 2: stable placement
  const unsigned lt = (1u << lane) - 1u;
  for (int base = seg_lo; base < seg_hi; base += 32 * kBatch) {
    int idv[kBatch];
    float wv[kBatch];
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int f = base + i * 32 + lane;
      idv[i] = (f < seg_hi) ? clamp_id(a.ids[f], E, nullptr) : -1;
      wv[i] = (f < seg_hi && a.weights) ? a.weights[f] : 1.0f;
    }
#pragma unroll
    for (int i = 0; i < kBatch; ++i) {
      const int f = base + i * 32 + lane;
      const bool valid = idv[i] >= 0;
      const int id = idv[i];
      const unsigned peers = __match_any_sync(0xffffffffu, id);
      int dst = 0;
      if (valid) dst = cw[warp * (E + 1) + id] + __popc(peers & lt);
      __syncwarp();
      if (valid) {
        const int tok = f / a.top;
        const int slot = f - tok * a.top;
        // rank of this route among its token's routes, ordered by (id, slot)
        const int64_t* trow = a.ids + (int64_t)tok * a.top;
        int rank = 0;
        for (int j = 0; j < a.top; ++j) {
          const int64_t oj = trow[j];
          const int idj = (oj < 0 || oj >= E) ? E : (int)oj;
          rank += (idj < id) || (idj == id && j < slot);
        }
        const int64_t o = (int64_t)tok * a.top + rank;
        if (a.inverse) a.inverse[f] = dst;
        if (a.pos32) a.pos32[dst] = tok;
        if (a.pos64) a.pos64[dst] = tok;
        if (a.rweight) a.rweight[dst] = wv[i];
        if (a.ordered32) a.ordered32[o] = dst;
        if (a.ordered64) a.ordered64[o] = dst;
        if (a.slots64) a.slots64[o] = slot;
        if (lane == 31 - __clz(peers)) cw[warp * (E + 1) + id] += __popc(peers);
      }
      __syncwarp();
    }
  }
  if (a.pos32 && a.with_shared)
    for (int t = threadIdx.x; t < a.T; t += blockDim.x) a.pos32[R + t] = t;
  __syncthreads();

  // counts again, per expert (from offsets held in cw row 0 + totals)
  // cw[0][e] was advanced by warp 0's routes; recompute counts from the scan
  // values instead: count(e) = first(e+1) - first(e).
  __shared__ int s_first[1025];
  if (e <= E) s_first[e] = first;
  if (e == 0) s_first[E + 1] = R;
  __syncthreads();

  // fused-path tiles, experts ordered by descending count (ties: lower id first)
  if (a.tiles != nullptr) write_tile_list(a.E, a.T, a.with_shared, s_first, R, R, a.tiles, a.hdr, warp_tot);

  // reference table: ends = cumsum(ceil(count / bm)) in expert-id order
  if (a.table64 != nullptr) {
    const int cnt = (e < E) ? (s_first[e + 1] - s_first[e]) : 0;
    const int nt = (cnt + a.bm - 1) / a.bm;
    const int ends_incl = block_incl_scan(e < E ? nt : 0, warp_tot);
    __shared__ int s_ends[1025];
    if (e < E) s_ends[e] = ends_incl;
    __syncthreads();
    const int total = s_ends[E - 1];
    for (int tile = threadIdx.x; tile < a.max_tiles_ref; tile += blockDim.x) {
      int64_t ex = 0, st = 0, sp = 0;
      if (tile < total) {
        int lo = 0, hi = E;  // first expert with ends > tile
        while (lo < hi) {
          const int mid = (lo + hi) >> 1;
          if (s_ends[mid] <= tile) lo = mid + 1; else hi = mid;
        }
        ex = lo;
        const int prior = lo > 0 ? s_ends[lo - 1] : 0;
        st = (int64_t)s_first[lo] + (int64_t)(tile - prior) * a.bm;
        sp = s_first[lo + 1];
      }
      a.table64[(int64_t)tile * 3] = ex;
      a.table64[(int64_t)tile * 3 + 1] = st;
      a.table64[(int64_t)tile * 3 + 2] = sp;
    }
  }
}

// ---------------------------------------------------------------------------
// Fused-path metadata on many CTAs (lmoe_route_meta): the same stable counting
// sort, cut into kMetaChunk-route chunks so every chunk runs on its own CTA.
//   1. meta_count_kernel  per-chunk expert histograms
//   2. meta_scan_kernel   (one CTA) exclusive scans over chunks and experts give
//                         every (chunk, expert) its first sorted slot; offsets,
//                         tile list, header, the shared expert's rows
//   3. meta_place_kernel  per chunk: ranks inside each warp (__match_any_sync),
//                         a scan over the chunk's warps, then each route's slot;
//                         the per-token ascending-expert order as in route_kernel
__global__ void __launch_bounds__(kMetaChunk) meta_count_kernel(const int64_t* __restrict__ ids, int R, int E,
                                                                int32_t* __restrict__ cc, int* err) {
  extern __shared__ int h[];  // [E + 1]
  grid_dep_wait();  // ids may be the previous kernel's output (the router)
  grid_dep_launch();
  for (int i = threadIdx.x; i <= E; i += kMetaChunk) h[i] = 0;
  __syncthreads();
  const int f = blockIdx.x * kMetaChunk + threadIdx.x;
  if (f < R) atomicAdd(&h[route_bucket(ids[f], E, err)], 1);
  __syncthreads();
  for (int i = threadIdx.x; i <= E; i += kMetaChunk) cc[(int64_t)blockIdx.x * (E + 1) + i] = h[i];
}

__global__ void __launch_bounds__(kRouteThreads) meta_scan_kernel(RouteArgs a, int32_t* __restrict__ cc,
                                                                  int nchunks) {
  __shared__ int warp_tot[32];
  __shared__ int s_first[1025];
  grid_dep_wait();  // the chunk counts of meta_count_kernel
  grid_dep_launch();
  const int E = a.E, R = a.T * a.top;
  const int e = threadIdx.x;
  // per expert: its total over the chunks (loads in independent batches, so the
  // chunk counts' latencies overlap), then the block scan over experts, then each
  // chunk's first slot written in a second batched pass
  constexpr int kB = 16;
  int count = 0;
  if (e <= E) {
    for (int c0 = 0; c0 < nchunks; c0 += kB) {
      int v[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) v[i] = c0 + i < nchunks ? cc[(int64_t)(c0 + i) * (E + 1) + e] : 0;
#pragma unroll
      for (int i = 0; i < kB; ++i) count += v[i];
    }
  }
  const int incl = block_incl_scan(e <= E ? count : 0, warp_tot);
  const int first = incl - (e <= E ? count : 0);
  if (e <= E) {
    int run = first;
    for (int c0 = 0; c0 < nchunks; c0 += kB) {
      int v[kB];
#pragma unroll
      for (int i = 0; i < kB; ++i) v[i] = c0 + i < nchunks ? cc[(int64_t)(c0 + i) * (E + 1) + e] : 0;
#pragma unroll
      for (int i = 0; i < kB; ++i)
        if (c0 + i < nchunks) {
          cc[(int64_t)(c0 + i) * (E + 1) + e] = run;
          run += v[i];
        }
    }
    s_first[e] = first;
    if (e < E) a.offsets[e] = first;
  }
  if (e == 0) {
    s_first[E + 1] = R;
    a.offsets[E] = R;
    a.offsets[E + 1] = R + (a.with_shared ? a.T : 0);
  }
  if (a.with_shared)
    for (int t = threadIdx.x; t < a.T; t += kRouteThreads) a.pos32[R + t] = t;
  __syncthreads();
  write_tile_list(E, a.T, a.with_shared, s_first, R, R, a.tiles, a.hdr, warp_tot);
}

__global__ void __launch_bounds__(kMetaChunk) meta_place_kernel(RouteArgs a, const int32_t* __restrict__ cc) {
  extern __shared__ int wc[];  // [kMetaChunk / 32][E + 1] per-warp counts, then first slots
  grid_dep_wait();  // the offsets of meta_scan_kernel
  grid_dep_launch();
  constexpr int kW = kMetaChunk / 32;
  const int E = a.E, R = a.T * a.top;
  const int lane = lane_id(), warp = warp_id();
  for (int i = threadIdx.x; i < kW * (E + 1); i += kMetaChunk) wc[i] = 0;
  __syncthreads();
  const int f = blockIdx.x * kMetaChunk + threadIdx.x;
  const bool valid = f < R;
  const int id = valid ? clamp_id(a.ids[f], E, nullptr) : -1;
  const unsigned peers = __match_any_sync(0xffffffffu, id);
  const int rank_w = __popc(peers & ((1u << lane) - 1u));
  if (valid && lane == __ffs(peers) - 1) wc[warp * (E + 1) + id] = __popc(peers);
  __syncthreads();
  if (threadIdx.x <= E) {
    int run = cc[(int64_t)blockIdx.x * (E + 1) + threadIdx.x];
    for (int w = 0; w < kW; ++w) {
      const int t = wc[w * (E + 1) + threadIdx.x];
      wc[w * (E + 1) + threadIdx.x] = run;
      run += t;
    }
  }
  __syncthreads();
  if (!valid) return;
  const int dst = wc[warp * (E + 1) + id] + rank_w;
  const int tok = f / a.top;
  const int slot = f - tok * a.top;
  // rank of this route among its token's routes, ordered by (id, slot)
  const int64_t* trow = a.ids + (int64_t)tok * a.top;
  int rank = 0;
  for (int j = 0; j < a.top; ++j) {
    const int64_t oj = trow[j];
    const int idj = (oj < 0 || oj >= E) ? E : (int)oj;
    rank += (idj < id) || (idj == id && j < slot);
  }
  a.inverse[f] = dst;
  a.pos32[dst] = tok;
  a.rweight[dst] = a.weights ? a.weights[f] : 1.0f;
  a.ordered32[(int64_t)tok * a.top + rank] = dst;
}

static size_t route_smem(int64_t E) { return (size_t)kRouteWarps * (E + 1) * sizeof(int); }

static int launch_route(RouteArgs& a, cudaStream_t st) {
  // static shared arrays (~16.5 KB) plus this dynamic part exceed the 48 KB
  // default, so the opt-in limit is always raised to the dynamic size
  const size_t smem = route_smem(a.E);
  LMOE_CUDA_CHECK(cudaFuncSetAttribute(route_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  route_kernel<<<1, kRouteThreads, smem, st>>>(a);
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

static bool route_geometry_ok(int64_t tokens, int64_t top, int64_t experts) {
  return tokens > 0 && top > 0 && top <= kMaxTop && experts > 0 && experts + 2 <= kRouteThreads &&
         tokens * top < (int64_t(1) << 30) && route_smem(experts) <= 200 * 1024;
}

}  // namespace lmoe

using namespace lmoe;

extern "C" int64_t lmoe_plan_workspace_size(int64_t tokens, int64_t top, int64_t experts) {
  (void)experts;
  return MetaLayout::align(tokens * top * 4) + 256;
}

extern "C" int lmoe_plan(const int64_t* ids, int64_t tokens, int64_t top, int64_t experts, int64_t bm, int64_t* pos,
                         int64_t* table, int64_t* ordered, int64_t* slots, void* ws, void* stream) {
  if (!ids || !pos || !table || !ordered || !slots || !ws || bm <= 0) return LMOE_ERR_INVALID;
  if (!route_geometry_ok(tokens, top, experts)) return LMOE_ERR_INVALID;
  RouteArgs a = {};
  a.ids = ids;
  a.T = (int)tokens;
  a.top = (int)top;
  a.E = (int)experts;
  a.inverse = (int32_t*)ws;
  a.err = (int*)((char*)ws + MetaLayout::align(tokens * top * 4));
  a.pos64 = pos;
  a.table64 = table;
  a.ordered64 = ordered;
  a.slots64 = slots;
  a.bm = (int)bm;
  a.max_tiles_ref = (int)((tokens * top + bm - 1) / bm + experts);
  return launch_route(a, (cudaStream_t)stream);
}

extern "C" int64_t lmoe_route_meta_size(int64_t tokens, int64_t top, int64_t experts) {
  return MetaLayout(tokens, top, experts).bytes;
}

// counts_ready: the per-chunk expert counts are already in the metadata's scratch (the
// fused router kernel wrote them), so the count kernel is skipped
static int route_meta_launch(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                             int with_shared, void* meta, int* err, cudaStream_t st, bool counts_ready) {
  // top == 0 with the shared expert: no routes, only the shared expert's tiles
  const bool shared_only = top == 0 && with_shared;
  if ((!ids && !shared_only) || !meta) return LMOE_ERR_INVALID;
  if (!route_geometry_ok(tokens, shared_only ? 1 : top, experts)) return LMOE_ERR_INVALID;
  const MetaLayout L(tokens, top, experts);
  char* m = (char*)meta;
  RouteArgs a = {};
  a.ids = ids;
  a.weights = weights;
  a.T = (int)tokens;
  a.top = (int)top;
  a.E = (int)experts;
  a.with_shared = with_shared ? 1 : 0;
  a.hdr = (int32_t*)(m + L.off_hdr);
  a.offsets = (int32_t*)(m + L.off_offsets);
  a.tiles = (Tile*)(m + L.off_tiles);
  a.pos32 = (int32_t*)(m + L.off_pos);
  a.rweight = (float*)(m + L.off_rweight);
  a.ordered32 = (int32_t*)(m + L.off_ordered);
  a.inverse = (int32_t*)(m + L.off_inverse);
  a.err = err;
  int32_t* cc = (int32_t*)(m + L.off_scratch);
  const int R = (int)(tokens * top);
  const int nchunks = (R + kMetaChunk - 1) / kMetaChunk;
  const size_t hsm = (size_t)(experts + 1) * sizeof(int);
  const size_t wsm = (size_t)(kMetaChunk / 32) * (experts + 1) * sizeof(int);
  if (nchunks > 0 && !counts_ready) {
    LMOE_CUDA_CHECK(launch_pdl(meta_count_kernel, dim3(nchunks), dim3(kMetaChunk), hsm, st, ids, R, (int)experts, cc,
                               err));
  }
  LMOE_CUDA_CHECK(launch_pdl(meta_scan_kernel, dim3(1), dim3(kRouteThreads), 0, st, a, cc, nchunks));
  if (nchunks > 0) {
    if (wsm > 48 * 1024)
      LMOE_CUDA_CHECK(cudaFuncSetAttribute(meta_place_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)wsm));
    LMOE_CUDA_CHECK(launch_pdl(meta_place_kernel, dim3(nchunks), dim3(kMetaChunk), wsm, st, a, cc));
  }
  return LMOE_OK;
}

int lmoe_route_meta_impl(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                         int with_shared, void* meta, int* err, cudaStream_t st) {
  return route_meta_launch(ids, weights, tokens, top, experts, with_shared, meta, err, st, false);
}

int lmoe_route_meta_after_counts(const int64_t* ids, const float* weights, int64_t tokens, int64_t top,
                                 int64_t experts, int with_shared, void* meta, int* err, cudaStream_t st) {
  return route_meta_launch(ids, weights, tokens, top, experts, with_shared, meta, err, st, true);
}

extern "C" int lmoe_route_meta(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                               int with_shared, void* meta, void* stream) {
  return lmoe_route_meta_impl(ids, weights, tokens, top, experts, with_shared, meta, nullptr, (cudaStream_t)stream);
}
