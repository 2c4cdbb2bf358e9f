// Device helpers shared by the routing-metadata kernels (routes.cu) and the
// expert-parallel layer kernels (ep.cu): a block-wide inclusive scan and the
// writer of the fused path's tile list and header.
#pragma once
#include "common.cuh"
#include "routes.cuh"

namespace lmoe {

constexpr int kRouteThreads = 1024;
constexpr int kRouteWarps = kRouteThreads / 32;

// inclusive block scan over kRouteThreads values (one per thread)
__device__ __forceinline__ int block_incl_scan(int v, int* warp_tot) {
  const int lane = lane_id(), warp = warp_id();
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int u = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += u;
  }
  if (lane == 31) warp_tot[warp] = v;
  __syncthreads();
  if (warp == 0) {
    int t = warp_tot[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int u = __shfl_up_sync(0xffffffffu, t, o);
      if (lane >= o) t += u;
    }
    warp_tot[lane] = t;
  }
  __syncthreads();
  const int r = v + (warp > 0 ? warp_tot[warp - 1] : 0);
  __syncthreads();
  return r;
}

// Tile list of the fused path and the metadata header, written by all
// kRouteThreads threads of one CTA.  Experts are listed by descending route
// count (ties: lower id first) so the persistent GEMMs take the longest tiles
// first; with_shared appends the shared expert as expert E, whose `tokens` rows
// start at row shared_start.  s_first[e] = first sorted slot of expert e (e <= E;
// s_first[E] = the number of valid routes); `routes` is the header's route count.
// E + 1 <= kRouteThreads.
__device__ __forceinline__ void write_tile_list(int E, int tokens, int with_shared, const int* s_first, int routes,
                                                int shared_start, Tile* tiles, int32_t* hdr, int* warp_tot) {
  __shared__ int s_total_tiles;
  __shared__ int s_by_rank[kRouteThreads + 1];
  __shared__ int s_tile_first[kRouteThreads + 1];
  __shared__ int s_cnt[kRouteThreads + 1];
  __shared__ int s_rank[kRouteThreads + 1];
  const int Es = E + (with_shared ? 1 : 0);
  const int valid = s_first[E];
  const int e = threadIdx.x;
  const int lane = lane_id(), warp = warp_id();
  int cnt = 0, ntl = 0, rank = 0;
  if (e < Es) {
    cnt = (e < E) ? (s_first[e + 1] - s_first[e]) : tokens;
    ntl = (cnt + kTileRoutes - 1) / kTileRoutes;
    s_cnt[e] = cnt;
  }
  __syncthreads();
  // rank of expert x among all: the number of experts with more routes, or as many and a
  // lower id; one warp per expert, its lanes counting over strided subsets of the others
  for (int x = warp; x < Es; x += kRouteWarps) {
    const int cx = s_cnt[x];
    int r = 0;
    for (int o = lane; o < Es; o += 32) {
      const int co = s_cnt[o];
      r += (co > cx) || (co == cx && o < x);
    }
    r = __reduce_add_sync(0xffffffffu, r);
    if (lane == 0) s_rank[x] = r;
  }
  __syncthreads();
  if (e < Es) rank = s_rank[e];
  if (e < Es) s_by_rank[rank] = ntl;
  __syncthreads();
  const int r_ntl = (e < Es) ? s_by_rank[e] : 0;  // thread e now holds rank e's tile count
  const int r_incl = block_incl_scan(r_ntl, warp_tot);
  if (e < Es) s_tile_first[e] = r_incl - r_ntl;
  if (e == Es - 1) s_total_tiles = r_incl;
  __syncthreads();
  if (e < Es) {
    const int t0 = s_tile_first[rank];
    const int start0 = (e < E) ? s_first[e] : shared_start;
    for (int j = 0; j < ntl; ++j) {
      Tile tl;
      tl.expert = e;
      tl.start = start0 + j * kTileRoutes;
      tl.count = min(kTileRoutes, cnt - j * kTileRoutes);
      tl.pad = 0;
      tiles[t0 + j] = tl;
    }
  }
  if (threadIdx.x == 0) {
    hdr[kHdrNumTiles] = Es > 0 ? s_total_tiles : 0;
    hdr[kHdrRoutes] = routes;
    hdr[kHdrTokens] = tokens;
    hdr[kHdrExperts] = E;
    hdr[kHdrShared] = with_shared;
    hdr[kHdrValid] = valid;
  }
}

}  // namespace lmoe
