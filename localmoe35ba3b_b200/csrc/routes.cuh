// Routing-metadata layout shared by the route kernel and its consumers.
#pragma once
#include <stdint.h>

namespace lmoe {

constexpr int kTileRoutes = 128;  // routes (tokens) per GEMM tile: the MMA M extent
constexpr int kMetaChunk = 1024;  // routes per CTA in the multi-CTA metadata kernels

struct __align__(16) Tile {
  int32_t expert;  // expert id; == experts for the shared-expert segment
  int32_t start;   // first route row of the tile (rows are sorted by expert)
  int32_t count;   // valid routes in the tile, 1..kTileRoutes
  int32_t pad;
};

// Byte layout of the metadata buffer written by lmoe_route_meta.  Every
// section starts on a 256-byte boundary.
struct MetaLayout {
  int64_t routes, tokens, top, experts, max_tiles;
  int64_t off_hdr, off_offsets, off_tiles, off_pos, off_rweight, off_ordered, off_inverse, off_scratch, bytes;

  __host__ __device__ static int64_t align(int64_t v) { return (v + 255) & ~int64_t(255); }
  __host__ __device__ MetaLayout(int64_t t, int64_t k, int64_t e) : routes(t * k), tokens(t), top(k), experts(e) {
    max_tiles = (routes + kTileRoutes - 1) / kTileRoutes + e + (t + kTileRoutes - 1) / kTileRoutes + 1;
    int64_t o = 0;
    off_hdr = o;      o = align(o + 16 * 4);
    off_offsets = o;  o = align(o + (e + 2) * 4);
    off_tiles = o;    o = align(o + max_tiles * (int64_t)sizeof(Tile));
    off_pos = o;      o = align(o + (routes + t) * 4);
    off_rweight = o;  o = align(o + routes * 4);
    off_ordered = o;  o = align(o + routes * 4);
    off_inverse = o;  o = align(o + routes * 4);
    off_scratch = o;  o = align(o + ((routes + kMetaChunk - 1) / kMetaChunk) * (e + 1) * 4);  // per-chunk counts
    bytes = o;
  }
};

// header words; kHdrValid = routes with an expert id in [0, experts) (sorted first)
enum { kHdrNumTiles = 0, kHdrRoutes = 1, kHdrTokens = 2, kHdrExperts = 3, kHdrShared = 4, kHdrValid = 5 };

}  // namespace lmoe
