// Expert-parallel MoE layer: the kernels on each side of the two all-to-all
// exchanges, with every exchange size fixed in advance (no host
// synchronisation inside a layer).
//
// The reference runs the MoE block on one GPU (gpu_routes.routed_moe,
// qwen35_deploy/runtime/gpu_routes.py:66-82, inside the HF block,
// transformers qwen3_5_moe/modeling_qwen3_5_moe.py:781-792); here the E
// experts are sharded over W ranks in contiguous blocks of e_loc = E / W and
// each rank keeps its own T tokens.  One layer:
//
//   sender   the routing metadata kernels: a stable counting sort of this rank's
//                                routes by expert (a route's rank among this sender's
//                                routes to its expert, in flat route order)
//            ep_slots_kernel     per (token, rank): the token's row index in that
//                                rank's segment (tokens ascending); the segment headers
//            ep_pack_kernel      one packed row per (token, destination)
//   ---- all_to_all of W segments of (cap + 1) rows each (row 0 = header) ----
//   owner    ep_owner_meta_kernel  per local expert: first sorted slot, and per
//                                (sender, expert) its base; tile list + header of
//                                the fused path (the shared expert's T rows after
//                                the valid routes)
//            ep_owner_scatter_kernel  each received route's sorted slot = base +
//                                rank (no sort on the owner); its routing weight;
//                                the row's payload (int8 wire: dequantised) into
//                                the route-order activation rows; own tokens into
//                                the shared expert's rows
//            gate_up (+SwiGLU) and down (+routing weight) on the TMEM-operand
//                                grouped GEMM, the shared expert's tiles included
//            ep_owner_combine_kernel  per received row: its routes summed in
//                                ascending expert order, acc = round(acc + v)
//   ---- all_to_all of the pre-reduced rows back to their senders ----
//   sender   ep_fold_kernel      per token: the returned rows in ascending rank
//                                order, then round(sigmoid(round(x . g)) * shared),
//                                then the residual
//
// A packed row is [payload | local expert ids int32 x top | weights fp32 x top |
// ranks int32 x top], padded to 16 bytes; the payload is the hidden row in the
// activation dtype or its W8A8 activation quantisation (int8 [H], fp32 scales
// [H/128], as w8a8.quantize, qwen35_deploy/operators/w8a8.py:8-22).  The route
// slots of a row are in ascending local expert id, -1 after the last.  A
// segment header row holds the segment's row count and, per local expert of
// the destination, how many routes it carries.
//
// Rounding sequence: per route round(round(down) * w) (prefill.py:45), per
// (token, rank) the routes in ascending expert order, per token the ranks in
// ascending order (= ascending expert order), then the shared expert and the
// residual (HF :787-790) -- the reference's single chain except that a
// rank's partial sum is added as one term.
#include <string.h>

#include "common.cuh"
#include "gemm.cuh"
#include "gemv.cuh"
#include "routes.cuh"
#include "routes_dev.cuh"

namespace lmoe {

constexpr int kEpMaxWorld = 8;
constexpr int kEpMaxTop = 16;
constexpr int kEpWarps = 8;          // warps per CTA of the row kernels
constexpr int kEpCombineThreads = 256;

struct EpGeom {
  int64_t T, top, E, W, e_loc, cap, H, I;
  int int8, dtype;
  int64_t payload, row_bytes, seg_rows, r_max, max_tiles;
  __host__ __device__ static int64_t a16(int64_t v) { return (v + 15) & ~int64_t(15); }
  __host__ __device__ EpGeom(int64_t t, int64_t k, int64_t e, int64_t w, int64_t c, int64_t h, int64_t i, int wire,
                             int dt)
      : T(t), top(k), E(e), W(w), e_loc(e / w), cap(c), H(h), I(i), int8(wire == LMOE_WIRE_INT8 ? 1 : 0), dtype(dt) {
    payload = int8 ? H + 4 * (H / kGroup) : 2 * H;
    row_bytes = a16(payload + 12 * top);
    seg_rows = cap + 1;
    r_max = W * cap * top;
    max_tiles = (r_max + kTileRoutes - 1) / kTileRoutes + e_loc + (T + kTileRoutes - 1) / kTileRoutes + 1;
  }
};

// owner workspace: metadata, then the route-order activation rows, the SwiGLU
// rows and the weighted down rows (r_max routes + the T shared-expert rows)
struct EpOwnerWs {
  int64_t off_hdr, off_tiles, off_base, off_rweight, off_ordered, off_xs, off_hidden, off_down, bytes;
  explicit EpOwnerWs(const EpGeom& g) {
    int64_t o = 0;
    off_hdr = o;      o = MetaLayout::align(o + 16 * 4);
    off_tiles = o;    o = MetaLayout::align(o + g.max_tiles * (int64_t)sizeof(Tile));
    off_base = o;     o = MetaLayout::align(o + g.W * g.e_loc * 4);
    off_rweight = o;  o = MetaLayout::align(o + g.r_max * 4);
    off_ordered = o;  o = MetaLayout::align(o + g.W * g.cap * g.top * 4);
    off_xs = o;       o = MetaLayout::align(o + (g.r_max + g.T) * g.H * 2);
    off_hidden = o;   o = MetaLayout::align(o + (g.r_max + g.T) * g.I * 2);
    off_down = o;     o = MetaLayout::align(o + (g.r_max + g.T) * g.H * 2);
    bytes = o;
  }
};

// sender plan workspace: the routing metadata of this rank's routes (the stable
// counting sort of the multi-CTA metadata kernels: per expert its first sorted slot,
// per route its sorted slot -- the rank of a route among this sender's routes to the
// same expert is the difference), then slot_of [T, W] int32
struct EpPlanWs {
  int64_t off_meta, off_slot, bytes;
  explicit EpPlanWs(const EpGeom& g) {
    off_meta = 0;
    off_slot = MetaLayout::align(MetaLayout(g.T, g.top, g.E).bytes);
    bytes = MetaLayout::align(off_slot + g.T * g.W * 4);
  }
};

__device__ __forceinline__ bool ep_valid_id(int64_t v, int64_t E) { return v >= 0 && v < E; }

// Direct transport (p2p != 0): every rank's receive and return buffers and flag words,
// mapped into this process (peers' through CUDA IPC).  The sender's pack kernel
// stores its rows straight into the destination's receive buffer and the owner's
// combine kernel its rows straight into the sender's return buffer, over NVLink;
// when a kernel's last CTA is done it raises the flag of this rank on each peer to the
// layer's epoch, and the receiving kernel waits (bounded) for every peer's flag.
// p2p == 0: the caller moves the segments between the kernels (e.g. NCCL all_to_all).
struct EpPeers {
  uint8_t* recv[kEpMaxWorld];
  uint8_t* back[kEpMaxWorld];
  unsigned* flags[kEpMaxWorld];  // [0, W): dispatch from rank s arrived; [W, 2W): returns from rank d
  unsigned* counter;             // this rank's last-CTA counters (pack, combine); zero between calls
  int rank;
  unsigned epoch;
  int p2p;
};

__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Called by every thread of every CTA at the end of a kernel whose stores went to the
// peers: the last CTA to finish raises flag word `slot` on every peer to the epoch.
__device__ __forceinline__ void ep_signal_peers(const EpPeers& P, int W, int which, int slot) {
  __shared__ int s_last;
  __threadfence_system();
  __syncthreads();
  if (threadIdx.x == 0) {
    const unsigned old = atomicAdd(P.counter + which, 1u);
    s_last = old == gridDim.x - 1;
    if (s_last) atomicExch(P.counter + which, 0u);
  }
  __syncthreads();
  if (s_last && (int)threadIdx.x < W) {
    __threadfence_system();
    st_release_sys(P.flags[threadIdx.x] + slot, P.epoch);
  }
}

// Every rank's flag word [base + s] of this rank reaches the epoch (bounded wait by
// threads 0..W-1); false after a timeout (LMOE_DEVERR_TIMEOUT raised).
__device__ __forceinline__ bool ep_wait_peers(const EpPeers& P, int W, int base, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < W) {
    const unsigned* f = P.flags[P.rank] + base + threadIdx.x;
    const uint64_t t0 = gtime_ns();
    while ((int)(ld_acquire_sys(f) - P.epoch) < 0) {
      if (gtime_ns() - t0 > LMOE_WAIT_NS) {
        raise_error(err, LMOE_DEVERR_TIMEOUT);
        s_ok = 0;
        break;
      }
    }
  }
  __syncthreads();
  return s_ok != 0;
}



// ---------------------------------------------------------------------------
// Sender slots (one CTA of kRouteThreads threads): per destination rank d, each
// token's row in segment d = the number of earlier tokens with a route to d (-1 when
// it has none); the segment headers [rows to d, routes per local expert of d] (the
// latter from the routing metadata's per-expert offsets).  Warp w takes a contiguous
// run of tokens, 32 at a time (lane = token); a destination's ballot ranks the
// batch's tokens.
__global__ void __launch_bounds__(kRouteThreads) ep_slots_kernel(const int64_t* __restrict__ ids, EpGeom g,
                                                                 const int32_t* __restrict__ offsets,
                                                                 int32_t* __restrict__ slot_of,
                                                                 uint8_t* __restrict__ send, const EpPeers P) {
  // segment d of this rank: the local send buffer, or (direct transport) segment
  // `rank` of rank d's receive buffer
  auto seg = [&](int64_t d) -> uint8_t* {
    return P.p2p ? P.recv[d] + (int64_t)P.rank * g.seg_rows * g.row_bytes : send + d * g.seg_rows * g.row_bytes;
  };
  extern __shared__ uint8_t s_mask[];  // [T] destination bits per token
  __shared__ int s_cnt[kRouteWarps][kEpMaxWorld];
  const int T = (int)g.T, top = (int)g.top, E = (int)g.E, W = (int)g.W, e_loc = (int)g.e_loc;
  const int lane = lane_id(), warp = warp_id();
  const int S = (T + kRouteWarps - 1) / kRouteWarps;
  const int t_lo = min(T, warp * S), t_hi = min(T, t_lo + S);
  const unsigned lt = (1u << lane) - 1u;
  int cnt[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) cnt[d] = 0;
  for (int b = t_lo; b < t_hi; b += 32) {
    const int t = b + lane;
    unsigned mask = 0;
    if (t < t_hi) {
      int64_t v[kEpMaxTop];
#pragma unroll
      for (int j = 0; j < kEpMaxTop; ++j) v[j] = j < top ? ids[(int64_t)t * top + j] : -1;
#pragma unroll
      for (int j = 0; j < kEpMaxTop; ++j)
        if (ep_valid_id(v[j], E)) mask |= 1u << (int)(v[j] / e_loc);
      s_mask[t] = (uint8_t)mask;
    }
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) cnt[d] += __popc(__ballot_sync(0xffffffffu, (mask >> d) & 1u));
  }
  if (lane == 0)
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) s_cnt[warp][d] = cnt[d];
  __syncthreads();
  if (threadIdx.x < W) {  // exclusive over warps, per destination
    const int d = threadIdx.x;
    int run = 0;
    for (int w = 0; w < kRouteWarps; ++w) {
      const int c = s_cnt[w][d];
      s_cnt[w][d] = run;
      run += c;
    }
    reinterpret_cast<int32_t*>(seg(d))[0] = run;
  }
  for (int e = threadIdx.x; e < E; e += kRouteThreads) {
    const int d = e / e_loc;
    reinterpret_cast<int32_t*>(seg(d))[1 + (e - d * e_loc)] = offsets[e + 1] - offsets[e];
  }
  __syncthreads();
  int base[kEpMaxWorld];
#pragma unroll
  for (int d = 0; d < kEpMaxWorld; ++d) base[d] = d < W ? s_cnt[warp][d] : 0;
  for (int b = t_lo; b < t_hi; b += 32) {
    const int t = b + lane;
    const unsigned mask = t < t_hi ? s_mask[t] : 0u;
#pragma unroll
    for (int d = 0; d < kEpMaxWorld; ++d) {
      if (d >= W) break;
      const unsigned bal = __ballot_sync(0xffffffffu, (mask >> d) & 1u);
      if (t < t_hi) slot_of[(int64_t)t * W + d] = ((mask >> d) & 1u) ? base[d] + __popc(bal & lt) : -1;
      base[d] += __popc(bal);
    }
  }
}

// ---------------------------------------------------------------------------
// Sender pack: one warp per (token, destination) pair that is sent.
template <int DT, bool INT8>
__global__ void __launch_bounds__(32 * kEpWarps) ep_pack_kernel(const typename Act<DT>::T* __restrict__ x,
                                                                const int64_t* __restrict__ ids,
                                                                const float* __restrict__ wts, EpGeom g,
                                                                const int32_t* __restrict__ slot_of,
                                                                const int32_t* __restrict__ inverse,
                                                                const int32_t* __restrict__ offsets,
                                                                uint8_t* __restrict__ send, const EpPeers P) {
  const int lane = lane_id();
  // a persistent grid: each warp takes (token, destination) pairs in turn, so that the
  // direct transport's end-of-kernel fence and signal run once per CTA, not per row
  for (int64_t task = (int64_t)blockIdx.x * kEpWarps + warp_id(); task < g.T * g.W;
       task += (int64_t)gridDim.x * kEpWarps) {
  const int64_t t = task / g.W, d = task - t * g.W;
  const int slot = slot_of[task];
  if (slot >= 0) {
  uint8_t* row = (P.p2p ? P.recv[d] + (int64_t)P.rank * g.seg_rows * g.row_bytes : send + d * g.seg_rows * g.row_bytes) +
                 (1 + slot) * g.row_bytes;
  const int top = (int)g.top;
  // the token's routes to rank d, sorted by local expert id; a route's rank among this
  // sender's routes to its expert = its sorted slot - the expert's first slot
  int lid = 0x7fffffff;
  bool mine = false;
  float w = 0.f;
  int rk = 0;
  if (lane < top) {
    const int64_t v = ids[t * top + lane];
    if (ep_valid_id(v, g.E) && v / g.e_loc == d) {
      mine = true;
      lid = (int)(v - d * g.e_loc);
      w = wts[t * top + lane];
      rk = inverse[t * top + lane] - offsets[v];
    }
  }
  int pos = 0;
  for (int k = 0; k < top; ++k) {
    const int ol = __shfl_sync(0xffffffffu, lid, k);
    const int om = __shfl_sync(0xffffffffu, mine ? 1 : 0, k);
    pos += om && (ol < lid || (ol == lid && k < lane));
  }
  const int nmine = __popc(__ballot_sync(0xffffffffu, mine));
  int32_t* rid = reinterpret_cast<int32_t*>(row + g.payload);
  float* rw = reinterpret_cast<float*>(row + g.payload + 4 * top);
  int32_t* rr = reinterpret_cast<int32_t*>(row + g.payload + 8 * top);
  if (mine) {
    rid[pos] = lid;
    rw[pos] = w;
    rr[pos] = rk;
  }
  if (lane < top && lane >= nmine) {
    rid[lane] = -1;
    rw[lane] = 0.f;
    rr[lane] = 0;
  }
  const typename Act<DT>::T* xr = x + t * g.H;
  if (INT8) {
    const int64_t groups = g.H / kGroup;
    for (int64_t gr = 0; gr < groups; ++gr)
      quant_group<DT>(xr + gr * kGroup, reinterpret_cast<int8_t*>(row + gr * kGroup),
                      reinterpret_cast<float*>(row + g.H + 4 * gr), lane);
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(xr);
    uint4* dst = reinterpret_cast<uint4*>(row);
    const int64_t n = g.H / 8;
    for (int64_t c = lane; c < n; c += 32) dst[c] = src[c];
  }
  }
  }
  if (P.p2p) ep_signal_peers(P, (int)g.W, 0, P.rank);
}

// ---------------------------------------------------------------------------
// Owner metadata (one CTA of kRouteThreads threads): from the W received
// headers, per local expert e its first sorted slot and per (sender s, e) the
// base of s's routes to e (senders ascending); the tile list and header.
__global__ void __launch_bounds__(kRouteThreads) ep_owner_meta_kernel(const uint8_t* __restrict__ recv, EpGeom g,
                                                                      int with_shared, int32_t* __restrict__ hdr,
                                                                      Tile* __restrict__ tiles,
                                                                      int32_t* __restrict__ base, int* err,
                                                                      const EpPeers P) {
  __shared__ int warp_tot[32];
  __shared__ int s_first[kRouteThreads + 1];
  __shared__ int s_bad;
  const int E = (int)g.e_loc, W = (int)g.W;
  const int e = threadIdx.x;
  // direct transport: every sender's segment has landed (a timeout empties the layer)
  const bool arrived = P.p2p ? ep_wait_peers(P, W, 0, err) : true;
  if (e == 0) s_bad = arrived ? 0 : 1;
  __syncthreads();
  int n = 0;
  if (e < E) {
    for (int s = 0; s < W; ++s) {
      const int32_t* h = reinterpret_cast<const int32_t*>(recv + (int64_t)s * g.seg_rows * g.row_bytes);
      const int c = __ldcg(h + 1 + e);
      const int rows = __ldcg(h);
      if (c < 0 || c > rows || rows < 0 || rows > g.cap) s_bad = 1;
      n += max(0, c);
    }
  }
  __syncthreads();
  if (s_bad) n = 0;
  int incl = block_incl_scan(e < E ? n : 0, warp_tot);
  if (e == E - 1 && (int64_t)incl > g.r_max) s_bad = 1;  // more routes than any sender can send
  __syncthreads();
  if (s_bad) incl = n = 0;
  const int first = incl - (e < E ? n : 0);
  if (e <= E) s_first[e] = first;  // s_first[E] = valid routes
  if (e < E) {
    int run = first;
    for (int s = 0; s < W; ++s) {
      const int32_t* h = reinterpret_cast<const int32_t*>(recv + (int64_t)s * g.seg_rows * g.row_bytes);
      base[s * E + e] = run;
      run += s_bad ? 0 : __ldcg(h + 1 + e);
    }
  }
  if (e == 0 && s_bad) raise_error(err, LMOE_DEVERR_BAD_INDEX);
  __syncthreads();
  const int valid = s_first[E];
  write_tile_list(E, (int)g.T, with_shared, s_first, valid, valid, tiles, hdr, warp_tot);
}

// ---------------------------------------------------------------------------
// Owner scatter: one warp per received row (sender s, row i), then one per own
// token for the shared expert's rows.  Each valid route of a row gets its sorted
// slot base[s][e] + rank; the row's payload is written to the activation row of
// every one of its routes.
template <int DT, bool INT8>
__global__ void __launch_bounds__(32 * kEpWarps) ep_owner_scatter_kernel(
    const uint8_t* __restrict__ recv, const typename Act<DT>::T* __restrict__ x, EpGeom g,
    const int32_t* __restrict__ hdr, const int32_t* __restrict__ base, float* __restrict__ rweight,
    int32_t* __restrict__ ordered, typename Act<DT>::T* __restrict__ xs, int with_shared, int* err) {
  using A = Act<DT>;
  const int lane = lane_id();
  const int64_t task = (int64_t)blockIdx.x * kEpWarps + warp_id();
  const int64_t nrecv = g.W * g.cap;
  const int64_t valid = hdr[kHdrValid];
  if (task >= nrecv) {
    const int64_t t = task - nrecv;
    if (!with_shared || t >= g.T) return;
    const uint4* src = reinterpret_cast<const uint4*>(x + t * g.H);
    uint4* dst = reinterpret_cast<uint4*>(xs + (valid + t) * g.H);
    for (int64_t c = lane; c < g.H / 8; c += 32) dst[c] = src[c];
    return;
  }
  const int64_t s = task / g.cap, i = task - s * g.cap;
  const int32_t* sh = reinterpret_cast<const int32_t*>(recv + s * g.seg_rows * g.row_bytes);
  const int top = (int)g.top;
  int32_t* ord = ordered + task * top;
  if (i >= sh[0] || valid == 0) {
    if (lane < top) ord[lane] = -1;
    return;
  }
  const uint8_t* row = recv + (s * g.seg_rows + 1 + i) * g.row_bytes;
  int dst = -1;
  if (lane < top) {
    const int lid = reinterpret_cast<const int32_t*>(row + g.payload)[lane];
    const float w = reinterpret_cast<const float*>(row + g.payload + 4 * top)[lane];
    const int rk = reinterpret_cast<const int32_t*>(row + g.payload + 8 * top)[lane];
    if (lid >= 0) {
      if (lid < g.e_loc && rk >= 0 && rk < sh[1 + lid]) {
        dst = base[s * g.e_loc + lid] + rk;
        rweight[dst] = w;
      } else {
        raise_error(err, LMOE_DEVERR_BAD_INDEX);
      }
    }
    ord[lane] = dst;
  }
  const unsigned has = __ballot_sync(0xffffffffu, dst >= 0);
  if (!has) return;
  if (INT8) {
    const int64_t groups = g.H / kGroup;
    for (int64_t gr = 0; gr < groups; ++gr) {
      const uint32_t q = *reinterpret_cast<const uint32_t*>(row + gr * kGroup + lane * 4);
      const float sc = *reinterpret_cast<const float*>(row + g.H + 4 * gr);
      float f0, f1, f2, f3;
      i8x4_to_f32(q, f0, f1, f2, f3);
      uint2 o;
      o.x = A::pack(__fmul_rn(f0, sc), __fmul_rn(f1, sc));
      o.y = A::pack(__fmul_rn(f2, sc), __fmul_rn(f3, sc));
      for (unsigned m = has; m; m &= m - 1) {
        const int r = __shfl_sync(0xffffffffu, dst, __ffs(m) - 1);
        *reinterpret_cast<uint2*>(xs + (int64_t)r * g.H + gr * kGroup + lane * 4) = o;
      }
    }
  } else {
    const uint4* src = reinterpret_cast<const uint4*>(row);
    const int64_t n = g.H / 8;
    for (int64_t c0 = 0; c0 < n; c0 += 4 * 32) {
      uint4 v[4];
#pragma unroll
      for (int u = 0; u < 4; ++u)
        if (c0 + u * 32 + lane < n) v[u] = src[c0 + u * 32 + lane];
      for (unsigned m = has; m; m &= m - 1) {
        const int r = __shfl_sync(0xffffffffu, dst, __ffs(m) - 1);
        uint4* d = reinterpret_cast<uint4*>(xs + (int64_t)r * g.H);
#pragma unroll
        for (int u = 0; u < 4; ++u)
          if (c0 + u * 32 + lane < n) d[c0 + u * 32 + lane] = v[u];
      }
    }
  }
}

// ---------------------------------------------------------------------------
// Owner combine: one CTA per received row; acc = round(acc + v) over its routes
// in ascending local expert order (the order they were packed in).
template <int DT>
__global__ void __launch_bounds__(kEpCombineThreads) ep_owner_combine_kernel(
    const uint8_t* __restrict__ recv, EpGeom g, const int32_t* __restrict__ ordered,
    const typename Act<DT>::T* __restrict__ down, typename Act<DT>::T* __restrict__ partial, const EpPeers P) {
  using A = Act<DT>;
  // a persistent grid over the received rows (one signal per CTA with the direct transport)
  for (int64_t task = blockIdx.x; task < g.W * g.cap; task += gridDim.x) {
  const int64_t s = task / g.cap, i = task - s * g.cap;
  if (i < reinterpret_cast<const int32_t*>(recv + s * g.seg_rows * g.row_bytes)[0]) {
    const int top = (int)g.top;
    const int32_t* ord = ordered + task * top;
    // the row's partial sum goes to the local buffer or (direct transport) straight into
    // row (rank, i) of its sender's return buffer
    typename A::T* dst = P.p2p ? reinterpret_cast<typename A::T*>(P.back[s]) + ((int64_t)P.rank * g.cap + i) * g.H
                               : partial + task * g.H;
    for (int64_t c = threadIdx.x * 8; c < g.H; c += kEpCombineThreads * 8) {
      float acc[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
      for (int k = 0; k < top; ++k) {
        const int r = ord[k];
        if (r < 0) continue;
        const uint4 v = *reinterpret_cast<const uint4*>(down + (int64_t)r * g.H + c);
        const uint32_t va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          acc[2 * j] = A::round(__fadd_rn(acc[2 * j], A::lo_f(va[j])));
          acc[2 * j + 1] = A::round(__fadd_rn(acc[2 * j + 1], A::hi_f(va[j])));
        }
      }
      uint4 o;
      o.x = A::pack(acc[0], acc[1]);
      o.y = A::pack(acc[2], acc[3]);
      o.z = A::pack(acc[4], acc[5]);
      o.w = A::pack(acc[6], acc[7]);
      *reinterpret_cast<uint4*>(dst + c) = o;
    }
  }
  }
  if (P.p2p) ep_signal_peers(P, (int)g.W, 1, (int)g.W + P.rank);
}

// ---------------------------------------------------------------------------
// Sender fold: one CTA per own token.  The returned rows in ascending rank
// order, then the gated shared expert (rows after the valid routes of this
// rank's own owner workspace), then the residual.
template <int DT>
__global__ void __launch_bounds__(kEpCombineThreads) ep_fold_kernel(
    const typename Act<DT>::T* __restrict__ back, EpGeom g, const int32_t* __restrict__ slot_of,
    const typename Act<DT>::T* __restrict__ x, const typename Act<DT>::T* __restrict__ gate_w, int with_shared,
    const int32_t* __restrict__ hdr, const typename Act<DT>::T* __restrict__ down,
    const typename Act<DT>::T* __restrict__ residual, typename Act<DT>::T* __restrict__ out, const EpPeers P,
    int* err) {
  using A = Act<DT>;
  __shared__ float red[kEpCombineThreads / 32];
  const int64_t t = blockIdx.x;
  const int64_t H = g.H;
  // direct transport: every owner's returned rows have landed
  if (P.p2p && !ep_wait_peers(P, (int)g.W, (int)g.W, err)) return;
  float sig = 1.f;
  if (with_shared && gate_w != nullptr) {
    float part = 0.f;
    for (int64_t c = threadIdx.x * 8; c < H; c += kEpCombineThreads * 8) {
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
    for (int w = 0; w < kEpCombineThreads / 32; ++w) tot += red[w];
    const float logit = A::round(tot);
    sig = A::round(__fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-logit))));
  }
  const int64_t shared_row = with_shared ? hdr[kHdrValid] + t : 0;
  for (int64_t c = threadIdx.x * 8; c < H; c += kEpCombineThreads * 8) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    for (int64_t d = 0; d < g.W; ++d) {
      const int slot = slot_of[t * g.W + d];
      if (slot < 0) continue;
      const uint4 v = __ldcg(reinterpret_cast<const uint4*>(back + (d * g.cap + slot) * H + c));
      const uint32_t va[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        acc[2 * j] = A::round(__fadd_rn(acc[2 * j], A::lo_f(va[j])));
        acc[2 * j + 1] = A::round(__fadd_rn(acc[2 * j + 1], A::hi_f(va[j])));
      }
    }
    if (with_shared) {
      const uint4 v = *reinterpret_cast<const uint4*>(down + shared_row * H + c);
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

static EpPeers make_peers(const lmoe_ep_peers* pp, int64_t world) {
  EpPeers P = {};
  if (pp == nullptr) return P;
  for (int64_t d = 0; d < world; ++d) {
    P.recv[d] = (uint8_t*)pp->recv[d];
    P.back[d] = (uint8_t*)pp->back[d];
    P.flags[d] = (unsigned*)pp->flags[d];
  }
  P.counter = (unsigned*)pp->counter;
  P.rank = pp->rank;
  P.epoch = pp->epoch;
  P.p2p = 1;
  return P;
}

static bool peers_ok(const lmoe_ep_peers* pp, int64_t world) {
  if (pp == nullptr) return true;
  if (pp->rank < 0 || pp->rank >= world || pp->counter == nullptr) return false;
  for (int64_t d = 0; d < world; ++d)
    if (!pp->recv[d] || !pp->back[d] || !pp->flags[d] || ((uintptr_t)pp->recv[d] & 15) || ((uintptr_t)pp->back[d] & 15))
      return false;
  return true;
}

static bool ep_geometry_ok(int64_t tokens, int64_t top, int64_t experts, int64_t world, int64_t cap, int64_t hidden,
                           int64_t inter, int wire, int dtype) {
  if (tokens <= 0 || top <= 0 || top > kEpMaxTop || experts <= 0 || world <= 0 || world > kEpMaxWorld) return false;
  if (experts % world || cap < tokens || hidden <= 0 || hidden % 256 || inter <= 0 || inter % kGroup) return false;
  if (wire != LMOE_WIRE_DTYPE && wire != LMOE_WIRE_INT8) return false;
  if (dtype != LMOE_BF16 && dtype != LMOE_F16) return false;
  const int64_t e_loc = experts / world;
  if (e_loc + 2 > kRouteThreads || experts > 4096) return false;
  const EpGeom g(tokens, top, experts, world, cap, hidden, inter, wire, dtype);
  if ((1 + e_loc) * 4 > g.row_bytes) return false;  // the segment header fits one row
  return g.r_max + tokens < (int64_t(1) << 31) / 4 && world * cap * top < (int64_t(1) << 30) &&
         tokens * top < (int64_t(1) << 30);
}

}  // namespace lmoe

using namespace lmoe;

int lmoe_route_meta_impl(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                         int with_shared, void* meta, int* err, cudaStream_t st);

extern "C" int64_t lmoe_ep_layer_row_bytes(int64_t hidden, int64_t top, int wire) {
  if (hidden <= 0 || hidden % kGroup || top <= 0 || top > kEpMaxTop) return LMOE_ERR_INVALID;
  if (wire != LMOE_WIRE_DTYPE && wire != LMOE_WIRE_INT8) return LMOE_ERR_INVALID;
  return EpGeom(1, top, 1, 1, 1, hidden, kGroup, wire, LMOE_BF16).row_bytes;
}

extern "C" int64_t lmoe_ep_plan_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t world) {
  if (tokens <= 0 || top <= 0 || experts <= 0 || world <= 0) return LMOE_ERR_INVALID;
  return EpPlanWs(EpGeom(tokens, top, experts, world, tokens, 256, kGroup, LMOE_WIRE_DTYPE, LMOE_BF16)).bytes;
}

extern "C" int64_t lmoe_ep_owner_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t world,
                                                int64_t cap, int64_t hidden, int64_t inter) {
  if (!ep_geometry_ok(tokens, top, experts, world, cap, hidden, inter, LMOE_WIRE_DTYPE, LMOE_BF16))
    return LMOE_ERR_INVALID;
  return EpOwnerWs(EpGeom(tokens, top, experts, world, cap, hidden, inter, LMOE_WIRE_DTYPE, LMOE_BF16)).bytes;
}

extern "C" int lmoe_ep_dispatch(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                                int64_t experts, int64_t world, int64_t cap, int64_t hidden, int wire, int dtype,
                                void* send, void* plan_ws, int* err, const lmoe_ep_peers* peers, void* stream) {
  if (!x || !weights || !ids || (!send && !peers) || !plan_ws || !peers_ok(peers, world)) return LMOE_ERR_INVALID;
  const EpPeers P = make_peers(peers, world);
  if (!ep_geometry_ok(tokens, top, experts, world, cap, hidden, kGroup, wire, dtype)) return LMOE_ERR_INVALID;
  if (((uintptr_t)x & 15) || ((uintptr_t)send & 15)) return LMOE_ERR_INVALID;
  cudaStream_t st = (cudaStream_t)stream;
  const EpGeom g(tokens, top, experts, world, cap, hidden, kGroup, wire, dtype);
  const EpPlanWs PW(g);
  const MetaLayout ML(tokens, top, experts);
  char* meta = (char*)plan_ws + PW.off_meta;
  int32_t* slot_of = (int32_t*)((char*)plan_ws + PW.off_slot);
  const int32_t* offsets = (const int32_t*)(meta + ML.off_offsets);
  const int32_t* inverse = (const int32_t*)(meta + ML.off_inverse);
  uint8_t* sb = (uint8_t*)send;
  // this rank's routes sorted by expert (stable): per route its sorted slot
  int rc = lmoe_route_meta_impl(ids, weights, tokens, top, experts, 0, meta, err, st);
  if (rc) return rc;
  if (tokens > 200 * 1024) return LMOE_ERR_UNSUPPORTED;  // the destination bits of every token in shared memory
  const size_t smem = (size_t)tokens;
  if (smem > 48 * 1024)
    LMOE_CUDA_CHECK(cudaFuncSetAttribute(ep_slots_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem));
  ep_slots_kernel<<<1, kRouteThreads, smem, st>>>(ids, g, offsets, slot_of, sb, P);
  LMOE_CUDA_CHECK(cudaGetLastError());
  const int64_t want = (tokens * world + kEpWarps - 1) / kEpWarps;
  const unsigned blocks = (unsigned)(want < 4 * sm_count() ? want : 4 * sm_count());
  const dim3 block(32 * kEpWarps);
  if (dtype == LMOE_BF16) {
    const __nv_bfloat16* xp = (const __nv_bfloat16*)x;
    if (wire == LMOE_WIRE_INT8)
      ep_pack_kernel<LMOE_BF16, true><<<blocks, block, 0, st>>>(xp, ids, weights, g, slot_of, inverse, offsets, sb, P);
    else
      ep_pack_kernel<LMOE_BF16, false><<<blocks, block, 0, st>>>(xp, ids, weights, g, slot_of, inverse, offsets, sb, P);
  } else {
    const __half* xp = (const __half*)x;
    if (wire == LMOE_WIRE_INT8)
      ep_pack_kernel<LMOE_F16, true><<<blocks, block, 0, st>>>(xp, ids, weights, g, slot_of, inverse, offsets, sb, P);
    else
      ep_pack_kernel<LMOE_F16, false><<<blocks, block, 0, st>>>(xp, ids, weights, g, slot_of, inverse, offsets, sb, P);
  }
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

template <int DT>
static int ep_owner_launch(const EpGeom& g, const uint8_t* recv, const void* x, const int8_t* qg, const float* sg,
                           const int8_t* qd, const float* sd, const int8_t* sh_qg, const float* sh_sg,
                           const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd, const float* sh_sd,
                           char* ws, void* partial, int* err, void** events, const EpPeers& P, cudaStream_t st) {
  using T = typename Act<DT>::T;
  const EpOwnerWs O(g);
  const bool with_shared = sh_qg != nullptr;
  int32_t* hdr = (int32_t*)(ws + O.off_hdr);
  Tile* tiles = (Tile*)(ws + O.off_tiles);
  int32_t* base = (int32_t*)(ws + O.off_base);
  float* rweight = (float*)(ws + O.off_rweight);
  int32_t* ordered = (int32_t*)(ws + O.off_ordered);
  T* xs = (T*)(ws + O.off_xs);
  void* hid = ws + O.off_hidden;
  T* dn = (T*)(ws + O.off_down);
  auto mark = [&](int i) -> int {
    if (events && events[i]) LMOE_CUDA_CHECK(cudaEventRecord((cudaEvent_t)events[i], st));
    return LMOE_OK;
  };
  int rc = mark(0);
  if (rc) return rc;
  ep_owner_meta_kernel<<<1, kRouteThreads, 0, st>>>(recv, g, with_shared ? 1 : 0, hdr, tiles, base, err, P);
  LMOE_CUDA_CHECK(cudaGetLastError());
  const int64_t tasks = g.W * g.cap + g.T;
  const unsigned blocks = (unsigned)((tasks + kEpWarps - 1) / kEpWarps);
  // a plain launch: the GEMMs after it start only once it has completed, so the
  // routing weights it writes are in place before the down kernel's epilogue reads them
  if (g.int8)
    ep_owner_scatter_kernel<DT, true><<<blocks, 32 * kEpWarps, 0, st>>>(recv, (const T*)x, g, hdr, base, rweight,
                                                                        ordered, xs, with_shared ? 1 : 0, err);
  else
    ep_owner_scatter_kernel<DT, false><<<blocks, 32 * kEpWarps, 0, st>>>(recv, (const T*)x, g, hdr, base, rweight,
                                                                         ordered, xs, with_shared ? 1 : 0, err);
  LMOE_CUDA_CHECK(cudaGetLastError());
  if ((rc = mark(1))) return rc;

  const int64_t rows = g.r_max + g.T;
  GemmLaunch gu = {};
  gu.x = xs;
  gu.x_rows = rows;
  gu.K = g.H;
  gu.tiles = tiles;
  gu.hdr = hdr;
  gu.grid_tiles = g.max_tiles;
  gu.q_bank = qg;
  gu.s_bank = sg;
  gu.experts = g.e_loc;
  gu.N = 2 * g.I;
  gu.inter = g.I;
  if (with_shared) {
    gu.q_lo = sh_qg;
    gu.s_lo = sh_sg;
    gu.q_hi = sh_qu;
    gu.s_hi = sh_su;
    gu.rows_lo = g.I;
    gu.rows_hi = g.I;
  }
  gu.y = hid;
  gu.ldy = g.I;
  gu.mode = kSwiGLU;
  gu.dtype = DT;
  gu.err = err;
  if ((rc = launch_swiglu_ts(gu, st))) return rc;
  if ((rc = mark(2))) return rc;
  GemmLaunch dw = gu;
  dw.x = hid;
  dw.K = g.I;
  dw.q_bank = qd;
  dw.s_bank = sd;
  dw.N = g.H;
  dw.inter = 0;
  dw.q_lo = with_shared ? sh_qd : nullptr;
  dw.s_lo = with_shared ? sh_sd : nullptr;
  dw.q_hi = nullptr;
  dw.s_hi = nullptr;
  dw.rows_lo = with_shared ? g.H : 0;
  dw.rows_hi = 0;
  dw.y = dn;
  dw.ldy = g.H;
  dw.rweight = rweight;
  dw.mode = kWeighted;
  if ((rc = launch_down_ts(dw, st))) return rc;
  if ((rc = mark(3))) return rc;
  // plain launch: reads the down kernel's output
  const int64_t rows_in = g.W * g.cap;
  const unsigned cblocks = (unsigned)(rows_in < 8 * sm_count() ? rows_in : 8 * sm_count());
  ep_owner_combine_kernel<DT><<<cblocks, kEpCombineThreads, 0, st>>>(recv, g, ordered, dn, (T*)partial, P);
  LMOE_CUDA_CHECK(cudaGetLastError());
  return mark(4);
}

extern "C" int lmoe_ep_owner(const void* recv, const void* x, int64_t tokens, int64_t top, int64_t experts,
                             int64_t world, int64_t cap, int64_t hidden, int64_t inter, int wire, const int8_t* qg,
                             const float* sg, const int8_t* qd, const float* sd, const int8_t* sh_qg,
                             const float* sh_sg, const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd,
                             const float* sh_sd, void* ws, void* partial, int dtype, int* err, void** stage_events,
                             const lmoe_ep_peers* peers, void* stream) {
  if (!peers_ok(peers, world)) return LMOE_ERR_INVALID;
  if (peers) recv = peers->recv[peers->rank];
  if (!recv || !x || !qg || !sg || !qd || !sd || !ws || (!partial && !peers)) return LMOE_ERR_INVALID;
  if (!ep_geometry_ok(tokens, top, experts, world, cap, hidden, inter, wire, dtype)) return LMOE_ERR_INVALID;
  if (sh_qg && (!sh_sg || !sh_qu || !sh_su || !sh_qd || !sh_sd)) return LMOE_ERR_INVALID;
  if (((uintptr_t)recv & 15) || ((uintptr_t)x & 15) || ((uintptr_t)partial & 15) || ((uintptr_t)ws & 255))
    return LMOE_ERR_INVALID;
  const EpGeom g(tokens, top, experts, world, cap, hidden, inter, wire, dtype);
  const EpPeers P = make_peers(peers, world);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    return ep_owner_launch<LMOE_BF16>(g, (const uint8_t*)recv, x, qg, sg, qd, sd, sh_qg, sh_sg, sh_qu, sh_su, sh_qd,
                                      sh_sd, (char*)ws, partial, err, stage_events, P, st);
  return ep_owner_launch<LMOE_F16>(g, (const uint8_t*)recv, x, qg, sg, qd, sd, sh_qg, sh_sg, sh_qu, sh_su, sh_qd,
                                   sh_sd, (char*)ws, partial, err, stage_events, P, st);
}

extern "C" int lmoe_ep_fold(const void* back, const void* plan_ws, const void* x, int64_t tokens, int64_t top,
                            int64_t experts, int64_t world, int64_t cap, int64_t hidden, int64_t inter,
                            const void* owner_ws, int with_shared, const void* sh_gate_w, const void* residual,
                            void* out, int dtype, int* err, const lmoe_ep_peers* peers, void* stream) {
  if (!peers_ok(peers, world)) return LMOE_ERR_INVALID;
  if (peers) back = peers->back[peers->rank];
  if (!back || !plan_ws || !x || !out || (with_shared && !owner_ws)) return LMOE_ERR_INVALID;
  if (!ep_geometry_ok(tokens, top, experts, world, cap, hidden, inter, LMOE_WIRE_DTYPE, dtype))
    return LMOE_ERR_INVALID;
  const EpGeom g(tokens, top, experts, world, cap, hidden, inter, LMOE_WIRE_DTYPE, dtype);
  const EpPlanWs Pw(g);
  const EpOwnerWs O(g);
  const EpPeers P = make_peers(peers, world);
  const int32_t* slot_of = (const int32_t*)((const char*)plan_ws + Pw.off_slot);
  const int32_t* hdr = with_shared ? (const int32_t*)((const char*)owner_ws + O.off_hdr) : nullptr;
  const char* dn = with_shared ? (const char*)owner_ws + O.off_down : nullptr;
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == LMOE_BF16)
    ep_fold_kernel<LMOE_BF16><<<(unsigned)tokens, kEpCombineThreads, 0, st>>>(
        (const __nv_bfloat16*)back, g, slot_of, (const __nv_bfloat16*)x, (const __nv_bfloat16*)sh_gate_w,
        with_shared ? 1 : 0, hdr, (const __nv_bfloat16*)dn, (const __nv_bfloat16*)residual, (__nv_bfloat16*)out, P,
        err);
  else
    ep_fold_kernel<LMOE_F16><<<(unsigned)tokens, kEpCombineThreads, 0, st>>>(
        (const __half*)back, g, slot_of, (const __half*)x, (const __half*)sh_gate_w, with_shared ? 1 : 0, hdr,
        (const __half*)dn, (const __half*)residual, (__half*)out, P, err);
  LMOE_CUDA_CHECK(cudaGetLastError());
  return LMOE_OK;
}

// ---------------------------------------------------------------------------
// Mapping the exchange buffers of the other ranks (CUDA IPC).  A handle names the
// whole allocation that holds `ptr`; the offset locates ptr inside it.
typedef CUresult (*MemRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

extern "C" int lmoe_ipc_get_handle(const void* ptr, void* handle, int64_t* offset) {
  if (!ptr || !handle || !offset) return LMOE_ERR_INVALID;
  static MemRangeFn range = []() -> MemRangeFn {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return (MemRangeFn)f;
    return nullptr;
  }();
  if (range == nullptr) return LMOE_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)ptr) != CUDA_SUCCESS) return LMOE_ERR_CUDA;
  cudaIpcMemHandle_t h;
  LMOE_CUDA_CHECK(cudaIpcGetMemHandle(&h, (void*)base));
  memcpy(handle, &h, sizeof(h));
  *offset = (int64_t)((CUdeviceptr)ptr - base);
  return LMOE_OK;
}

extern "C" int lmoe_ipc_open_handle(const void* handle, int64_t offset, void** ptr, void** base) {
  if (!handle || !ptr || !base || offset < 0) return LMOE_ERR_INVALID;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* b = nullptr;
  LMOE_CUDA_CHECK(cudaIpcOpenMemHandle(&b, h, cudaIpcMemLazyEnablePeerAccess));
  *base = b;
  *ptr = (char*)b + offset;
  return LMOE_OK;
}

extern "C" int lmoe_ipc_close(void* base) {
  if (!base) return LMOE_ERR_INVALID;
  LMOE_CUDA_CHECK(cudaIpcCloseMemHandle(base));
  return LMOE_OK;
}
