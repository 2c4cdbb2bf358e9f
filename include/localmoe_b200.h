/*
 * localmoe_b200.h -- C ABI of the B200 (sm_100a) INT8 group-128 MoE matmul path.
 *
 * Conventions shared by every entry point:
 *  - all tensor arguments are DEVICE pointers to contiguous row-major memory;
 *  - weights use the converted-checkpoint layout: int8 q[.., N, K] (K fastest)
 *    and float32 scale[.., N, K/128], one scale per 128-wide K group;
 *    expert banks are stacked [E, N, K]; gate_up rows [0, I) are gate and
 *    [I, 2I) are up;
 *  - activations are bf16 (dtype LMOE_BF16) or fp16 (LMOE_F16);
 *  - `stream` is a cudaStream_t passed as void*; work is enqueued on it with
 *    no host synchronisation, so the calls can be captured in a CUDA graph
 *    (this does not cover lmoe_routed_moe_noalloc, which makes no such promise);
 *  - no entry point allocates device memory: scratch ("workspace") buffers are
 *    passed in by the caller, sized by the *_workspace_size functions
 *    (lmoe_routed_moe_noalloc uses a fixed array inside the library instead);
 *  - most kernels are launched as programmatic dependents of the work before
 *    them on the stream and let the next kernel launch early: a library kernel
 *    reads its inputs only after that work has completed, and a caller's own
 *    kernel launched with programmatic stream serialization after a library
 *    call must wait (griddepcontrol.wait / cudaGridDependencySynchronize)
 *    before reading the call's outputs, as for any programmatic dependent;
 *    ordinary launches, copies and events need nothing;
 *  - the return value is LMOE_OK or a negative LMOE_ERR_* code (invalid
 *    geometry or a CUDA launch error); nothing aborts or traps.  Device-side
 *    bounded waits that give up set LMOE_DEVERR_* bits in the caller's
 *    int32 error word (`err`), which the caller may read after the stream.
 *
 * Each declaration names the reference interface it replaces
 * (heliosz616/LocalMoe35Ba3b, file:line).
 */
#ifndef LOCALMOE_B200_H
#define LOCALMOE_B200_H
#include <stdint.h>

#if defined(__GNUC__)
#define LMOE_API __attribute__((visibility("default")))
#else
#define LMOE_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define LMOE_OK 0
#define LMOE_ERR_INVALID (-1)
#define LMOE_ERR_CUDA (-2)
#define LMOE_ERR_UNSUPPORTED (-3)

#define LMOE_DEVERR_TIMEOUT 1
#define LMOE_DEVERR_BAD_EXPERT 2 /* an expert id outside [0, experts): read as expert 0 */
#define LMOE_DEVERR_BAD_INDEX 4  /* a row index outside its buffer: that row is written as zeros */
#define LMOE_ERR_TIMEOUT LMOE_DEVERR_TIMEOUT

#define LMOE_BF16 0
#define LMOE_F16 1

/* Library ABI version (increments on any signature change). */
LMOE_API int lmoe_abi_version(void);

/* Replaces w8a8.quantize / w8a8._quant (qwen35_deploy/operators/w8a8.py:8-22).
 * Per (row, 128-group): s = max(absmax, 1e-10) * fp32(1/127), q = rint(x / s). */
LMOE_API int lmoe_quantize_rows(const void* x, int8_t* q, float* s, int64_t rows, int64_t k, int dtype, void* stream);

/* Replaces int8.linear / int8._linear (qwen35_deploy/operators/int8.py:9-37).
 * y[m, n] = sum_k x[m, k] * round_dtype(q[n, k] * scale[n, k/128]), fp32 accumulation.
 * One row runs an HBM-streaming GEMV; more rows a tcgen05 tensor-core GEMM (the weights
 * on the MMA's M side when n % 128 == 0). */
LMOE_API int lmoe_linear_w8a16(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                      int64_t k, int dtype, int* err, void* stream);

/* The same linear with a scratch workspace (no reference counterpart beyond int8.linear):
 * when its (128-row tile, 128-column block) units would not fill the GPU, the
 * tensor-core kernel splits K over lmoe_linear_w8a16_workspace_size(m, n, k) bytes of ws
 * (fp32 partial sums, added in split order, rounded once).  A size of 0 means no split;
 * ws may then be NULL.  With a smaller ws the call runs without splitting. */
LMOE_API int64_t lmoe_linear_w8a16_workspace_size(int64_t m, int64_t n, int64_t k);
LMOE_API int lmoe_linear_w8a16_ws(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                                  int64_t k, int dtype, void* ws, int64_t ws_bytes, int* err, void* stream);

/* Dense W8A8 linear for any number of rows m (BASELINE's dense sweep; the reference has the
 * same arithmetic only as its one-row decode GEMV, qwen35_deploy/operators/w8a8.py:8-48):
 * x [m, k] quantised per (row, 128-group) as w8a8.quantize, then on int8 tensor cores
 * y[r, n] = round_dtype(acc), acc = acc + (float(dot_g) * xs[r, g]) * ws[n, g] over the
 * groups g in order, dot_g the exact int32 group dot.  n % 128 == 0, k % 128 == 0,
 * k <= 8192; ws: lmoe_linear_w8a8_workspace_size(m, k) bytes, 256-byte aligned (the
 * quantised rows and their scales). */
LMOE_API int64_t lmoe_linear_w8a8_workspace_size(int64_t m, int64_t k);
LMOE_API int lmoe_linear_w8a8(const void* x, const int8_t* q, const float* scale, void* y, int64_t m, int64_t n,
                              int64_t k, int dtype, void* ws, int* err, void* stream);

/* Replaces int8.grouped_linear / int8._grouped_linear (qwen35_deploy/operators/int8.py:213-237).
 * table is a device int64 [experts, 5] of (gate_up.q, gate_up.scale, down.q, down.scale, slot);
 * field 0 selects the gate_up pair, field 2 the down pair.  Row e uses x row 0 when
 * shared != 0, else x row e.  y is [experts, n]. */
LMOE_API int lmoe_grouped_linear_w8a16(const void* x, const int64_t* table, void* y, int64_t experts, int64_t n, int64_t k,
                              int field, int shared, int dtype, void* stream);

/* Replaces w8a8.grouped_linear / w8a8._linear (qwen35_deploy/operators/w8a8.py:25-48):
 * per-(row,128) int8 activation quantisation (into xq/xs, [rows, k] and [rows, k/128])
 * followed by per-group int32 dots, acc = acc + (float(dot) * xs) * ws in group order. */
LMOE_API int lmoe_grouped_linear_w8a8(const void* x, const int64_t* table, void* y, int64_t experts, int64_t n, int64_t k,
                             int field, int shared, int dtype, int8_t* xq, float* xs, void* stream);

/* Replaces int8._ordered_reduce (qwen35_deploy/operators/int8.py:240-250):
 * y[n] = ordered sum over table rows e of round(values[e, n] * weights[table[e, 4]]). */
LMOE_API int lmoe_ordered_reduce(const void* values, const int64_t* table, const float* weights, void* y, int64_t n,
                        int64_t experts, int dtype, void* stream);

/* Replaces gpu_routes.plan / gpu_routes._table (qwen35_deploy/runtime/gpu_routes.py:17-63).
 * Outputs (int64): pos [tokens*top], table [ceil(tokens*top/bm)+experts, 3],
 * ordered [tokens, top], slots [tokens, top]. ws: lmoe_plan_workspace_size bytes. */
LMOE_API int64_t lmoe_plan_workspace_size(int64_t tokens, int64_t top, int64_t experts);
LMOE_API int lmoe_plan(const int64_t* ids, int64_t tokens, int64_t top, int64_t experts, int64_t bm, int64_t* pos,
              int64_t* table, int64_t* ordered, int64_t* slots, void* ws, void* stream);

/* Routing metadata for the fused prefill path (replaces the torch sort/searchsorted/
 * argsort/scatter of gpu_routes.py:51-62 plus _table with this build's 256-route tiles).
 * meta: lmoe_route_meta_size bytes.  with_shared != 0 appends a segment of `tokens`
 * identity routes for the shared expert. */
LMOE_API int64_t lmoe_route_meta_size(int64_t tokens, int64_t top, int64_t experts);
LMOE_API int lmoe_route_meta(const int64_t* ids, const float* weights, int64_t tokens, int64_t top, int64_t experts,
                    int with_shared, void* meta, void* stream);

/* Replaces prefill._routed via gpu_routes._nonempty (qwen35_deploy/runtime/prefill.py:12-34,
 * gpu_routes.py:39-44): for every route r of expert e, y[r] = x[gather ? pos[r] : r] . W_e^T.
 * meta comes from lmoe_route_meta (its expert segments and tiles).  With gather != 0 the
 * token rows are first copied in route order into ws (lmoe_routed_linear_workspace_size). */
LMOE_API int64_t lmoe_routed_linear_workspace_size(int64_t tokens, int64_t top, int64_t k);
LMOE_API int lmoe_routed_linear(const void* x, const int8_t* q, const float* scale, int64_t experts, int64_t n,
                       int64_t k, const void* meta, int64_t tokens, int64_t top, int gather, void* y,
                       int dtype, void* ws, int* err, void* stream);

/* Replaces prefill._reduce (qwen35_deploy/runtime/prefill.py:37-49): per token, ordered
 * combine of its routes (ordered/slots as returned by lmoe_plan; weights fp32 [tokens, top]). */
LMOE_API int lmoe_routed_reduce(const void* down, const int64_t* ordered, const int64_t* slots, const float* weights,
                       void* y, int64_t tokens, int64_t n, int64_t top, int dtype, void* stream);

/* Replaces gpu_routes.routed_moe (qwen35_deploy/runtime/gpu_routes.py:66-82) -- and, when
 * the shared-expert arguments are non-null, the whole Qwen3_5MoeSparseMoeBlock expert part
 * (transformers qwen3_5_moe/modeling_qwen3_5_moe.py:781-792):
 *   out = routed(x) [+ round(sigmoid(round(x . shared_gate_w)) * shared_expert(x))]
 *   [+ residual]
 * Launches: route metadata, gate_up GEMM with fused SwiGLU, down GEMM with fused routing
 * weight, ordered combine.  ws: lmoe_moe_workspace_size bytes.  stage_events (nullable)
 * is an array of 5 cudaEvent_t recorded before/between/after the four launches.
 * top == 0 (ids and weights may then be NULL) is accepted with a shared expert: the output
 * is the gated shared expert alone (+ residual) -- how an expert-parallel caller computes
 * its own tokens' shared expert while their routes run on other GPUs.  A route id of -1
 * is "no route": it is not computed and the combine skips it (an expert-parallel owner's
 * received rows list only its own experts); any other id outside [0, experts) sets
 * LMOE_DEVERR_BAD_EXPERT. */
LMOE_API int64_t lmoe_moe_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t hidden, int64_t inter);
LMOE_API int lmoe_routed_moe(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                    const int8_t* qg, const float* sg, const int8_t* qd, const float* sd, int64_t experts,
                    int64_t hidden, int64_t inter, const int8_t* sh_qg, const float* sh_sg, const int8_t* sh_qu,
                    const float* sh_su, const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w,
                    const void* residual, void* out, int dtype, void* ws, int* err, void** stage_events,
                    void* stream);

/* Allocation-free form of lmoe_routed_moe (no counterpart in the reference: the reference
 * runtime allocates its own buffers with torch).  For callers that cannot allocate device
 * memory where they run the block: host runtimes that hand out device memory only from a
 * fixed, pre-sized arena they keep to themselves, and C/FFI hosts that link this library
 * with no device allocator of their own.  Same arguments as lmoe_routed_moe without
 * ws/stage_events; the scratch is a file-scope device array of
 * lmoe_routed_moe_noalloc_limit() bytes (16 MiB) that each GPU using the library keeps for
 * the life of the process.  Returns LMOE_ERR_UNSUPPORTED when lmoe_moe_workspace_size()
 * for the call exceeds that limit (at hidden 2048, inter 512, top 8 and 256 experts about 200
 * tokens fit; 256 do not), LMOE_ERR_INVALID for hidden or inter above 2^20.  The first call
 * in each CUDA context (per device) looks up the array's device address, which may load the
 * module: make it before any stream capture.  All calls share the array and a call leaves
 * its contents behind, so calls that overlap on the GPU (different streams, or different
 * threads) race: serialise them. */
LMOE_API int64_t lmoe_routed_moe_noalloc_limit(void);
LMOE_API int lmoe_routed_moe_noalloc(const void* x, const float* weights, const int64_t* ids, int64_t tokens,
                            int64_t top, const int8_t* qg, const float* sg, const int8_t* qd, const float* sd,
                            int64_t experts, int64_t hidden, int64_t inter, const int8_t* sh_qg,
                            const float* sh_sg, const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd,
                            const float* sh_sd, const void* sh_gate_w, const void* residual, void* out,
                            int dtype, int* err, void* stream);

/* One-token decode of the MoE block: replaces the decode branch of Int8Experts.forward
 * (qwen35_deploy/operators/int8.py:158-187: the ids.cpu() sync, the descriptor table
 * upload of int8.py:139-153/170-179, grouped_linear for gate_up, silu*up, grouped_linear
 * for down, _ordered_reduce of int8.py:240-250) and, when sh_qg != NULL, the HF shared
 * expert and its sigmoid gate (modeling_qwen3_5_moe.py:781-790, three Int8Linear calls).
 * x [1, hidden]; ids [top] int64 and weights [top] fp32 (the router's row); banks as in
 * lmoe_routed_moe; w8a8 != 0 selects the W8A8 grouped GEMV for the routed experts (the
 * reference's --activation w8a8, cli.py:37-39), else W8A16; the shared expert always uses
 * the W8A16 arithmetic of Int8Linear.  out [1, hidden] = ordered routed combine (+ gated
 * shared) (+ residual).  One launch (gate_up, a grid barrier, down); the experts' ascending
 * order is built on the device from ids: no host synchronisation, so the call can be
 * captured in a CUDA graph.  hidden and inter up to 4096 (else LMOE_ERR_UNSUPPORTED);
 * weights, scales, x and ws 16-byte aligned.  ws: lmoe_decode_workspace_size() bytes whose
 * first 8 KiB are zero before the first call (the kernel's grid barrier keeps one counter
 * per grid size there, at the same offset for every geometry, and leaves them usable after
 * every call; after a call that set LMOE_DEVERR_TIMEOUT, zero them again).  Calls that
 * share a workspace must not overlap on the GPU.  An id outside [0, experts) sets
 * LMOE_DEVERR_BAD_EXPERT in *err. */
LMOE_API int64_t lmoe_decode_workspace_size(int64_t top, int64_t hidden, int64_t inter);
LMOE_API int lmoe_decode_moe(const void* x, const float* weights, const int64_t* ids, int64_t top,
                             const int8_t* qg, const float* sg, const int8_t* qd, const float* sd,
                             int64_t experts, int64_t hidden, int64_t inter, const int8_t* sh_qg,
                             const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                             const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w,
                             const void* residual, void* out, int dtype, int w8a8, void* ws, int* err,
                             void* stream);

/* Router tail of the sparse-MoE block: replaces the HF Qwen3_5MoeTopKRouter.forward tail
 * (transformers qwen3_5_moe/modeling_qwen3_5_moe.py:765-769) that the reference drives
 * unchanged (qwen35_deploy/model.py:57-68 swaps only the experts and the linears).
 * logits [tokens, experts] in the activation dtype (the block's F.linear(x, gate.weight));
 * weights [tokens, top] fp32 = topk(softmax(float(logits))) / their sum, ids [tokens, top]
 * int64 in descending probability, ties to the lower expert id; probs (nullable)
 * [tokens, experts] fp32 = the softmax (HF returns it as router_logits).  experts must be
 * 32, 64, 128, 256 or 512 (else LMOE_ERR_UNSUPPORTED); 1 <= top <= min(32, experts). */
LMOE_API int lmoe_router_topk(const void* logits, int64_t tokens, int64_t experts, int64_t top, float* weights,
                              int64_t* ids, float* probs, int dtype, void* stream);

/* Diagnostic (no reference counterpart): the SwiGLU epilogue of the routed gate_up
 * (torch.nn.functional.silu(gate) * up, qwen35_deploy/runtime/gpu_routes.py:75) evaluates silu
 * with a branch-free correctly rounded division; this counts, over all 65,536 16-bit
 * patterns of `dtype` taken as the gate value, the inputs where that SiLU differs from
 * fp32 g / (1 + expf(-g)) with an IEEE division.  *mismatches (device int32) is added to;
 * 0 after the stream means every input agrees bit for bit. */
LMOE_API int lmoe_selftest_silu(int dtype, int* mismatches, void* stream);

/* The router on tensor cores (replaces the HF Qwen3_5MoeTopKRouter.forward,
 * transformers qwen3_5_moe/modeling_qwen3_5_moe.py:762-770, that the reference keeps,
 * qwen35_deploy/model.py:57-68): logits = x [tokens, hidden] . router_w [experts, hidden]^T
 * with fp32 accumulation rounded to the activation dtype, then lmoe_router_topk's tail on
 * them in the same kernel.  logits (nullable) receives them [tokens, experts], probs
 * (nullable) the fp32 softmax.  experts 64, 128 or 256, hidden % 64 == 0, 1 <= top <=
 * min(32, experts) (else LMOE_ERR_INVALID); x, router_w, logits, ws 16-byte aligned; ws:
 * lmoe_router_gemm_workspace_size(tokens, experts) bytes (fp32 partial sums of K). */
LMOE_API int64_t lmoe_router_gemm_workspace_size(int64_t tokens, int64_t experts);
LMOE_API int lmoe_router_gemm_topk(const void* x, const void* router_w, int64_t tokens, int64_t hidden,
                                   int64_t experts, int64_t top, float* weights, int64_t* ids, float* probs,
                                   void* logits, void* ws, int dtype, int* err, void* stream);

/* The whole sparse-MoE block from the hidden states: lmoe_router_gemm_topk (which also
 * counts each 128-token tile's routes per expert when top == 8, the first step of the
 * routing metadata) and then lmoe_routed_moe's launches on the routing it produced; the
 * routing is returned in weights [tokens, top] fp32 and ids [tokens, top] int64.  HF
 * Qwen3_5MoeSparseMoeBlock.forward (modeling_qwen3_5_moe.py:781-792) with the experts the
 * reference installs.  ws: lmoe_moe_workspace_size(tokens, top, experts, hidden, inter)
 * bytes.  Geometry outside lmoe_router_gemm_topk's: LMOE_ERR_UNSUPPORTED. */
LMOE_API int lmoe_moe_block_router(const void* x, const void* router_w, int64_t tokens, int64_t top,
                                   const int8_t* qg, const float* sg, const int8_t* qd, const float* sd,
                                   int64_t experts, int64_t hidden, int64_t inter, const int8_t* sh_qg,
                                   const float* sh_sg, const int8_t* sh_qu, const float* sh_su,
                                   const int8_t* sh_qd, const float* sh_sd, const void* sh_gate_w,
                                   const void* residual, void* out, float* weights, int64_t* ids, int dtype,
                                   void* ws, int* err, void* stream);

#define LMOE_WIRE_DTYPE 0 /* expert-parallel dispatch payload: the hidden row in the activation dtype */
#define LMOE_WIRE_INT8 1  /* ... or its W8A8 activation quantisation (w8a8.quantize, operators/w8a8.py:8-22) */

/* Expert-parallel MoE layer with fixed-size exchanges (no host synchronisation
 * inside a layer).  The reference runs the whole block on one GPU
 * (gpu_routes.routed_moe, qwen35_deploy/runtime/gpu_routes.py:66-82, inside the HF
 * block, modeling_qwen3_5_moe.py:781-792): these three calls split that block
 * around two exchanges of equal-sized segments.  `experts` is the global expert
 * count E, sharded over `world` ranks (1..8) in contiguous blocks of E / world;
 * every rank uses the same `cap` (>= its tokens) so that all segments have the
 * same size.
 *
 * 1. lmoe_ep_dispatch: from this rank's x [tokens, hidden], ids [tokens, top]
 *    (global expert ids) and weights [tokens, top] fp32, fills W segments of
 *    [cap + 1][row_bytes]: segment d, row 0 = header (row count, routes per local
 *    expert of rank d), rows 1.. = one packed row per token with a route to rank d
 *    (tokens ascending): [payload | local ids int32 x top | weights fp32 x top |
 *    ranks int32 x top], the payload being the hidden row (wire LMOE_WIRE_DTYPE) or
 *    its W8A8 activation quantisation (LMOE_WIRE_INT8).  plan_ws:
 *    lmoe_ep_plan_workspace_size bytes, read again by lmoe_ep_fold.
 * 2. exchange: segment d of rank s goes to segment s of rank d's `recv`.
 * 3. lmoe_ep_owner: this rank's experts (banks [E/world, ...]) on the received
 *    rows, plus the shared expert on its own x; per received row the ordered sum of
 *    its routes' round(round(down) * w).  ws: lmoe_ep_owner_workspace_size bytes
 *    (256-byte aligned), read again by lmoe_ep_fold.  stage_events (nullable): 5
 *    cudaEvent_t recorded before the metadata, after the scatter, after gate_up, after
 *    down and after the combine.
 * 4. exchange: partial segment s of rank d goes to segment d of rank s's `back`.
 * 5. lmoe_ep_fold: out [tokens, hidden] = the returned rows in ascending rank order,
 *    + round(sigmoid(round(x . sh_gate_w)) * shared expert) when with_shared,
 *    + residual.
 *
 * Transport.  peers == NULL: the caller runs both exchanges between the calls
 * (e.g. NCCL all_to_all with equal splits): dispatch fills `send`
 * [world][cap + 1][row_bytes], the owner reads `recv` and fills `partial`
 * [world][cap][hidden], the fold reads `back`.  peers != NULL (direct transport over
 * NVLink): every rank's `recv` and `back` buffers and flag words are mapped into
 * every process (lmoe_ipc_*); the dispatch stores segment d straight into rank d's
 * recv, the owner's combine stores straight into the senders' back buffers, and the
 * owner and the fold wait (bounded; a timeout sets LMOE_DEVERR_TIMEOUT) until every
 * peer's flag for this rank reaches `epoch`, which the caller increases by one per
 * layer on every rank alike.  flags[d] points to rank d's 2 * world 32-bit flag words
 * and counter to this rank's 2 words, all zero before the first layer.  The kernels
 * of one rank then wait on kernels of the other ranks: run one rank per GPU.
 * hidden % 256 == 0, inter % 128 == 0, 1 <= top <= 16. */
typedef struct {
  void* recv[8];  /* rank d's receive buffer, [world][cap + 1][row_bytes] */
  void* back[8];  /* rank d's return buffer, [world][cap][hidden] */
  void* flags[8]; /* rank d's flag words, 2 * world uint32 */
  void* counter;  /* this rank's 2 uint32 counters */
  int rank;
  unsigned epoch;
} lmoe_ep_peers;
LMOE_API int64_t lmoe_ep_layer_row_bytes(int64_t hidden, int64_t top, int wire);
LMOE_API int64_t lmoe_ep_plan_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t world);
LMOE_API int64_t lmoe_ep_owner_workspace_size(int64_t tokens, int64_t top, int64_t experts, int64_t world,
                                              int64_t cap, int64_t hidden, int64_t inter);
LMOE_API int lmoe_ep_dispatch(const void* x, const float* weights, const int64_t* ids, int64_t tokens, int64_t top,
                              int64_t experts, int64_t world, int64_t cap, int64_t hidden, int wire, int dtype,
                              void* send, void* plan_ws, int* err, const lmoe_ep_peers* peers, void* stream);
LMOE_API int lmoe_ep_owner(const void* recv, const void* x, int64_t tokens, int64_t top, int64_t experts,
                           int64_t world, int64_t cap, int64_t hidden, int64_t inter, int wire, const int8_t* qg,
                           const float* sg, const int8_t* qd, const float* sd, const int8_t* sh_qg,
                           const float* sh_sg, const int8_t* sh_qu, const float* sh_su, const int8_t* sh_qd,
                           const float* sh_sd, void* ws, void* partial, int dtype, int* err, void** stage_events,
                           const lmoe_ep_peers* peers, void* stream);
LMOE_API int lmoe_ep_fold(const void* back, const void* plan_ws, const void* x, int64_t tokens, int64_t top,
                          int64_t experts, int64_t world, int64_t cap, int64_t hidden, int64_t inter,
                          const void* owner_ws, int with_shared, const void* sh_gate_w, const void* residual,
                          void* out, int dtype, int* err, const lmoe_ep_peers* peers, void* stream);
/* CUDA IPC for the direct transport: the handle (64 bytes) of the allocation holding
 * ptr and ptr's offset in it; opening a peer's handle maps that allocation (base) and
 * returns the pointer at the offset; close unmaps a base. */
LMOE_API int lmoe_ipc_get_handle(const void* ptr, void* handle, int64_t* offset);
LMOE_API int lmoe_ipc_open_handle(const void* handle, int64_t offset, void** ptr, void** base);
LMOE_API int lmoe_ipc_close(void* base);

#ifdef __cplusplus
}
#endif
#endif /* LOCALMOE_B200_H */
