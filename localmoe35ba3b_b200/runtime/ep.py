"""Expert parallelism for the routed MoE block over ``torch.distributed``.

The reference runs on one GPU (its experts stream over PCIe); on B200s the
256 experts shard by contiguous blocks across G GPUs (rank g owns experts
``[g*E/G, (g+1)*E/G)``) and each rank keeps its own tokens.  One layer:

1. ``plan``: every (token, destination rank) pair with at least one route to
   that rank becomes one send row -- the token's hidden row plus its routes
   for that rank (local expert ids, routing weights; unused slots -1 / 0).
   Rows are grouped by destination rank, tokens ascending.
2. ``all_to_all_single`` of the row counts, then ONE of the packed send rows
   (NCCL on GPUs, gloo on CPU).  A packed row is ``[payload | route ids int32
   x top | route weights fp32 x top]`` as bytes; the payload is the hidden row
   itself (``wire='bf16'``) or, with ``wire='int8'``, its W8A8 activation
   quantisation (int8 [H] + fp32 scales [H/128], operators/w8a8.py:8-22):
   2,112 instead of 4,096 bytes at H = 2048.  The owner dequantises an int8
   row to ``round_dtype(q * s)`` before its experts read it.
3. The owner runs its routed experts on the received rows with their route
   lists (``gpu_routes.moe_block``; -1 slots, routed to other ranks, are
   skipped: gate_up + SwiGLU, down, ``round(round(v) * w)``), whose ordered
   combine pre-reduces each row's routes in ascending expert order:
   ``acc = round(acc + v)``.
4. The reverse ``all_to_all_single`` returns one row per (token, rank).
5. Each token folds its returned rows in ascending rank order (= ascending
   expert order, the shards are contiguous), adds its gated shared expert
   (computed locally -- the shared expert and the gate are replicated -- while
   the dispatch exchange of step 2 is in flight) and the residual.

The rounding sequence equals the reference's single chain
(int8.py:245-249, prefill.py:44-46) except at the rank boundaries, where a
pre-reduced partial sum is added instead of its terms one by one; the results
stay within the 1e-2 bar (tests/test_ep.py checks both the bound and the exact
EP sequence against the oracle).  The int8 wire adds the activation
quantisation error of the routed experts' input (the shared expert reads the
local bf16 row); the return trip always carries the dtype rows.

The compute is injected (``local_moe(x, weights, ids)`` and
``shared_part(x)``), so the same orchestration runs the GPU kernels in the
product and oracle functions in the CPU multi-process tests.
"""
import torch
import torch.distributed as dist


def plan_counts(ids, experts, world):
    """Device-side first half of ``plan``: ``(dest [T, top], mask [T, world], send_counts
    [world] int64)``, no host synchronisation."""
    t, top = ids.shape
    if experts % world:
        raise ValueError('experts must divide evenly across ranks')
    e_loc = experts // world
    dest = torch.div(ids.long(), e_loc, rounding_mode='floor')                   # [T, top]
    mask = torch.zeros((t, world), dtype=torch.bool, device=ids.device)
    mask.scatter_(1, dest, True)
    return dest, mask, mask.sum(0).to(torch.int64)


def plan_rows(ids, weights, experts, dest, mask, n):
    """Second half of ``plan`` for ``n`` (host-known) send rows: the selected
    (rank, token) pairs in ascending (rank, token) order come first in a stable
    sort of the unselected flags, so no ``nonzero`` (and no synchronisation) is
    needed."""
    t = ids.shape[0]
    world = mask.shape[1]
    e_loc = experts // world
    flat = (~mask.t()).reshape(-1).to(torch.int8)                                 # 0 = selected, index g*T + t
    order = torch.argsort(flat, stable=True)[:n]
    g_idx, t_idx = torch.div(order, t, rounding_mode='floor'), order % t
    rows_ids = ids.long()[t_idx]                                                  # [n, top]
    mine = dest[t_idx] == g_idx[:, None]
    route_ids = torch.where(mine, rows_ids - g_idx[:, None] * e_loc, torch.full_like(rows_ids, -1)).to(torch.int32)
    route_w = torch.where(mine, weights[t_idx].float(), torch.zeros((), dtype=torch.float32, device=ids.device))
    return t_idx, route_ids, route_w


def plan(ids, weights, experts, world):
    """Send rows for one rank's tokens.

    Returns ``(send_tok [n] int64, send_counts [world] int64, route_ids [n, top]
    int32 local expert ids or -1, route_w [n, top] fp32)``; rows are grouped by
    destination rank (ascending), tokens ascending within a rank."""
    dest, mask, send_counts = plan_counts(ids, experts, world)
    t_idx, route_ids, route_w = plan_rows(ids, weights, experts, dest, mask, int(send_counts.sum()))
    return t_idx, send_counts, route_ids, route_w


def _round_add(acc, v):
    """round_dtype(acc + v) elementwise (fp32 add of two dtype values, one rounding)."""
    return (acc.float() + v.float()).to(acc.dtype)


def expand_routes(route_ids, route_w):
    """Received rows -> one entry per route, sorted by (row, local expert id).

    Returns ``(row [R'], expert [R'], weight [R'], rank_in_row [R'], max_routes)``."""
    valid = route_ids >= 0
    row, slot = torch.nonzero(valid, as_tuple=True)
    expert = route_ids[row, slot].long()
    weight = route_w[row, slot]
    n = route_ids.shape[0]
    # lexicographic (row, expert): stable sort by expert, then stable sort by row
    o = torch.argsort(expert, stable=True)
    row, expert, weight = row[o], expert[o], weight[o]
    o = torch.argsort(row, stable=True)
    row, expert, weight = row[o], expert[o], weight[o]
    counts = torch.bincount(row, minlength=n)
    first = torch.cumsum(counts, 0) - counts
    rank = torch.arange(row.numel(), device=row.device) - first[row]
    max_routes = int(counts.max().item()) if n else 0
    return row, expert, weight, rank, max_routes


def prereduce(out_routes, row, rank, n_rows, max_routes, like):
    """Per received row: acc = round(acc + v) over its routes in ascending expert order."""
    acc = torch.zeros((n_rows, like.shape[-1]), dtype=like.dtype, device=like.device)
    for j in range(max_routes):
        sel = rank == j
        r = row[sel]
        acc[r] = _round_add(acc[r], out_routes[sel])
    return acc


def _a2a(out, inp, out_splits, in_splits, group):
    dist.all_to_all_single(out, inp, output_split_sizes=out_splits, input_split_sizes=in_splits, group=group)


WIRES = ('bf16', 'int8')
GROUP = 128


def _bytes(t):
    """A contiguous 2-D tensor's rows as uint8 ``[n, row bytes]``."""
    return t.contiguous().view(torch.uint8).reshape(t.shape[0], -1)


def _field(buf, start, stop, dtype):
    """Columns ``[start, stop)`` of uint8 rows, reinterpreted as ``dtype`` rows."""
    return buf[:, start:stop].contiguous().view(dtype)


def wire_row_bytes(h, top, wire, itemsize=2):
    """Bytes of one packed send row: payload + route ids + route weights."""
    if wire not in WIRES:
        raise ValueError("wire must be 'bf16' or 'int8'")
    payload = h + 4 * (h // GROUP) if wire == 'int8' else itemsize * h
    return payload + 8 * top


def pack_rows(rows, route_ids, route_w, wire, quantize=None):
    """Send rows -> uint8 ``[n, wire_row_bytes]``: ``[payload | ids | weights]``.
    With ``wire='int8'`` the payload is ``quantize(rows) -> (q int8 [n, H], s fp32
    [n, H/128])`` (the W8A8 activation quantiser) as bytes."""
    if wire == 'int8':
        q, s = quantize(rows)
        parts = [_bytes(q), _bytes(s)]
    elif wire == 'bf16':
        parts = [_bytes(rows)]
    else:
        raise ValueError("wire must be 'bf16' or 'int8'")
    parts += [_bytes(route_ids.to(torch.int32)), _bytes(route_w.to(torch.float32))]
    return torch.cat(parts, dim=1)


def route_fields(buf, h, top, wire, dtype):
    """Route ids int32 ``[n, top]`` and weights fp32 ``[n, top]`` of packed rows."""
    n = buf.shape[0]
    off = wire_row_bytes(h, top, wire, torch.empty((), dtype=dtype).element_size()) - 8 * top
    ids = _field(buf, off, off + 4 * top, torch.int32)
    w = _field(buf, off + 4 * top, off + 8 * top, torch.float32)
    return ids.reshape(n, top), w.reshape(n, top)


def unpack_rows(buf, h, top, wire, dtype):
    """Received packed rows -> ``(rows dtype [n, H], route ids int32 [n, top],
    route weights fp32 [n, top])``; int8 payloads become ``round_dtype(float(q) * s)``
    per 128-column group."""
    n = buf.shape[0]
    if wire == 'int8':
        g = h // GROUP
        q = _field(buf, 0, h, torch.int8)
        s = _field(buf, h, h + 4 * g, torch.float32)
        rows = (q.float().view(n, g, GROUP) * s.view(n, g, 1)).view(n, h).to(dtype)
    else:
        rows = _field(buf, 0, torch.empty((), dtype=dtype).element_size() * h, dtype)
    return (rows.reshape(n, h), *route_fields(buf, h, top, wire, dtype))


def _wire_code(wire):
    from .. import _native as N
    return N.WIRE_INT8 if wire == 'int8' else N.WIRE_DTYPE


def pack_rows_gpu(x, tok, route_ids, route_w, wire):
    """``pack_rows(x[tok], ...)`` in one kernel (``lmoe_ep_pack_rows``): gather, W8A8
    quantisation on the int8 wire, route ids and weights."""
    from .. import _native as N
    x, tok = x.contiguous(), tok.to(torch.int64).contiguous()
    route_ids = route_ids.to(torch.int32).contiguous()
    route_w = route_w.to(torch.float32).contiguous()
    n, top = route_ids.shape
    h = x.shape[-1]
    out = torch.empty((n, wire_row_bytes(h, top, wire, x.element_size())), dtype=torch.uint8, device=x.device)
    N.call('lmoe_ep_pack_rows', N.ptr(x), x.shape[0], N.ptr(tok), N.ptr(route_ids), N.ptr(route_w), n, h, top,
           _wire_code(wire), N.ptr(out), N.dtype_code(x.dtype), N.ptr(N.error_word(x.device)), N.stream(x.device))
    return out


def unpack_rows_gpu(buf, row_of, h, top, wire, dtype):
    """Payload of packed row ``row_of[r]`` (row r when ``row_of`` is None) as
    activation row r, in one kernel (``lmoe_ep_unpack_rows``; the int8 wire
    dequantised to ``round_dtype(q * s)``)."""
    from .. import _native as N
    if row_of is not None:
        row_of = row_of.to(torch.int64).contiguous()
    n = buf.shape[0] if row_of is None else row_of.numel()
    y = torch.empty((n, h), dtype=dtype, device=buf.device)
    N.call('lmoe_ep_unpack_rows', N.ptr(buf.contiguous()), buf.shape[0], N.ptr(row_of), n, h, top,
           _wire_code(wire), N.ptr(y), N.dtype_code(dtype), N.ptr(N.error_word(buf.device)), N.stream(buf.device))
    return y


def prereduced(route_fn):
    """A ``local_moe`` built from a one-route-per-row expert function
    ``route_fn(x_rows [R', H], w [R', 1], ids [R', 1]) -> [R', H]``: the received
    rows are expanded into one row per route, and each received row's routes are
    then summed in ascending expert order, ``acc = round(acc + v)``."""
    def run(x_rows, w, ids):
        row, expert, weight, rank, max_routes = expand_routes(ids, w)
        if not row.numel():
            return torch.zeros_like(x_rows)
        y = route_fn(x_rows[row].contiguous(), weight[:, None].contiguous(), expert[:, None].contiguous())
        return prereduce(y, row, rank, x_rows.shape[0], max_routes, x_rows)
    return run


def moe_forward(x, weights, ids, experts, local_moe, shared_part=None, residual=None, group=None,
                wire='bf16', quantize=None):
    """Expert-parallel MoE block for this rank's tokens ``x [T, H]``.

    ``local_moe(x_rows [n, H], w [n, top] fp32, ids [n, top] int32) -> [n, H]``
    runs this rank's experts on the received rows: ids are local expert ids,
    -1 where the slot routes to another rank, and row i of the result is
    ``acc = round(acc + round(round(down_e(x_i)) * w))`` over the row's routes in
    ascending expert order (``gpu_local_moe``: the routed block itself;
    ``prereduced``: the same from a one-route-per-row function).
    ``shared_part(x) -> [T, H]`` is round(sigmoid(gate) * shared_expert(x)) (or None).  ``wire`` is the format
    of the dispatched hidden rows ('bf16': the rows as they are; 'int8': W8A8
    activation quantisation).  CUDA tensors pack and unpack through the library
    kernels; CPU ranks (gloo) pack with torch and quantise through ``quantize``
    (``rows -> (q int8 [n, H], s fp32 [n, H/128])``)."""
    if wire not in WIRES:
        raise ValueError("wire must be 'bf16' or 'int8'")
    h = x.shape[-1]
    if h % GROUP:
        raise ValueError('hidden size must be a multiple of 128')
    if wire == 'int8' and not x.is_cuda and quantize is None:
        raise ValueError('the int8 wire on CPU ranks needs a quantize function')
    world = dist.get_world_size(group)
    # 1. counts: computed and exchanged on the device, then read once (the layer's one
    #    host synchronisation: the exchange sizes must be known on the host)
    dest, mask, send_counts = plan_counts(ids, experts, world)
    recv_counts = torch.empty_like(send_counts)
    dist.all_to_all_single(recv_counts, send_counts, group=group)
    counts = torch.cat([send_counts, recv_counts]).tolist()
    sc, rc = counts[:world], counts[world:]
    n_recv, top = sum(rc), ids.shape[1]
    route_tok, route_ids, route_w = plan_rows(ids, weights, experts, dest, mask, sum(sc))
    # 2. packed rows: payload, route ids and weights in one exchange (on the GPU one
    #    kernel gathers, quantises and packs; CPU ranks pack with torch byte views)
    n_send = route_tok.numel()
    row_bytes = wire_row_bytes(h, top, wire, x.element_size())
    if x.is_cuda:
        send_buf = pack_rows_gpu(x, route_tok, route_ids, route_w, wire)
    elif n_send:
        send_buf = pack_rows(x[route_tok].contiguous(), route_ids, route_w, wire, quantize)
    else:
        send_buf = torch.empty((0, row_bytes), dtype=torch.uint8, device=x.device)
    recv_buf = torch.empty((n_recv, row_bytes), dtype=torch.uint8, device=x.device)
    # the exchange runs asynchronously (NCCL on its own stream) while this rank's gated
    # shared expert, which reads only the local rows, runs on the current stream
    work = dist.all_to_all_single(recv_buf, send_buf, output_split_sizes=rc, input_split_sizes=sc, group=group,
                                  async_op=True)
    sh = shared_part(x) if shared_part is not None else None
    work.wait()
    # 3. local experts on the received rows, each row's routes pre-reduced in
    #    ascending expert order (on GPUs the block's own ordered combine)
    if n_recv:
        if x.is_cuda:
            recv_rows = unpack_rows_gpu(recv_buf, None, h, top, wire, x.dtype)
            recv_ids, recv_w = route_fields(recv_buf, h, top, wire, x.dtype)
        else:
            recv_rows, recv_ids, recv_w = unpack_rows(recv_buf, h, top, wire, x.dtype)
        partial = local_moe(recv_rows, recv_w, recv_ids)
    else:
        partial = torch.zeros((0, h), dtype=x.dtype, device=x.device)
    # 4. partial rows back to their tokens' ranks
    back = torch.empty((n_send, h), dtype=x.dtype, device=x.device)
    _a2a(back, partial, sc, rc, group)
    # 5. per token: ascending rank order, then the gated shared expert, then the residual
    #    (the rows are grouped by rank, sc[g] of them for rank g, each token at most once
    #    per rank: host-known slices, no device synchronisation)
    out = torch.zeros_like(x)
    start = 0
    for g in range(world):
        stop = start + sc[g]
        if stop > start:
            tok = route_tok[start:stop]
            out[tok] = _round_add(out[tok], back[start:stop])
        start = stop
    if sh is not None:
        out = _round_add(out, sh)
    if residual is not None:
        out = _round_add(residual, out)
    return out


def gpu_local_moe(banks):
    """This rank's experts through the routed-MoE kernels on the received rows:
    a -1 id is a slot routed elsewhere, which the block's routing metadata sorts
    after every expert, gives no GEMM tile and leaves out of the ordered combine,
    so the combine is the per-row pre-reduction."""
    from . import gpu_routes

    def run(x_rows, w, ids):
        return gpu_routes.moe_block(x_rows, w, ids, banks)
    return run


def gpu_shared_part(banks, shared, shared_gate_weight):
    """round(sigmoid(round(x . gate)) * shared_expert(x)) through the same library call
    with no routed experts (top 0)."""
    from . import gpu_routes

    def run(x):
        t = x.shape[0]
        ids = torch.empty((t, 0), dtype=torch.int64, device=x.device)
        w = torch.empty((t, 0), dtype=torch.float32, device=x.device)
        return gpu_routes.moe_block(x, w, ids, banks, shared=shared, shared_gate_weight=shared_gate_weight)
    return run
