"""Expert parallelism for the routed MoE block over ``torch.distributed``.

The reference runs on one GPU (its experts stream over PCIe); on B200s the
256 experts shard by contiguous blocks across G ranks (rank g owns experts
``[g*E/G, (g+1)*E/G)``) and each rank keeps its own tokens.  The sequence of one
layer:

1. every (token, destination rank) pair with at least one route to that rank
   becomes one send row -- the token's hidden row plus its routes for that
   rank (local expert ids, routing weights; unused slots -1 / 0), rows grouped
   by destination rank, tokens ascending;
2. an all-to-all carries the rows; the payload is the hidden row itself
   (``wire='bf16'``) or, with ``wire='int8'``, its W8A8 activation
   quantisation (int8 [H] + fp32 scales [H/128], operators/w8a8.py:8-22),
   2,112 instead of 4,096 bytes at H = 2048, which the owner dequantises to
   ``round_dtype(q * s)`` before its experts read it;
3. the owner runs its experts on the received rows (gate_up + SwiGLU, down,
   ``round(round(v) * w)``) and pre-reduces each row's routes in ascending
   expert order, ``acc = round(acc + v)``;
4. the reverse all-to-all returns one row per (token, rank);
5. each token folds its returned rows in ascending rank order (= ascending
   expert order: the shards are contiguous), then adds its gated shared
   expert (the shared expert and the gate are replicated) and the residual.

The rounding sequence equals the reference's single chain
(int8.py:245-249, prefill.py:44-46) except at the rank boundaries, where a
pre-reduced partial sum is added instead of its terms one by one; the results
stay within the 1e-2 bar.

Two implementations of that sequence:

* ``GpuLayer`` / ``moe_forward_gpu`` -- the product path on B200s.  Every
  exchange size is fixed in advance (W segments of ``cap + 1`` rows; row 0 of a
  segment is its header: row count and routes per local expert), so a layer has
  no host synchronisation: ``lmoe_ep_dispatch`` (the routing metadata of this
  rank's routes, the destination slots, the pack: 5 kernels), ``lmoe_ep_owner``
  (the owner's metadata, scatter, the two grouped GEMMs with the shared expert's
  own-token tiles folded in, the ordered combine: 5 kernels), ``lmoe_ep_fold``
  (1 kernel).  With the direct transport (default for W > 1) the pack and
  combine kernels store their rows straight into the peers' buffers over
  NVLink; with 'nccl' two ``all_to_all_single`` calls move them between the
  kernels.
* ``moe_forward`` -- the same sequence with variable-size exchanges and
  injected compute (``local_moe(x, weights, ids)``, ``shared_part(x)``), which
  the CPU multi-process tests (gloo) run with oracle functions to check the
  orchestration and the rounding sequence.
"""
import ctypes

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
    ascending expert order (``prereduced`` builds one from a one-route-per-row
    function).
    ``shared_part(x) -> [T, H]`` is round(sigmoid(gate) * shared_expert(x)) (or None).  ``wire`` is the format
    of the dispatched hidden rows ('bf16': the rows as they are; 'int8': W8A8
    activation quantisation, through ``quantize``: ``rows -> (q int8 [n, H], s fp32
    [n, H/128])``).  Rows are packed with torch byte views; the product path on
    GPUs is ``moe_forward_gpu``."""
    if wire not in WIRES:
        raise ValueError("wire must be 'bf16' or 'int8'")
    h = x.shape[-1]
    if h % GROUP:
        raise ValueError('hidden size must be a multiple of 128')
    if wire == 'int8' and quantize is None:
        raise ValueError('the int8 wire needs a quantize function')
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
    # 2. packed rows: payload, route ids and weights in one exchange
    n_send = route_tok.numel()
    row_bytes = wire_row_bytes(h, top, wire, x.element_size())
    if n_send:
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
    #    ascending expert order
    if n_recv:
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




# ---------------------------------------------------------------------------- GPU path
class GpuLayer:
    """Buffers and calls of one expert-parallel layer on this rank's GPU.

    ``tokens`` rows per rank (every rank must use the same ``cap`` >= its token
    count, default ``tokens``: the exchanges are equal-split), ``experts`` global
    experts sharded over ``world`` ranks, ``top`` routes per token.  The buffers
    are allocated once and reused by every layer and step of the same geometry.

    ``transport``: 'p2p' (the default with more than one rank) -- the dispatch and
    combine kernels store straight into the peers' buffers over NVLink, mapped once
    through CUDA IPC (a collective over ``group``: every rank constructs its layer
    together), and the receiving kernels wait on per-layer epoch flags; 'nccl' --
    two ``all_to_all_single`` calls between the kernels.  One rank per GPU.
    """

    FLAG_BYTES = 4096

    def __init__(self, tokens, top, experts, world, hidden, inter, dtype, device, wire='bf16', cap=None,
                 transport=None, group=None):
        from .. import _native as N
        if wire not in WIRES:
            raise ValueError("wire must be 'bf16' or 'int8'")
        transport = transport or ('p2p' if world > 1 else 'nccl')
        if transport not in ('p2p', 'nccl'):
            raise ValueError("transport must be 'p2p' or 'nccl'")
        self.N = N
        self.tokens, self.top, self.experts, self.world = int(tokens), int(top), int(experts), int(world)
        self.hidden, self.inter, self.dtype, self.wire = int(hidden), int(inter), dtype, wire
        self.cap = int(cap if cap is not None else tokens)
        self.device = torch.device(device)
        self.transport, self.group = transport, group
        self.wire_code = N.WIRE_INT8 if wire == 'int8' else N.WIRE_DTYPE
        lib = N.lib()
        self.row_bytes = lib.lmoe_ep_layer_row_bytes(self.hidden, self.top, self.wire_code)
        ows = lib.lmoe_ep_owner_workspace_size(self.tokens, self.top, self.experts, self.world, self.cap,
                                               self.hidden, self.inter)
        pws = lib.lmoe_ep_plan_workspace_size(self.tokens, self.top, self.experts, self.world)
        if min(self.row_bytes, ows, pws) < 0:
            raise ValueError('unsupported expert-parallel geometry')
        seg = (self.cap + 1) * self.row_bytes
        dev = self.device
        self.plan_ws = torch.empty(pws, dtype=torch.uint8, device=dev)
        self.owner_ws = torch.empty(ows, dtype=torch.uint8, device=dev)
        self.epoch = 0
        self._bases = []
        if transport == 'nccl':
            self.peers = None
            self.send = torch.empty(self.world * seg, dtype=torch.uint8, device=dev)
            self.recv = self.send if self.world == 1 else torch.empty_like(self.send)
            self.partial = torch.empty((self.world * self.cap, self.hidden), dtype=dtype, device=dev)
            self.back = self.partial if self.world == 1 else torch.empty_like(self.partial)
            return
        # one allocation: [flag words | receive buffer | return buffer], shared with the peers
        back_bytes = self.world * self.cap * self.hidden * torch.empty((), dtype=dtype).element_size()
        self.exbuf = torch.zeros(self.FLAG_BYTES + self.world * seg + back_bytes, dtype=torch.uint8, device=dev)
        self.counter = torch.zeros(2, dtype=torch.int32, device=dev)
        self.send = None
        self.recv = self.exbuf[self.FLAG_BYTES:self.FLAG_BYTES + self.world * seg]
        self.back = self.exbuf[self.FLAG_BYTES + self.world * seg:].view(dtype).view(self.world * self.cap,
                                                                                     self.hidden)
        self.partial = None
        rank = dist.get_rank(group) if self.world > 1 else 0
        handle = (ctypes.c_uint8 * 64)()
        off = ctypes.c_int64()
        N.call('lmoe_ipc_get_handle', ctypes.c_void_p(self.exbuf.data_ptr()), handle, ctypes.byref(off))
        mine = torch.tensor(list(bytes(handle)) + list(int(off.value).to_bytes(8, 'little')), dtype=torch.uint8,
                            device=dev)
        everyone = torch.empty((self.world, 72), dtype=torch.uint8, device=dev)
        if self.world > 1:
            dist.all_gather_into_tensor(everyone, mine, group=group)
        else:
            everyone[0] = mine
        table = everyone.cpu().numpy()
        p = N.EpPeers()
        for d in range(self.world):
            if d == rank:
                ptr = self.exbuf.data_ptr()
            else:
                h = (ctypes.c_uint8 * 64)(*table[d, :64].tolist())
                o = int.from_bytes(bytes(table[d, 64:].tolist()), 'little')
                out, base = ctypes.c_void_p(), ctypes.c_void_p()
                N.call('lmoe_ipc_open_handle', h, o, ctypes.byref(out), ctypes.byref(base))
                self._bases.append(base)
                ptr = out.value
            p.flags[d] = ptr
            p.recv[d] = ptr + self.FLAG_BYTES
            p.back[d] = ptr + self.FLAG_BYTES + self.world * seg
        p.counter = self.counter.data_ptr()
        p.rank = rank
        self.peers = p
        if self.world > 1:
            dist.barrier(group=group)

    def close(self):
        """Unmap the peers' buffers (direct transport; every rank calls it together)."""
        if self._bases:
            torch.cuda.synchronize(self.device)
            if self.world > 1:
                dist.barrier(group=self.group)
            for b in self._bases:
                self.N.call('lmoe_ipc_close', b)
            self._bases = []

    def _peers_arg(self):
        return None if self.peers is None else ctypes.byref(self.peers)

    def _check(self, x, weights, ids):
        if x.shape != (self.tokens, self.hidden) or x.dtype != self.dtype or not x.is_contiguous():
            raise ValueError('x does not match the layer geometry')
        if ids.shape != (self.tokens, self.top) or weights.shape != (self.tokens, self.top):
            raise ValueError('routing does not match the layer geometry')

    def dispatch(self, x, weights, ids):
        """This rank's tokens and their routing into the send segments (direct
        transport: into the peers' receive buffers).  Starts a new layer epoch."""
        N = self.N
        self._check(x, weights, ids)
        ids = ids if ids.dtype == torch.int64 else ids.long()
        weights = weights if weights.dtype == torch.float32 else weights.float()
        if self.peers is not None:
            self.epoch = (self.epoch + 1) & 0xffffffff
            self.peers.epoch = self.epoch
        N.call('lmoe_ep_dispatch', N.ptr(x), N.ptr(weights.contiguous()), N.ptr(ids.contiguous()), self.tokens,
               self.top, self.experts, self.world, self.cap, self.hidden, self.wire_code, N.dtype_code(self.dtype),
               N.ptr(self.send), N.ptr(self.plan_ws), N.ptr(N.error_word(self.device)), self._peers_arg(),
               N.stream(self.device))

    def owner(self, x, banks, shared=None, stage_events=None):
        """This rank's experts on the received rows (+ the shared expert on its own
        ``x``); ``banks`` hold the local experts ``[E / world, ...]``."""
        N = self.N
        qg, sg, qd, sd = banks
        if qg.shape != (self.experts // self.world, 2 * self.inter, self.hidden):
            raise ValueError('local expert bank does not match the layer geometry')
        sh = [None] * 6
        if shared is not None:
            (qsg, ssg), (qsu, ssu), (qsd, ssd) = shared
            sh = [qsg, ssg, qsu, ssu, qsd, ssd]
        evs = None
        if stage_events is not None:
            for ev in stage_events:
                ev.record()
            evs = (ctypes.c_void_p * 5)(*[ctypes.c_void_p(ev.cuda_event) for ev in stage_events])
        N.call('lmoe_ep_owner', N.ptr(self.recv), N.ptr(x), self.tokens, self.top, self.experts, self.world,
               self.cap, self.hidden, self.inter, self.wire_code, N.ptr(qg), N.ptr(sg), N.ptr(qd), N.ptr(sd),
               *[N.ptr(v) for v in sh], N.ptr(self.owner_ws), N.ptr(self.partial), N.dtype_code(self.dtype),
               N.ptr(N.error_word(self.device)), evs, self._peers_arg(), N.stream(self.device))
        self.with_shared = shared is not None

    def fold(self, x, shared_gate_weight=None, residual=None):
        """Per token: the returned rows (``back``) in ascending rank order, the
        gated shared expert computed by ``owner`` and the residual."""
        N = self.N
        out = torch.empty_like(x)
        gate = None if shared_gate_weight is None else shared_gate_weight.to(self.dtype).contiguous()
        N.call('lmoe_ep_fold', N.ptr(self.back), N.ptr(self.plan_ws), N.ptr(x), self.tokens, self.top, self.experts,
               self.world, self.cap, self.hidden, self.inter, N.ptr(self.owner_ws), 1 if self.with_shared else 0,
               N.ptr(gate), N.ptr(residual), N.ptr(out), N.dtype_code(self.dtype), N.ptr(N.error_word(self.device)),
               self._peers_arg(), N.stream(self.device))
        return out

    def exchange(self, out, inp, group=None):
        """The caller-run exchange of the 'nccl' transport (nothing to do with 'p2p')."""
        if self.peers is None and self.world > 1:
            dist.all_to_all_single(out, inp, group=group if group is not None else self.group)

    def forward(self, x, weights, ids, banks, shared=None, shared_gate_weight=None, residual=None, group=None,
                events=None):
        """One expert-parallel layer for this rank's ``x [tokens, hidden]``.  ``events``
        (optional): 6 CUDA events recorded around dispatch, the first exchange, the
        owner, the return exchange and the fold (with the direct transport the
        exchanges happen inside dispatch and owner, and the waits for them inside
        owner and fold)."""
        def mark(i):
            if events is not None:
                events[i].record()
        mark(0)
        self.dispatch(x, weights, ids)
        mark(1)
        self.exchange(self.recv, self.send, group)
        mark(2)
        self.owner(x, banks, shared)
        mark(3)
        self.exchange(self.back, self.partial, group)
        mark(4)
        out = self.fold(x, shared_gate_weight, residual)
        mark(5)
        return out


_layers = {}


def moe_forward_gpu(x, weights, ids, experts, banks, shared=None, shared_gate_weight=None, residual=None,
                    group=None, wire='bf16', cap=None, transport=None):
    """Expert-parallel MoE block on this rank's GPU (``GpuLayer``, cached per
    geometry; its first call is a collective when the transport is 'p2p'): ``banks``
    are this rank's experts ``[experts / world, ...]``, ``shared``/``shared_gate_weight``
    the replicated shared expert and its gate."""
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    t, top = ids.shape
    key = (x.device, t, top, experts, world, x.shape[1], banks[2].shape[2], x.dtype, wire, cap, transport, group)
    layer = _layers.get(key)
    if layer is None:
        layer = _layers[key] = GpuLayer(t, top, experts, world, x.shape[1], banks[2].shape[2], x.dtype, x.device,
                                        wire, cap, transport, group)
    return layer.forward(x.contiguous(), weights, ids, banks, shared, shared_gate_weight, residual, group)
