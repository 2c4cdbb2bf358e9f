"""GPU routing metadata and the routed expert FFN (replaces
qwen35_deploy/runtime/gpu_routes.py).

* ``plan(ids, experts, bm)`` -- gpu_routes.py:47-63: one kernel returns the
  reference's ``(pos, table, ordered, slots)`` bit for bit;
* ``routed_moe(x, weights, ids, banks, ...)`` -- gpu_routes.py:66-82: four
  launches (metadata, gate_up GEMM with fused SwiGLU, down GEMM with the
  routing weight fused, ordered combine), no host synchronisation;
* ``moe_block(...)`` -- the same launches with the shared expert folded in as
  one more expert segment and the HF gate/add fused into the combine
  (transformers qwen3_5_moe/modeling_qwen3_5_moe.py:781-792).
"""
import ctypes

import torch

from .. import _native as N


def plan(ids, experts, bm):
    if ids.device.type != 'cuda' or ids.ndim != 2 or not ids.is_contiguous():
        raise ValueError('Expected contiguous CUDA [tokens,top_k] routing IDs')
    if ids.dtype != torch.int64:
        ids = ids.long()
    t, top = ids.shape
    routes = t * top
    dev = ids.device
    pos = torch.empty(routes, dtype=torch.int64, device=dev)
    table = torch.empty(((routes + bm - 1) // bm + experts, 3), dtype=torch.int64, device=dev)
    ordered = torch.empty((t, top), dtype=torch.int64, device=dev)
    slots = torch.empty((t, top), dtype=torch.int64, device=dev)
    ws = N.workspace(dev, N.lib().lmoe_plan_workspace_size(t, top, experts), 'plan')
    N.call('lmoe_plan', N.ptr(ids), t, top, experts, bm, N.ptr(pos), N.ptr(table), N.ptr(ordered), N.ptr(slots),
           N.ptr(ws), N.stream(dev))
    return pos, table, ordered, slots


def _check_banks(x, banks):
    qg, sg, qd, sd = banks
    e, n2, h = qg.shape
    if (h != x.shape[-1] or n2 % 2 or tuple(sg.shape) != (e, n2, h // 128) or qd.shape[0] != e
            or qd.shape[1] != h or qd.shape[2] != n2 // 2 or tuple(sd.shape) != (e, h, n2 // 256)):
        raise ValueError('Invalid INT8 expert bank geometry')
    for t in banks:
        if not t.is_cuda or not t.is_contiguous():
            raise ValueError('Expert banks must be contiguous CUDA tensors')
    return e, h, n2 // 2


def moe_block(x, weights, ids, banks, shared=None, shared_gate_weight=None, residual=None, ready_event=None,
              stage_events=None):
    """Routed experts (+ gated shared expert, + residual) for ``x [T, H]``.

    ``banks = [qg [E,2I,H], sg [E,2I,H/128], qd [E,H,I], sd [E,H,I/128]]``;
    ``shared = ((q_gate, s_gate), (q_up, s_up), (q_down, s_down))`` of the
    shared expert's Int8Linear layers; ``shared_gate_weight`` [1, H] in x.dtype.
    """
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2:
        raise ValueError('Expected CUDA [tokens, hidden] FP16/BF16 activations')
    if ids.device.type != 'cuda' or ids.ndim != 2:
        raise ValueError('Expected contiguous CUDA [tokens,top_k] routing IDs')
    x = x.contiguous()
    ids = ids.contiguous() if ids.dtype == torch.int64 else ids.long().contiguous()
    w = weights.float().contiguous() if weights.dtype != torch.float32 else weights.contiguous()
    e, h, inter = _check_banks(x, banks)
    t, top = ids.shape
    dev = x.device
    out = torch.empty_like(x)
    ws = N.workspace(dev, N.lib().lmoe_moe_workspace_size(t, top, e, h, inter), 'moe')
    sh = [None] * 6
    if shared is not None:
        (qsg, ssg), (qsu, ssu), (qsd, ssd) = shared
        if (tuple(qsg.shape) != (inter, h) or tuple(qsu.shape) != (inter, h) or tuple(qsd.shape) != (h, inter)):
            raise ValueError('Shared expert must have the routed experts\' shapes')
        sh = [qsg, ssg, qsu, ssu, qsd, ssd]
    gate = None
    if shared_gate_weight is not None:
        gate = shared_gate_weight.to(x.dtype).contiguous()
    if ready_event is not None:
        torch.cuda.current_stream(dev).wait_event(ready_event)
    qg, sg, qd, sd = banks
    evs = None
    if stage_events is not None:
        # torch only reports elapsed_time for events it recorded itself; record
        # each once here, the library then re-records it at its stage boundary
        for ev in stage_events:
            ev.record()
        evs = (ctypes.c_void_p * 5)(*[ctypes.c_void_p(ev.cuda_event) for ev in stage_events])
    N.call('lmoe_routed_moe', N.ptr(x), N.ptr(w), N.ptr(ids), t, top, N.ptr(qg), N.ptr(sg), N.ptr(qd), N.ptr(sd),
           e, h, inter, *[N.ptr(v) for v in sh], N.ptr(gate), N.ptr(residual), N.ptr(out), N.dtype_code(x.dtype),
           N.ptr(ws), N.ptr(N.error_word(dev)), evs, N.stream(dev))
    return out


def routed_moe(x, weights, ids, banks, large_tile=False, ready_event=None):
    """gpu_routes.routed_moe (gpu_routes.py:66-82); ``large_tile`` is accepted
    for signature parity."""
    return moe_block(x, weights, ids, banks, ready_event=ready_event)
