"""GPU routing metadata and the routed expert FFN (replaces
qwen35_deploy/runtime/gpu_routes.py).

* ``plan(ids, experts, bm)`` -- gpu_routes.py:47-63: one kernel returns the
  reference's ``(pos, table, ordered, slots)`` bit for bit;
* ``routed_moe(x, weights, ids, banks, ...)`` -- gpu_routes.py:66-82: four
  launches (metadata, gate_up GEMM with fused SwiGLU, down GEMM with the
  routing weight fused, ordered combine), no host synchronisation;
* ``moe_block(...)`` -- the same launches with the shared expert folded in as
  one more expert segment and the HF gate/add fused into the combine
  (transformers qwen3_5_moe/modeling_qwen3_5_moe.py:781-792);
* ``moe_block_router(...)`` -- the same block from the hidden states, its router
  (logits GEMM + softmax/top-k + the metadata's route counts) one more kernel
  (modeling_qwen3_5_moe.py:762-770).
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


ROUTER_EXPERTS = (64, 128, 256)  # expert counts the fused router kernel takes


def router_gemm_ok(x, router_weight, top_k):
    """Whether ``moe_block_router`` / ``router_topk_fused`` take this geometry."""
    t, h = x.shape
    return (router_weight.shape[0] in ROUTER_EXPERTS and router_weight.shape[1] == h and h % 64 == 0 and
            1 <= top_k <= min(32, router_weight.shape[0]) and t > 0)


def router_topk_fused(x, router_weight, top_k, return_probs=False, return_logits=False):
    """The router on tensor cores (``lmoe_router_gemm_topk``): the logits
    ``x . router_weight^T`` (K split over 4 CTAs per 128-token tile, the splits added in
    order), rounded to ``x.dtype``, and the fp32 softmax / top-k / renormalise tail.  Returns ``(weights, ids)`` and, as asked,
    the fp32 softmax and the logits."""
    x = x.contiguous()
    w_r = router_weight.to(x.dtype).contiguous()
    t, e = x.shape[0], w_r.shape[0]
    dev = x.device
    w = torch.empty((t, top_k), dtype=torch.float32, device=dev)
    ids = torch.empty((t, top_k), dtype=torch.int64, device=dev)
    probs = torch.empty((t, e), dtype=torch.float32, device=dev) if return_probs else None
    logits = torch.empty((t, e), dtype=x.dtype, device=dev) if return_logits else None
    ws = N.workspace(dev, N.lib().lmoe_router_gemm_workspace_size(t, e), 'router')
    N.call('lmoe_router_gemm_topk', N.ptr(x), N.ptr(w_r), t, x.shape[1], e, top_k, N.ptr(w), N.ptr(ids), N.ptr(probs),
           N.ptr(logits), N.ptr(ws), N.dtype_code(x.dtype), N.ptr(N.error_word(dev)), N.stream(dev))
    out = (w, ids)
    if return_probs:
        out = out + (probs,)
    if return_logits:
        out = out + (logits,)
    return out


def moe_block_router(x, router_weight, top_k, banks, shared=None, shared_gate_weight=None, residual=None):
    """The whole sparse-MoE block from the hidden states (``lmoe_moe_block_router``):
    the fused router kernel (which also counts the routes per expert of each 128-token
    tile for the metadata when ``top_k == 8``) and then ``moe_block``'s launches on the
    routing it produced.  Returns ``(out, weights, ids)``."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2:
        raise ValueError('Expected CUDA FP16/BF16 activations')
    x = x.contiguous()
    e, h, inter = _check_banks(x, banks)
    w_r = router_weight.to(x.dtype).contiguous()
    if w_r.shape[0] != e:
        raise ValueError('Router weight must be [experts, hidden]')
    t = x.shape[0]
    dev = x.device
    out = torch.empty_like(x)
    w = torch.empty((t, top_k), dtype=torch.float32, device=dev)
    ids = torch.empty((t, top_k), dtype=torch.int64, device=dev)
    ws = N.workspace(dev, N.lib().lmoe_moe_workspace_size(t, top_k, e, h, inter), 'moe')
    sh = [None] * 6
    if shared is not None:
        (qsg, ssg), (qsu, ssu), (qsd, ssd) = shared
        sh = [qsg, ssg, qsu, ssu, qsd, ssd]
    gate = shared_gate_weight.to(x.dtype).contiguous() if shared_gate_weight is not None else None
    qg, sg, qd, sd = banks
    N.call('lmoe_moe_block_router', N.ptr(x), N.ptr(w_r), t, top_k, N.ptr(qg), N.ptr(sg), N.ptr(qd), N.ptr(sd), e, h,
           inter, *[N.ptr(v) for v in sh], N.ptr(gate), N.ptr(residual), N.ptr(out), N.ptr(w), N.ptr(ids),
           N.dtype_code(x.dtype), N.ptr(ws), N.ptr(N.error_word(dev)), N.stream(dev))
    return out, w, ids


def routed_moe(x, weights, ids, banks, large_tile=False, ready_event=None):
    """gpu_routes.routed_moe (gpu_routes.py:66-82); ``large_tile`` is accepted
    for signature parity."""
    return moe_block(x, weights, ids, banks, ready_event=ready_event)
