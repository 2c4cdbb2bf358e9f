"""One-token MoE decode (replaces the decode branch of Int8Experts.forward,
qwen35_deploy/operators/int8.py:158-187, and the HF shared expert + gate of
modeling_qwen3_5_moe.py:781-790).

``decode_block`` runs the whole block for ``x [1, H]`` as one library call
(``lmoe_decode_moe``, one kernel launch): the experts' order is built on the
device from the router's ids (no ``ids.cpu()`` synchronisation and no table
upload), then the gate_up GEMV + silu*up, a grid barrier, the down GEMV and the
ordered combine with the gated shared expert.  Nothing synchronises with the
host, so a caller can capture a whole decode step in a CUDA graph.
"""
import torch

from .. import _native as N
from .gpu_routes import _check_banks


def decode_block(x, weights, ids, banks, shared=None, shared_gate_weight=None, residual=None, activation='w8a8'):
    """``x [1, H]`` -> ``[1, H]``: routed experts (``activation`` 'w8a8' as
    installed by the reference's ``--activation w8a8`` (cli.py:37-39), or
    'w8a16') + the gated shared expert (always the W8A16 Int8Linear arithmetic)
    + ``residual``.  ``weights``/``ids`` are the router's ``[1, top]`` row."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16) or x.ndim != 2 or x.shape[0] != 1:
        raise ValueError('Expected one CUDA FP16/BF16 token row [1, hidden]')
    if ids.device.type != 'cuda' or ids.ndim != 2 or ids.shape[0] != 1:
        raise ValueError('Expected contiguous CUDA [tokens,top_k] routing IDs')
    if activation not in ('w8a8', 'w8a16'):
        raise ValueError("activation must be 'w8a8' or 'w8a16'")
    x = x.contiguous()
    ids = ids.contiguous() if ids.dtype == torch.int64 else ids.long().contiguous()
    w = weights.float().contiguous() if weights.dtype != torch.float32 else weights.contiguous()
    e, h, inter = _check_banks(x, banks)
    top = ids.shape[1]
    dev = x.device
    sh = [None] * 6
    if shared is not None:
        (qsg, ssg), (qsu, ssu), (qsd, ssd) = shared
        if (tuple(qsg.shape) != (inter, h) or tuple(qsu.shape) != (inter, h) or tuple(qsd.shape) != (h, inter)):
            raise ValueError('Shared expert must have the routed experts\' shapes')
        sh = [qsg, ssg, qsu, ssu, qsd, ssd]
    gate = shared_gate_weight.to(x.dtype).contiguous() if shared_gate_weight is not None else None
    res = residual.to(x.dtype).contiguous() if residual is not None else None
    out = torch.empty_like(x)
    # zero-filled once: the kernel's grid barrier keeps its counter at zero between calls
    ws = N.workspace(dev, N.lib().lmoe_decode_workspace_size(top, h, inter), 'decode', zeroed=True)
    qg, sg, qd, sd = banks
    N.call('lmoe_decode_moe', N.ptr(x), N.ptr(w), N.ptr(ids), top, N.ptr(qg), N.ptr(sg), N.ptr(qd), N.ptr(sd), e, h,
           inter, *[N.ptr(v) for v in sh], N.ptr(gate), N.ptr(res), N.ptr(out), N.dtype_code(x.dtype),
           1 if activation == 'w8a8' else 0, N.ptr(ws), N.ptr(N.error_word(dev)), N.stream(dev))
    return out
