"""W8A16 group-128 operators (replaces qwen35_deploy/operators/int8.py).

Same call signatures, shapes, dtypes and ``ValueError`` texts as the
reference; the arithmetic runs in ``liblocalmoe_b200.so``:
* ``linear``/``Int8Linear`` -- int8.py:26-48 (GEMV for one row, tcgen05 GEMM above, K split over a
  cached workspace when the output alone would not fill the GPU);
* ``grouped_linear``        -- int8.py:233-237 (table-driven decode GEMV);
* ``ordered_reduce``        -- the launch of ``_ordered_reduce`` at int8.py:185-186;
* ``Int8Experts``           -- int8.py:127-210, with the expert bank resident in HBM.
"""
import torch

from .. import _native as N


def _weights(q, scale):
    """The weight and its group scales as the library reads them.  The reference's kernel
    indexes both as contiguous row-major tensors without checking, so a strided view is
    made contiguous here rather than refused; only a weight the library cannot read at all
    (not CUDA int8 with float32 scales) raises."""
    if not (q.is_cuda and scale.is_cuda and q.dtype == torch.int8 and scale.dtype == torch.float32):
        raise ValueError('Expected CUDA int8 weights with float32 group scales')
    return q.contiguous(), scale.contiguous()


def linear(x, q, scale, large_tile=False):
    """``y = x . round(q * scale)^T`` (int8.py:26-37).  ``large_tile`` is accepted
    for signature parity; the library picks its own tiling."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError('W8A16 requires CUDA FP16/BF16 activations')
    n, k = q.shape
    if k % 128 or x.shape[-1] != k or tuple(scale.shape) != (n, k // 128):
        raise ValueError('Invalid INT8 group geometry')
    q, scale = _weights(q, scale)
    x = x.contiguous()
    m = x.numel() // k
    out = torch.empty((*x.shape[:-1], n), device=x.device, dtype=x.dtype)
    wsb = N.lib().lmoe_linear_w8a16_workspace_size(m, n, k)
    ws = N.workspace(x.device, wsb, 'linear') if wsb > 0 else None
    N.call('lmoe_linear_w8a16_ws', N.ptr(x), N.ptr(q), N.ptr(scale), N.ptr(out), m, n, k, N.dtype_code(x.dtype),
           N.ptr(ws), wsb, N.ptr(N.error_word(x.device)), N.stream(x.device))
    return out


class Int8Linear(torch.nn.Module):
    """Buffers ``q`` [N, K] int8 and ``scale`` [N, K/128] fp32 (int8.py:40-48)."""

    def __init__(self, q, scale):
        super().__init__()
        self.register_buffer('q', q)
        self.register_buffer('scale', scale)
        self.large_prefill_tile = False

    def forward(self, x):
        return linear(x, self.q, self.scale, self.large_prefill_tile)


def grouped_linear(x, table, experts, n, field, shared):
    """Decode GEMV over a ``[experts, 5]`` int64 descriptor table of raw device
    pointers (int8.py:233-237).  Returns ``[experts, n]`` in ``x.dtype``."""
    x = x.contiguous()
    out = torch.empty((experts, n), dtype=x.dtype, device=x.device)
    N.call('lmoe_grouped_linear_w8a16', N.ptr(x), N.ptr(table), N.ptr(out), experts, n, x.shape[-1], field,
           1 if shared else 0, N.dtype_code(x.dtype), N.stream(x.device))
    return out


def ordered_reduce(values, table, weights, out):
    """``_ordered_reduce`` launch (int8.py:185-186): out[n] = ordered bf16 sum of
    round(values[e, n] * weights[table[e, 4]]) over table rows."""
    w = weights if weights.dtype == torch.float32 else weights.float()
    w = w.contiguous()
    v = values.contiguous()  # bound to a name: kept alive until the launch is enqueued
    N.call('lmoe_ordered_reduce', N.ptr(v), N.ptr(table), N.ptr(w), N.ptr(out), v.shape[-1], v.shape[0],
           N.dtype_code(out.dtype), N.stream(v.device))
    return out


class Int8Experts(torch.nn.Module):
    """The routed experts of one MoE layer with the bank resident in HBM
    (int8.py:127-210, the HF ``Qwen3_5MoeExperts`` module boundary).

    ``forward(hidden_states, top_k_index, top_k_weights)`` returns the routed
    output ``[T, H]``: one token runs the decode chain (device-built table,
    grouped GEMVs, ordered combine; int8.py:158-187), more tokens run the
    routed prefill GEMMs (gpu_routes.routed_moe).  ``activation`` selects the
    decode GEMV arithmetic, like the reference's ``--activation`` switch
    (cli.py:37-39): 'w8a16' (default, int8.grouped_linear) or 'w8a8'.
    """

    def __init__(self, gate_up_q, gate_up_scale, down_q, down_scale, activation='w8a16'):
        super().__init__()
        self.register_buffer('gate_up_q', gate_up_q)
        self.register_buffer('gate_up_scale', gate_up_scale)
        self.register_buffer('down_q', down_q)
        self.register_buffer('down_scale', down_scale)
        self.activation = activation

    def banks(self):
        return [self.gate_up_q, self.gate_up_scale, self.down_q, self.down_scale]

    def forward(self, hidden_states, top_k_index, top_k_weights):
        from ..runtime import decode, gpu_routes
        if hidden_states.shape[0] == 1:
            return decode.decode_block(hidden_states, top_k_weights, top_k_index, self.banks(),
                                       activation=self.activation)
        return gpu_routes.routed_moe(hidden_states, top_k_weights, top_k_index, self.banks())

