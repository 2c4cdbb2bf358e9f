"""W8A8 group-128 operators (replaces qwen35_deploy/operators/w8a8.py).

``quantize`` -- per-(row, 128-group) absmax int8 activations (w8a8.py:17-22);
``grouped_linear`` -- the table-driven int8 GEMV with per-group rescale
(w8a8.py:44-48); it quantises inside the GEMV launch;
``linear`` -- the same arithmetic for a dense linear of any number of rows on int8
tensor cores (the dense sweep's W8A8 half; the reference has it only as the one-row
GEMV).
"""
import torch

from .. import _native as N


def quantize(x):
    x = x.contiguous()
    k = x.shape[-1]
    if not x.is_cuda or x.ndim != 2 or k % 128:
        raise ValueError('Expected CUDA rows with K divisible by 128')
    q = torch.empty_like(x, dtype=torch.int8)
    s = torch.empty((x.shape[0], k // 128), device=x.device, dtype=torch.float32)
    N.call('lmoe_quantize_rows', N.ptr(x), N.ptr(q), N.ptr(s), x.shape[0], k, N.dtype_code(x.dtype),
           N.stream(x.device))
    return q, s


def grouped_linear(x, table, experts, n, field, shared, return_quantized=False):
    x = x.contiguous()
    out = torch.empty((experts, n), device=x.device, dtype=x.dtype)
    k = x.shape[-1]
    xq = xs = None
    if return_quantized:
        xq = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        xs = torch.empty((x.shape[0], k // 128), dtype=torch.float32, device=x.device)
    N.call('lmoe_grouped_linear_w8a8', N.ptr(x), N.ptr(table), N.ptr(out), experts, n, k, field,
           1 if shared else 0, N.dtype_code(x.dtype), N.ptr(xq), N.ptr(xs), N.stream(x.device))
    return (out, xq, xs) if return_quantized else out


def linear(x, q, scale):
    """``y = W8A8(x) . W^T`` for ``x [..., K]`` (FP16/BF16, CUDA), ``q [N, K]`` int8 and
    ``scale [N, K/128]`` fp32: each row of x quantised as ``quantize``, exact int32 dots
    per 128-group on tensor cores, ``acc = acc + (float(dot) * xs) * ws`` in group order
    (w8a8.py:37-40), rounded once to ``x.dtype``.  N must be a multiple of 128."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError('W8A8 requires CUDA FP16/BF16 activations')
    n, k = q.shape
    if k % 128 or x.shape[-1] != k or tuple(scale.shape) != (n, k // 128) or n % 128:
        raise ValueError('Invalid INT8 group geometry')
    if not (q.is_cuda and scale.is_cuda and q.dtype == torch.int8 and scale.dtype == torch.float32):
        raise ValueError('Expected CUDA int8 weights with float32 group scales')
    q, scale, x = q.contiguous(), scale.contiguous(), x.contiguous()
    m = x.numel() // k
    out = torch.empty((*x.shape[:-1], n), device=x.device, dtype=x.dtype)
    if m == 0:
        return out
    ws = N.workspace(x.device, N.lib().lmoe_linear_w8a8_workspace_size(m, k), 'w8a8')
    N.call('lmoe_linear_w8a8', N.ptr(x), N.ptr(q), N.ptr(scale), N.ptr(out), m, n, k, N.dtype_code(x.dtype),
           N.ptr(ws), N.ptr(N.error_word(x.device)), N.stream(x.device))
    return out
