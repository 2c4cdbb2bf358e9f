"""W8A8 group-128 operators (replaces qwen35_deploy/operators/w8a8.py).

``quantize`` -- per-(row, 128-group) absmax int8 activations (w8a8.py:17-22);
``grouped_linear`` -- the table-driven int8 GEMV with per-group rescale
(w8a8.py:44-48); it quantises inside the GEMV launch.
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
