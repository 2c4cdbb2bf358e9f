"""Seeded inputs for the golden fixtures (shared by make_golden.py and tests).

Every generator is deterministic (NumPy PCG64 with a fixed seed) and depends
only on NumPy, so the GPU box can rebuild the exact inputs of each fixture.
Shapes are small, odd where the kernels mask (N not a multiple of the tile,
token counts not a multiple of 16) and use K divisible by 128.
"""
import hashlib
import os
import sys

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__)))))
from oracle.oracle import quantize_weight, bf16_bits, to_bf16, route, zipf_bias  # noqa: E402


def _rng(tag):
    return np.random.default_rng(int.from_bytes(hashlib.sha256(tag.encode()).digest()[:8], 'little'))


def weight_quant_input():
    r = _rng('wq')
    w = r.standard_normal((3, 2, 256), dtype=np.float32) * 0.02
    w[0, 0, :128] = 0.0          # an all-zero group: scale clamps to 1e-30
    w[1, 1, 5] = 0.5             # an outlier dominating its group
    return w


def act_quant_input():
    """bf16 bit patterns [6, 384]: random rows, a zero row, a tiny row and a
    row of exact multiples of its scale that land on .5 ties."""
    r = _rng('aq')
    x = r.standard_normal((6, 384), dtype=np.float32) * 3
    x[1] = 0.0
    x[2] *= 1e-12
    x[3] = np.round(r.standard_normal(384) * 40) / 2 + 0.25
    x[4, :128] = 127.0
    x[4, 7] = 0.5
    x[4, 8] = -1.5
    return bf16_bits(x)


def linear_inputs():
    r = _rng('lin')
    x = r.standard_normal((37, 384), dtype=np.float32).astype(np.float16)
    q, s = quantize_weight(r.standard_normal((96, 384), dtype=np.float32) * 0.02)
    return x, q, s


def grouped_inputs():
    r = _rng('grouped')
    H, I, E = 256, 128, 5
    qg, sg = quantize_weight(r.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.02)
    qd, sd = quantize_weight(r.standard_normal((E, H, I), dtype=np.float32) * 0.02)
    experts = np.array([0, 2, 3], dtype=np.int64)
    slots = np.array([1, 2, 0], dtype=np.int64)
    xs = r.standard_normal((1, H), dtype=np.float32)
    xr = r.standard_normal((3, I), dtype=np.float32)
    return dict(qg=qg, sg=sg, qd=qd, sd=sd, experts=experts, slots=slots,
                x_shared=xs.astype(np.float16), x_rows=xr.astype(np.float16),
                x_shared_bf16=bf16_bits(xs), x_rows_bf16=bf16_bits(xr))


def reduce_inputs():
    r = _rng('reduce')
    v = r.standard_normal((8, 300), dtype=np.float32).astype(np.float16)
    slots = r.permutation(8).astype(np.int64)
    w = r.random((1, 8), dtype=np.float32)
    w = (w / w.sum()).astype(np.float32)
    return v, slots, w


def _distinct_ids(r, t, top, experts, bias=None):
    logits = r.standard_normal((t, experts), dtype=np.float32)
    if bias is not None:
        logits = logits + bias[None]
    return route(logits, top)[0]


def route_cases():
    r = _rng('routes')
    cases = {}
    cases['uniform'] = (_distinct_ids(r, 37, 8, 16), 16)
    cases['skew'] = (_distinct_ids(r, 29, 4, 12, zipf_bias(12, r)), 12)
    cases['tiny'] = (_distinct_ids(r, 1, 8, 16), 16)
    cases['dups'] = (r.integers(0, 4, size=(5, 3)).astype(np.int64), 4)
    cases['empty_experts'] = (np.array([[7, 3], [3, 7], [7, 9]], dtype=np.int64), 12)
    return cases


def routed_inputs():
    r = _rng('routed')
    T, H, I, E, top = 24, 256, 128, 6, 4
    qg, sg = quantize_weight(r.standard_normal((E, 2 * I, H), dtype=np.float32) * 0.02)
    qd, sd = quantize_weight(r.standard_normal((E, H, I), dtype=np.float32) * 0.02)
    x = r.standard_normal((T, H), dtype=np.float32).astype(np.float16)
    logits = r.standard_normal((T, E), dtype=np.float32) + zipf_bias(E, r)[None]
    ids, w = route(logits, top)
    return dict(x=x, qg=qg, sg=sg, qd=qd, sd=sd, ids=ids, weights=w)


def checksums():
    h = hashlib.sha256()
    h.update(weight_quant_input().tobytes())
    h.update(act_quant_input().tobytes())
    for a in linear_inputs():
        h.update(np.ascontiguousarray(a).tobytes())
    g = grouped_inputs()
    for k in sorted(g):
        h.update(np.ascontiguousarray(g[k]).tobytes())
    for a in reduce_inputs():
        h.update(a.tobytes())
    for k, (ids, e) in sorted(route_cases().items()):
        h.update(ids.tobytes())
    r = routed_inputs()
    for k in sorted(r):
        h.update(np.ascontiguousarray(r[k]).tobytes())
    return np.frombuffer(h.digest(), dtype=np.uint8)


_ = to_bf16  # re-exported for tests
