"""CPU baseline: the reference's PyTorch dequantise-then-matmul expert path.

TEST/BENCH INFRASTRUCTURE: timed by ``bench.py`` (its ``cpu_baseline`` leg and
``--impl reference``) on the host cores; never called by the package.

It restates HF ``Qwen3_5MoeExperts.forward`` (transformers qwen3_5_moe/
modeling_qwen3_5_moe.py:727-751) -- one-hot routing mask, a loop over hit
experts, ``linear`` for gate_up, ``silu(gate) * up``, ``linear`` for down,
``* top_k_weights`` and ``index_add_`` -- on weights dequantised from the
converted INT8 g128 layout (``q.float() * scale``, convert.py:31-37), in fp32,
plus the shared expert MLP and its sigmoid gate (hf :781-792).
"""
import os
import time

import numpy as np
import torch


def dequant(q, s):
    return q.float() * s.repeat_interleave(128, -1)


def experts_forward(x, top_k_index, top_k_weights, qg, sg, qd, sd):
    final = torch.zeros_like(x)
    num_experts = qg.shape[0]
    expert_mask = torch.nn.functional.one_hot(top_k_index, num_classes=num_experts).permute(2, 1, 0)
    hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero()
    for e in hit[:, 0].tolist():
        top_k_pos, token_idx = torch.where(expert_mask[e])
        cur = x[token_idx]
        gate, up = torch.nn.functional.linear(cur, dequant(qg[e], sg[e])).chunk(2, dim=-1)
        h = torch.nn.functional.silu(gate) * up
        h = torch.nn.functional.linear(h, dequant(qd[e], sd[e]))
        h = h * top_k_weights[token_idx, top_k_pos, None]
        final.index_add_(0, token_idx, h)
    return final


def moe_block(x, top_k_index, top_k_weights, bank, shared, gate_w):
    qg, sg, qd, sd = bank
    routed = experts_forward(x, top_k_index, top_k_weights, qg, sg, qd, sd)
    (q1, s1), (q2, s2), (q3, s3) = shared
    g = torch.nn.functional.linear(x, dequant(q1, s1))
    u = torch.nn.functional.linear(x, dequant(q2, s2))
    sh = torch.nn.functional.linear(torch.nn.functional.silu(g) * u, dequant(q3, s3))
    return routed + torch.sigmoid(torch.nn.functional.linear(x, gate_w)) * sh


def make_case(tokens=256, experts=256, hidden=2048, inter=512, top=8, seed=0, exact_quant=False):
    """Config C1-style inputs: N(0,1) activations, Zipf-biased softmax top-8
    routing, INT8 g128 weights.  With ``exact_quant`` the weights are N(0,0.02)
    quantised by the converter's rule; otherwise int8 values and scales are
    drawn directly (same layout and cost, ~20x faster to generate)."""
    g = torch.Generator().manual_seed(seed)

    def quant(shape):
        if not exact_quant:
            q = torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)
            s = (torch.rand(shape[:-1] + (shape[-1] // 128,), generator=g) + 0.5) * (0.06 / 127)
            return q, s
        w = torch.randn(shape, generator=g) * 0.02
        v = w.reshape(*shape[:-1], shape[-1] // 128, 128)
        s = v.abs().amax(-1).div(127).clamp_min(1e-30)
        q = (v / s.unsqueeze(-1)).round().clamp(-127, 127).to(torch.int8)
        return q.reshape(shape), s

    qg, sg = quant((experts, 2 * inter, hidden))
    qd, sd = quant((experts, hidden, inter))
    shared = [quant((inter, hidden)), quant((inter, hidden)), quant((hidden, inter))]
    gate_w = torch.randn((1, hidden), generator=g) * 0.02
    x = torch.randn((tokens, hidden), generator=g).bfloat16().float()
    ranks = torch.randperm(experts, generator=g) + 1
    logits = torch.randn((tokens, experts), generator=g) - 1.1 * torch.log(ranks.float())[None]
    p = torch.softmax(logits, dim=-1)
    w, idx = torch.topk(p, top, dim=-1)
    w = w / w.sum(-1, keepdim=True)
    return x, idx, w, (qg, sg, qd, sd), shared, gate_w


def time_layer(case, repeats=3, threads=None, warmup=True):
    """Median seconds for one MoE block on the host (after 1 warm-up call unless
    ``warmup`` is False)."""
    threads = threads or os.cpu_count()
    torch.set_num_threads(threads)
    x, idx, w, bank, shared, gate_w = case
    with torch.no_grad():
        if warmup:
            moe_block(x, idx, w, bank, shared, gate_w)
        times = []
        for _ in range(repeats):
            t0 = time.perf_counter()
            moe_block(x, idx, w, bank, shared, gate_w)
            times.append(time.perf_counter() - t0)
    return float(np.median(times)), threads


def cpu_model():
    try:
        for line in open('/proc/cpuinfo'):
            if line.startswith('model name'):
                return line.split(':', 1)[1].strip()
    except OSError:
        pass
    return 'unknown'
