"""NumPy restatement of the reference's INT8 group-128 MoE matmul path.

TEST INFRASTRUCTURE: the CPU checker for the CUDA kernels in
``localmoe35ba3b_b200``. It is never called by the package itself.

Every function names the reference file:line it restates (paths are inside the
reference project ``heliosz616/LocalMoe35Ba3b``; ``hf/...`` means the installed
third-party ``transformers`` 5.5.0 module
``transformers/models/qwen3_5_moe/modeling_qwen3_5_moe.py`` that the reference
drives).

Floating-point conventions:
* activations and stored outputs are ``float32`` arrays that hold values exactly
  representable in the activation dtype (``'bf16'`` or ``'f16'``); ``round_to``
  performs the IEEE round-to-nearest-even store conversion;
* sums whose order the reference leaves to ``tl.dot`` are accumulated in
  float64 here (``linear_w8a16``) -- the GPU result must then agree within a
  tolerance, stated in the tests;
* every step whose order the reference fixes (the W8A8 per-group rescale, the
  ordered bf16 combine, activation quantisation, routing metadata) is restated
  operation by operation in float32/int arithmetic, so the GPU must agree
  bit for bit.
"""
import numpy as np

GROUP = 128
_F32 = np.float32


# --------------------------------------------------------------------------
# dtype helpers
# --------------------------------------------------------------------------
def bf16_bits(a):
    """float32 -> bf16 bit pattern (uint16), round to nearest even."""
    a = np.ascontiguousarray(a, dtype=np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = ((u + 0x7FFF + ((u >> 16) & 1)) >> 16).astype(np.uint16)
    nan = np.isnan(a)
    if nan.any():
        r = np.where(nan, np.uint16(0x7FC0), r)
    return r


def bf16_from_bits(b):
    """bf16 bit pattern (uint16) -> float32 values."""
    b = np.ascontiguousarray(b, dtype=np.uint16)
    return (b.astype(np.uint32) << 16).view(np.float32)


def to_bf16(a):
    return bf16_from_bits(bf16_bits(a))


def round_to(a, dtype):
    """Store conversion float32 -> activation dtype (value kept as float32)."""
    a = np.asarray(a, dtype=np.float32)
    if dtype == 'bf16':
        return to_bf16(a)
    if dtype == 'f16':
        return a.astype(np.float16).astype(np.float32)
    if dtype == 'f32':
        return a
    raise ValueError(dtype)


def dequant(q, scale, dtype=None):
    """``(q.float() * s)`` expanded over 128-wide K groups, optionally rounded
    to the activation dtype as ``operators/int8.py:19-21`` does."""
    q = np.asarray(q)
    s = np.repeat(np.asarray(scale, dtype=np.float32), GROUP, axis=-1)
    w = q.astype(np.float32) * s
    return w if dtype is None else round_to(w, dtype)


# --------------------------------------------------------------------------
# a15  weight quantiser (layout producer)  -- convert.py:31-37
# --------------------------------------------------------------------------
def quantize_weight(w):
    """Per-128-K-group absmax RTN: ``scale = max|v| / 127`` (IEEE divide),
    clamped below at 1e-30; ``q = clamp(rint(v / scale), +-127)`` as int8.
    Returns ``(q int8 [..., K], scale float32 [..., K/128])``."""
    w = np.asarray(w, dtype=np.float32)
    shape = w.shape
    v = w.reshape(*shape[:-1], shape[-1] // GROUP, GROUP)
    scale = np.abs(v).max(-1) / _F32(127)
    scale = np.maximum(scale, _F32(1e-30)).astype(np.float32)
    q = np.clip(np.rint(v / scale[..., None]), -127, 127).astype(np.int8)
    return q.reshape(shape), scale


# --------------------------------------------------------------------------
# a5  W8A8 activation quantiser  -- operators/w8a8.py:8-22
# --------------------------------------------------------------------------
def quantize_act(x):
    """Per (row, 128-group): ``s = max(absmax, 1e-10) * fp32(1/127)`` (a
    multiply, not a divide); ``q = rint_half_even(x / s)`` with an IEEE
    division; no clamp (|q| <= 127 by construction)."""
    x = np.asarray(x, dtype=np.float32)
    rows, k = x.shape
    if k % GROUP:
        raise ValueError('Expected CUDA rows with K divisible by 128')
    v = x.reshape(rows, k // GROUP, GROUP)
    amax = np.abs(v).max(-1)
    s = (np.maximum(amax, _F32(1e-10)) * _F32(1.0 / 127.0)).astype(np.float32)
    q = np.rint(v / s[..., None]).astype(np.int8)
    return q.reshape(rows, k), s


# --------------------------------------------------------------------------
# a1  dense W8A16 linear  -- operators/int8.py:9-37
# --------------------------------------------------------------------------
def linear_w8a16(x, q, scale, dtype='bf16'):
    """``Y = X . round_dtype(q * s)^T`` accumulated (here exactly, in float64),
    stored in the activation dtype.  ``x`` is ``[..., K]``."""
    x = np.asarray(x, dtype=np.float32)
    w = dequant(q, scale, dtype).astype(np.float64)
    y = x.reshape(-1, x.shape[-1]).astype(np.float64) @ w.T
    return round_to(y.astype(np.float32), dtype).reshape(*x.shape[:-1], w.shape[0])


def linear_fp32_reference(x, q, scale):
    """The north-star tolerance reference: fp32 dequantise-then-matmul with no
    rounding of the dequantised weight (float64 sums)."""
    x = np.asarray(x, dtype=np.float64)
    w = dequant(q, scale).astype(np.float64)
    return (x.reshape(-1, x.shape[-1]) @ w.T).reshape(*x.shape[:-1], w.shape[0])


# --------------------------------------------------------------------------
# a6  W8A8 GEMV/GEMM  -- operators/w8a8.py:25-41
# --------------------------------------------------------------------------
def group_dots(xq, wq):
    """Exact int32 per-group dot products: ``[M, N, K/128]``."""
    xq = np.asarray(xq, dtype=np.int64)
    wq = np.asarray(wq, dtype=np.int64)
    m, k = xq.shape
    n = wq.shape[0]
    g = k // GROUP
    xg = xq.reshape(m, g, GROUP)
    wg = wq.reshape(n, g, GROUP)
    return np.einsum('mgk,ngk->mng', xg, wg).astype(np.int32)


def linear_w8a8_acc(xq, xs, wq, ws):
    """fp32 accumulator before the store: for g in order,
    ``acc = acc + (float(dot_g) * xs[g]) * ws[n, g]`` (no fused multiply-add)."""
    dots = group_dots(xq, wq)
    xs = np.asarray(xs, dtype=np.float32)
    ws = np.asarray(ws, dtype=np.float32)
    m, n, g = dots.shape
    acc = np.zeros((m, n), dtype=np.float32)
    for b in range(g):
        t = (dots[:, :, b].astype(np.float32) * xs[:, b:b + 1]).astype(np.float32)
        t = (t * ws[None, :, b]).astype(np.float32)
        acc = (acc + t).astype(np.float32)
    return acc


def linear_w8a8(xq, xs, wq, ws, dtype='bf16'):
    return round_to(linear_w8a8_acc(xq, xs, wq, ws), dtype)


# --------------------------------------------------------------------------
# a4 / a6  table-driven decode GEMV  -- int8.py:213-237, w8a8.py:44-48
# --------------------------------------------------------------------------
def grouped_linear_w8a16(x, weights, shared, dtype='bf16'):
    """``weights`` lists ``(q, s)`` per table row (the table's pointer pair);
    row e uses x row 0 when ``shared`` else x row e."""
    x = np.asarray(x, dtype=np.float32).reshape(-1, np.asarray(weights[0][0]).shape[1])
    out = []
    for e, (q, s) in enumerate(weights):
        xr = x[0 if shared else e][None]
        out.append(linear_w8a16(xr, q, s, dtype)[0])
    return np.stack(out)


def grouped_linear_w8a8(x, weights, shared, dtype='bf16'):
    """``w8a8.grouped_linear``: quantise every row of x, then the per-group
    rescaled int8 GEMV per table row."""
    xq, xs = quantize_act(x)
    out = []
    for e, (q, s) in enumerate(weights):
        r = 0 if shared else e
        out.append(linear_w8a8(xq[r:r + 1], xs[r:r + 1], q, s, dtype)[0])
    return np.stack(out)


# --------------------------------------------------------------------------
# a7  ordered bf16 combine  -- int8.py:240-250
# --------------------------------------------------------------------------
def ordered_reduce(values, slots, weights, dtype='bf16'):
    """``acc = round(acc + round(V[e] * W[slot_e]))`` over table rows in order."""
    values = np.asarray(values, dtype=np.float32)
    w = np.asarray(weights, dtype=np.float32).reshape(-1)
    acc = np.zeros(values.shape[1], dtype=np.float32)
    for e, slot in enumerate(slots):
        v = round_to(values[e] * w[int(slot)], dtype)
        acc = round_to(acc + v, dtype)
    return acc


# --------------------------------------------------------------------------
# a8  CPU route planner  -- operators/routing.py:5-20
# --------------------------------------------------------------------------
def plan_routes(ids, experts):
    ids = np.asarray(ids)
    if ids.ndim != 2 or ids.size == 0:
        raise ValueError('Expected nonempty CPU [tokens,top_k] IDs')
    if int(ids.min()) < 0 or int(ids.max()) >= experts:
        raise ValueError('Out-of-range expert ID')
    flat = ids.reshape(-1)
    order = np.argsort(flat, kind='stable')
    counts = np.bincount(flat, minlength=experts)
    positions = np.stack((order // ids.shape[1], order % ids.shape[1])).astype(np.int64)
    segments, start = [], 0
    for e, c in enumerate(counts.tolist()):
        if c:
            segments.append((e, start, start + c))
            start += c
    return positions, segments


# --------------------------------------------------------------------------
# a9  GPU route plan  -- runtime/gpu_routes.py:17-36 (_table), 47-63 (plan)
# --------------------------------------------------------------------------
def plan(ids, experts, bm):
    """Returns ``(pos, table, ordered, slots)`` exactly as ``gpu_routes.plan``."""
    ids = np.asarray(ids, dtype=np.int64)
    t, top = ids.shape
    flat = ids.reshape(-1)
    routes = flat.size
    original = np.argsort(flat, kind='stable')
    sorted_ids = flat[original]
    offsets = np.searchsorted(sorted_ids, np.arange(experts + 1), side='left')
    counts = offsets[1:] - offsets[:-1]
    ends = np.cumsum((counts + bm - 1) // bm)
    max_tiles = -(-routes // bm) + experts
    table = np.zeros((max_tiles, 3), dtype=np.int64)
    total = int(ends[experts - 1])
    for tile in range(min(total, max_tiles)):
        expert = int(np.searchsorted(ends, tile, side='right'))
        prior = int(ends[expert - 1]) if expert > 0 else 0
        table[tile] = (expert, offsets[expert] + (tile - prior) * bm, offsets[expert + 1])
    slots = np.argsort(ids, axis=1, kind='stable').astype(np.int64)
    inverse = np.empty(routes, dtype=np.int64)
    inverse[original] = np.arange(routes)
    ordered = inverse[np.arange(t)[:, None] * top + slots]
    return (original // top).astype(np.int64), table, ordered, slots


def expert_offsets(ids, experts):
    """Exclusive prefix of per-expert route counts (``offsets`` in plan)."""
    flat = np.asarray(ids, dtype=np.int64).reshape(-1)
    counts = np.bincount(flat, minlength=experts)
    return np.concatenate([[0], np.cumsum(counts)]).astype(np.int64)


# --------------------------------------------------------------------------
# a10-a13  prefill routed expert FFN  -- runtime/prefill.py:12-49,
#          runtime/gpu_routes.py:66-82
# --------------------------------------------------------------------------
def silu_mul(gate, up, dtype='bf16'):
    """``silu(gate) * up`` on dtype tensors (gpu_routes.py:74-75): silu is
    evaluated in fp32 and stored, then the product is evaluated and stored."""
    g = np.asarray(gate, dtype=np.float32)
    s = round_to(g / (_F32(1) + np.exp(-g)), dtype)
    return round_to(s * np.asarray(up, dtype=np.float32), dtype)


def routed_linear(x, q_bank, s_bank, pos, offsets, gather, dtype='bf16'):
    """``_routed`` over every non-empty expert segment (prefill.py:12-34):
    row r of expert e reads ``x[pos[r]]`` (gather) or ``x[r]``."""
    x = np.asarray(x, dtype=np.float32)
    routes = int(offsets[-1])
    n = q_bank.shape[1]
    y = np.zeros((routes, n), dtype=np.float32)
    for e in range(len(offsets) - 1):
        a, b = int(offsets[e]), int(offsets[e + 1])
        if a == b:
            continue
        rows = x[np.asarray(pos[a:b])] if gather else x[a:b]
        y[a:b] = linear_w8a16(rows, q_bank[e], s_bank[e], dtype)
    return y


def routed_reduce(down, ordered, slots, weights, dtype='bf16'):
    """``_reduce`` (prefill.py:37-49): per token, ordered combine of its
    routes in ascending expert order."""
    down = np.asarray(down, dtype=np.float32)
    w = np.asarray(weights, dtype=np.float32)
    t, top = ordered.shape
    acc = np.zeros((t, down.shape[1]), dtype=np.float32)
    for i in range(top):
        wv = w[np.arange(t), slots[:, i]][:, None]
        v = round_to(down[ordered[:, i]] * wv, dtype)
        acc = round_to(acc + v, dtype)
    return acc


def routed_moe(x, weights, ids, banks, dtype='bf16', return_parts=False):
    """``gpu_routes.routed_moe`` (gpu_routes.py:66-82)."""
    qg, sg, qd, sd = banks
    experts = qg.shape[0]
    pos, _, ordered, slots = plan(ids, experts, 16)
    offsets = expert_offsets(ids, experts)
    gu = routed_linear(x, qg, sg, pos, offsets, True, dtype)
    inter = gu.shape[1] // 2
    hidden = silu_mul(gu[:, :inter], gu[:, inter:], dtype)
    down = routed_linear(hidden, qd, sd, pos, offsets, False, dtype)
    out = routed_reduce(down, ordered, slots, weights, dtype)
    if return_parts:
        return out, dict(gu=gu, hidden=hidden, down=down, pos=pos,
                         ordered=ordered, slots=slots, offsets=offsets)
    return out


# --------------------------------------------------------------------------
# a14  HF sparse-MoE block semantics  -- hf/modeling_qwen3_5_moe.py:697-792
# --------------------------------------------------------------------------
def shared_expert(x, shared, dtype='bf16'):
    """``Qwen3_5MoeMLP.forward`` over three ``Int8Linear`` layers
    (hf :708-710; model.py:61-62 swaps the nn.Linear for Int8Linear)."""
    (qg, sg), (qu, su), (qd, sd) = shared
    g = linear_w8a16(x, qg, sg, dtype)
    u = linear_w8a16(x, qu, su, dtype)
    return linear_w8a16(silu_mul(g, u, dtype), qd, sd, dtype)


def shared_gate_combine(routed, shared_out, x, gate_w, dtype='bf16'):
    """``expert_output + sigmoid(shared_expert_gate(x)) * shared`` (hf :784-790):
    the gate logit is a dtype linear (fp32 sum, stored), sigmoid is evaluated
    in fp32 and stored, the product and the sum are each stored."""
    x = np.asarray(x, dtype=np.float64)
    logit = round_to((x @ np.asarray(gate_w, dtype=np.float64).reshape(-1)).astype(np.float32), dtype)
    sig = round_to(_F32(1) / (_F32(1) + np.exp(-logit)), dtype)
    shw = round_to(sig[:, None] * np.asarray(shared_out, dtype=np.float32), dtype)
    return round_to(np.asarray(routed, dtype=np.float32) + shw, dtype)


def moe_block(x, weights, ids, banks, shared, gate_w, dtype='bf16'):
    """Prefill MoE block output: routed experts (W8A16 routed GEMM) plus the
    gated shared expert."""
    routed = routed_moe(x, weights, ids, banks, dtype)
    sh = shared_expert(x, shared, dtype)
    return shared_gate_combine(routed, sh, x, gate_w, dtype)


# --------------------------------------------------------------------------
# a2 decode (T=1) -- int8.py:158-187 with w8a8.grouped_linear installed
#                    (cli.py:37-39), plus the HF shared expert and gate
# --------------------------------------------------------------------------
def decode_routed(x, ids, weights, banks, activation='w8a8', dtype='bf16'):
    """Routed experts for one token: table rows in ascending expert id, the
    table-driven gate_up GEMV, silu*up, the down GEMV, the ordered combine."""
    qg, sg, qd, sd = banks
    ids = np.asarray(ids).reshape(-1)
    order = sorted((int(e), s) for s, e in enumerate(ids.tolist()))
    gl = grouped_linear_w8a8 if activation == 'w8a8' else grouped_linear_w8a16
    x = np.asarray(x, dtype=np.float32).reshape(1, -1)
    gu = gl(x, [(qg[e], sg[e]) for e, _ in order], True, dtype)
    inter = gu.shape[1] // 2
    h = silu_mul(gu[:, :inter], gu[:, inter:], dtype)
    v = gl(h, [(qd[e], sd[e]) for e, _ in order], False, dtype)
    return ordered_reduce(v, [s for _, s in order], np.asarray(weights).reshape(-1), dtype)


def decode_block(x, ids, weights, banks, shared, gate_w, activation='w8a8', dtype='bf16'):
    x = np.asarray(x, dtype=np.float32).reshape(1, -1)
    routed = decode_routed(x, ids, weights, banks, activation, dtype)[None]
    sh = shared_expert(x, shared, dtype)
    return shared_gate_combine(routed, sh, x, gate_w, dtype)


# --------------------------------------------------------------------------
# inputs: seeded synthetic data with the benchmark's distributions
# --------------------------------------------------------------------------
def zipf_bias(experts, rng, exponent=1.1):
    """Per-expert logit bias ``-exponent * ln(rank)`` for ranks 1..E assigned
    by a seeded permutation (multiplies the softmax by Zipf weights)."""
    ranks = rng.permutation(experts) + 1
    return (-exponent * np.log(ranks)).astype(np.float32)


def route(logits, top):
    """HF router tail (hf :762-770): fp32 softmax, top-k, renormalise.
    Ties resolve to the lower expert id."""
    lg = np.asarray(logits, dtype=np.float32)
    p = np.exp(lg - lg.max(-1, keepdims=True))
    p = (p / p.sum(-1, keepdims=True)).astype(np.float32)
    idx = np.argsort(-p, axis=-1, kind='stable')[:, :top]
    val = np.take_along_axis(p, idx, -1)
    val = (val / val.sum(-1, keepdims=True)).astype(np.float32)
    return idx.astype(np.int64), val


def make_layer(rng, experts=256, hidden=2048, inter=512, std=0.02):
    """One layer's expert bank and shared expert, quantised by ``quantize_weight``."""
    qg, sg = quantize_weight(rng.standard_normal((experts, 2 * inter, hidden), dtype=np.float32) * std)
    qd, sd = quantize_weight(rng.standard_normal((experts, hidden, inter), dtype=np.float32) * std)
    shared = []
    for shape in ((inter, hidden), (inter, hidden), (hidden, inter)):
        shared.append(quantize_weight(rng.standard_normal(shape, dtype=np.float32) * std))
    gate_w = to_bf16(rng.standard_normal((1, hidden), dtype=np.float32) * std)
    return (qg, sg, qd, sd), shared, gate_w


def make_tokens(rng, tokens, hidden=2048, experts=256, top=8, zipf=True):
    x = to_bf16(rng.standard_normal((tokens, hidden), dtype=np.float32))
    logits = rng.standard_normal((tokens, experts), dtype=np.float32)
    if zipf:
        logits = logits + zipf_bias(experts, rng)[None]
    ids, w = route(logits, top)
    return x, ids, w
