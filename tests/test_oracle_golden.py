"""Pin the CPU oracle against outputs of the reference's own code
(tests/golden/golden.npz, made by tests/golden/make_golden.py)."""
import os

import numpy as np
import pytest

import inputs as gi
from oracle import oracle as O

GOLD = np.load(os.path.join(os.path.dirname(__file__), 'golden', 'golden.npz'))


def f16(bits):
    return np.asarray(bits, dtype=np.uint16).view(np.float16).astype(np.float32)


def bf16(bits):
    return O.bf16_from_bits(bits)


def test_inputs_reproduce():
    assert np.array_equal(gi.checksums(), GOLD['input_checksums'])


def test_weight_quantiser_known_answer():
    import torch
    w = torch.linspace(-1, 1, 256).reshape(2, 128).bfloat16().float().numpy()
    q, s = O.quantize_weight(w)
    assert np.array_equal(q, GOLD['wq_known_q'])
    assert np.array_equal(s, GOLD['wq_known_s'])


def test_weight_quantiser_random():
    q, s = O.quantize_weight(gi.weight_quant_input())
    assert np.array_equal(q, GOLD['wq_rand_q'])
    assert np.array_equal(s.view(np.uint32), GOLD['wq_rand_s'].view(np.uint32))


def test_activation_quantiser_bit_exact():
    x = bf16(gi.act_quant_input())
    q, s = O.quantize_act(x)
    assert np.array_equal(q, GOLD['aq_q'])
    assert np.array_equal(s.view(np.uint32), GOLD['aq_s'].view(np.uint32))


@pytest.mark.parametrize('tile', ['16x32', '32x64'])
def test_linear_w8a16_fp16(tile):
    x, q, s = gi.linear_inputs()
    y = O.linear_w8a16(x.astype(np.float32), q, s, 'f16')
    ref = f16(GOLD[f'lin_y_{tile}'])
    # tl.dot's fp32 summation order is unspecified: allow one fp16 ulp
    assert np.abs(y - ref).max() <= np.abs(ref).max() * 2 ** -10 * 1.01
    assert (y == ref).mean() > 0.97


def _grouped_weights(g, field):
    if field == 0:
        return [(g['qg'][e], g['sg'][e]) for e in g['experts']]
    return [(g['qd'][e], g['sd'][e]) for e in g['experts']]


def test_grouped_linear_w8a16_fp16():
    g = gi.grouped_inputs()
    gu = O.grouped_linear_w8a16(g['x_shared'].astype(np.float32), _grouped_weights(g, 0), True, 'f16')
    dn = O.grouped_linear_w8a16(g['x_rows'].astype(np.float32), _grouped_weights(g, 2), False, 'f16')
    for y, key in ((gu, 'gl16_gu'), (dn, 'gl16_dn')):
        ref = f16(GOLD[key])
        assert np.abs(y - ref).max() <= np.abs(ref).max() * 2 ** -10 * 1.01


def test_grouped_linear_w8a8_bit_exact():
    g = gi.grouped_inputs()
    xs, xr = bf16(g['x_shared_bf16']), bf16(g['x_rows_bf16'])
    gu = O.grouped_linear_w8a8(xs, _grouped_weights(g, 0), True, 'f16')
    dn = O.grouped_linear_w8a8(xr, _grouped_weights(g, 2), False, 'f16')
    assert np.array_equal(gu, f16(GOLD['gl8_gu']))
    assert np.array_equal(dn, f16(GOLD['gl8_dn']))


def test_ordered_reduce_bit_exact():
    v, slots, w = gi.reduce_inputs()
    y = O.ordered_reduce(v.astype(np.float32), slots, w, 'f16')
    assert np.array_equal(y.astype(np.float16).view(np.uint16), GOLD['ored_y'])


def test_bf16_rounding_matches_torch():
    import torch
    r = np.random.default_rng(5)
    a = np.concatenate([r.standard_normal(100000).astype(np.float32) * 10 ** r.uniform(-30, 30, 100000).astype(np.float32),
                        np.array([0.0, -0.0, 1.00390625, 1.01171875, 3.4e38, -3.4e38, 1e-40, np.inf], dtype=np.float32)])
    a = a.astype(np.float32)
    ref = torch.from_numpy(a).bfloat16().view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(O.bf16_bits(a), ref)


@pytest.mark.parametrize('name', sorted(gi.route_cases()))
def test_route_plans_bit_exact(name):
    ids, experts = gi.route_cases()[name]
    positions, segments = O.plan_routes(ids, experts)
    assert np.array_equal(positions, GOLD[f'{name}_positions'])
    assert np.array_equal(np.asarray(segments, dtype=np.int64).reshape(-1, 3), GOLD[f'{name}_segments'])
    for bm in (16, 32):
        pos, table, ordered, slots = O.plan(ids, experts, bm)
        assert np.array_equal(pos, GOLD[f'{name}_bm{bm}_pos'])
        assert np.array_equal(table, GOLD[f'{name}_bm{bm}_table'])
        assert np.array_equal(ordered, GOLD[f'{name}_bm{bm}_ordered'])
        assert np.array_equal(slots, GOLD[f'{name}_bm{bm}_slots'])


def test_plan_routes_rejects_bad_ids():
    with pytest.raises(ValueError, match='Out-of-range expert ID'):
        O.plan_routes(np.array([[0, 4]]), 4)
    with pytest.raises(ValueError, match='Expected nonempty'):
        O.plan_routes(np.zeros((0, 8), dtype=np.int64), 4)


def test_routed_moe_fp16():
    r = gi.routed_inputs()
    banks = (r['qg'], r['sg'], r['qd'], r['sd'])
    out, parts = O.routed_moe(r['x'].astype(np.float32), r['weights'], r['ids'], banks, 'f16', True)
    gu_ref = f16(GOLD['rmoe_gu'])
    assert np.abs(parts['gu'] - gu_ref).max() <= np.abs(gu_ref).max() * 2 ** -10 * 1.01
    for key in ('rmoe_cpuplan', 'rmoe_cpuplan_large', 'rmoe_gpuplan'):
        ref = f16(GOLD[key])
        err = np.abs(out - ref).max() / np.abs(ref).max()
        assert err < 4e-3, (key, err)
    # both reference plan variants are the same arithmetic
    assert np.array_equal(GOLD['rmoe_cpuplan'], GOLD['rmoe_gpuplan'])
