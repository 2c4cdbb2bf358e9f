"""The oracle's sparse-MoE block pinned against the HF module it restates.

The reference keeps transformers' ``Qwen3_5MoeSparseMoeBlock`` around its INT8
operators (qwen35_deploy/model.py:57-68): the router's fp32 softmax / top-k /
renormalise, the experts' ``index_add_`` in ascending expert order, the shared
expert, its sigmoid gate and the final add (modeling_qwen3_5_moe.py:698-792).
Here the installed transformers (5.5.0; the reference pins 5.15.0) runs that
block in bf16 on the CPU with every weight set to round_bf16(q * s), the weight
the reference's Int8Linear / Int8Experts multiply with (int8.py:19-21), and the
oracle must agree: the same expert sets with the same weights, and the block
within the 1e-2 bar with most elements bit-equal (the freedom left is the fp32
summation order inside each bf16 matmul, which the oracle sums exactly).
"""
import numpy as np
import pytest
import torch

from helpers import rel_maxabs
from oracle import oracle as O

E, H, I, TOP, T = 16, 256, 128, 4, 24


def _bf16(a):
    return torch.from_numpy(np.ascontiguousarray(a, dtype=np.float32)).to(torch.bfloat16)


@pytest.fixture(scope='module')
def case():
    hf = pytest.importorskip('transformers.models.qwen3_5_moe.modeling_qwen3_5_moe')
    cfg_mod = pytest.importorskip('transformers.models.qwen3_5_moe.configuration_qwen3_5_moe')
    r = np.random.default_rng(2024)
    qg, sg = O.quantize_weight(r.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.02)
    qd, sd = O.quantize_weight(r.standard_normal((E, H, I)).astype(np.float32) * 0.02)
    shared = [O.quantize_weight(r.standard_normal(s).astype(np.float32) * 0.02) for s in ((I, H), (I, H), (H, I))]
    gate_w = O.round_to(r.standard_normal((1, H)).astype(np.float32) * 0.02, 'bf16')
    router = O.round_to(r.standard_normal((E, H)).astype(np.float32) * 0.05, 'bf16')
    x = O.round_to(r.standard_normal((T, H)).astype(np.float32), 'bf16')
    cfg = cfg_mod.Qwen3_5MoeTextConfig(hidden_size=H, num_experts=E, num_experts_per_tok=TOP,
                                       moe_intermediate_size=I, shared_expert_intermediate_size=I,
                                       hidden_act='silu')
    cfg._experts_implementation = 'eager'
    blk = hf.Qwen3_5MoeSparseMoeBlock(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        blk.gate.weight.copy_(_bf16(router))
        blk.experts.gate_up_proj.copy_(_bf16(O.dequant(qg, sg, 'bf16')))
        blk.experts.down_proj.copy_(_bf16(O.dequant(qd, sd, 'bf16')))
        for lin, (q, s) in zip((blk.shared_expert.gate_proj, blk.shared_expert.up_proj, blk.shared_expert.down_proj),
                               shared):
            lin.weight.copy_(_bf16(O.dequant(q, s, 'bf16')))
        blk.shared_expert_gate.weight.copy_(_bf16(gate_w))
        xt = _bf16(x)
        _, hf_w, hf_ids = blk.gate(xt)
        y = blk(xt.reshape(1, T, H)).reshape(T, H)
        logits = torch.nn.functional.linear(xt, blk.gate.weight)
    return dict(x=x, banks=(qg, sg, qd, sd), shared=shared, gate_w=gate_w, logits=logits.float().numpy(),
                hf_w=hf_w.float().numpy(), hf_ids=hf_ids.numpy(), y=y.float().numpy())


def test_router_tail_matches_hf(case):
    ids, w = O.route(case['logits'], TOP)
    o_hf = np.argsort(case['hf_ids'], -1)
    o_or = np.argsort(ids, -1)
    assert np.array_equal(np.take_along_axis(ids, o_or, -1), np.take_along_axis(case['hf_ids'], o_hf, -1))
    got = np.take_along_axis(w, o_or, -1)
    want = np.take_along_axis(case['hf_w'], o_hf, -1)
    assert np.abs(got - want).max() / np.abs(want).max() < 1e-5


def test_block_matches_hf(case):
    """The oracle's block on HF's own routing: routed experts summed in ascending
    expert order with a bf16 rounding per add, the gated shared expert, the add."""
    ref = O.moe_block(case['x'], case['hf_w'], case['hf_ids'], case['banks'], case['shared'], case['gate_w'], 'bf16')
    assert rel_maxabs(case['y'], ref) < 1e-2
    assert (case['y'] == ref).mean() > 0.9
