"""``runtime.install.install(model)`` on a model shaped like the reference's loaded
model (qwen35_deploy/model.py:61-70): HF sparse-MoE blocks whose experts hold the
converted banks as ``gate_up`` / ``down`` dicts (the reference's ``Int8Experts``)
and whose shared-expert linears, like the attention projections, hold int8 ``q``
and fp32 ``scale`` buffers (the reference's ``Int8Linear``).  CPU only: the
replacement is module surgery; the replaced modules' kernels are tested on GPUs."""
import numpy as np
import pytest
import torch

from oracle import oracle as O

E, H, I, TOP = 8, 256, 128, 2


class RefInt8Linear(torch.nn.Module):
    """The reference Int8Linear's state (int8.py:40-48)."""

    def __init__(self, q, scale):
        super().__init__()
        self.register_buffer('q', q)
        self.register_buffer('scale', scale)


class RefInt8Experts(torch.nn.Module):
    """The reference Int8Experts' bank attributes (int8.py:127-130)."""

    def __init__(self, gate_up, down):
        super().__init__()
        self.gate_up, self.down = gate_up, down


def _quant(r, shape):
    q, s = O.quantize_weight(r.standard_normal(shape).astype(np.float32) * 0.02)
    return torch.from_numpy(q), torch.from_numpy(s)


def _model(r, layers=2, float_experts=False, experts=E):
    hf = pytest.importorskip('transformers.models.qwen3_5_moe.modeling_qwen3_5_moe')
    cfg_mod = pytest.importorskip('transformers.models.qwen3_5_moe.configuration_qwen3_5_moe')
    cfg = cfg_mod.Qwen3_5MoeTextConfig(hidden_size=H, num_experts=experts, num_experts_per_tok=TOP,
                                       moe_intermediate_size=I, shared_expert_intermediate_size=I,
                                       hidden_act='silu')
    cfg._experts_implementation = 'eager'
    model = torch.nn.Module()
    model.layers = torch.nn.ModuleList()
    for _ in range(layers):
        layer = torch.nn.Module()
        layer.self_attn = torch.nn.Module()
        layer.self_attn.o_proj = RefInt8Linear(*_quant(r, (H, 2 * H)))
        mlp = hf.Qwen3_5MoeSparseMoeBlock(cfg).to(torch.bfloat16)
        if not float_experts:
            gq, gs = _quant(r, (experts, 2 * I, H))
            dq, ds = _quant(r, (experts, H, I))
            mlp.experts = RefInt8Experts({'q': gq, 'scale': gs}, {'q': dq, 'scale': ds})
        for p in ('gate_proj', 'up_proj', 'down_proj'):
            setattr(mlp.shared_expert, p, RefInt8Linear(*_quant(r, (I, H) if p != 'down_proj' else (H, I))))
        layer.mlp = mlp
        model.layers.append(layer)
    return model


def test_install_replaces_blocks_and_linears():
    from localmoe35ba3b_b200.operators.int8 import Int8Linear
    from localmoe35ba3b_b200.runtime.block import SparseMoeBlock
    from localmoe35ba3b_b200.runtime.install import install
    model = _model(np.random.default_rng(7))
    old = [(l.mlp, l.self_attn.o_proj) for l in model.layers]
    assert install(model, device='cpu') == {'blocks': 2, 'linears': 2}
    for layer, (mlp, o_proj) in zip(model.layers, old):
        blk = layer.mlp
        assert isinstance(blk, SparseMoeBlock) and blk.activation == 'w8a8' and blk.gate.top_k == TOP
        for got, want in zip(blk.banks, [mlp.experts.gate_up['q'], mlp.experts.gate_up['scale'],
                                         mlp.experts.down['q'], mlp.experts.down['scale']]):
            assert torch.equal(got, want)
        for (q, s), p in zip(blk.shared, ('gate_proj', 'up_proj', 'down_proj')):
            ref = getattr(mlp.shared_expert, p)
            assert torch.equal(q, ref.q) and torch.equal(s, ref.scale)
        assert torch.equal(blk.gate.weight, mlp.gate.weight)
        assert torch.equal(blk.shared_gate_weight, mlp.shared_expert_gate.weight.reshape(1, -1))
        assert isinstance(layer.self_attn.o_proj, Int8Linear)
        assert torch.equal(layer.self_attn.o_proj.q, o_proj.q)
    # a second install finds nothing left to replace
    assert install(model, device='cpu') == {'blocks': 0, 'linears': 0}


def test_install_refuses_float_experts_and_bad_arguments():
    from localmoe35ba3b_b200.runtime.install import install
    with pytest.raises(ValueError, match='no INT8 group-128 banks'):
        install(_model(np.random.default_rng(8), layers=1, float_experts=True), device='cpu')
    with pytest.raises(ValueError, match='activation'):
        install(torch.nn.Module(), activation='fp8')
    with pytest.raises(ValueError, match='pass the model'):
        install(RefInt8Linear(*_quant(np.random.default_rng(9), (128, 256))))


@pytest.mark.gpu
@pytest.mark.parametrize('T', [1, 37])
def test_installed_model_forward_matches_oracle(T):
    """After install(model) on cuda, each layer's replaced modules run the B200 kernels:
    the o_proj Int8Linear against the oracle's W8A16 linear, and the sparse-MoE block
    (router on the GPU, then the prefill block or, for one token, the W8A8 decode chain)
    against the oracle block on the same routing.  32 experts: the smallest count the
    device router takes."""
    import torch.nn.functional as F
    from localmoe35ba3b_b200.runtime.install import install
    r = np.random.default_rng(31 + T)
    model = _model(r, experts=32)
    truth = []
    for layer in model.layers:
        m = layer.mlp
        truth.append(((m.experts.gate_up['q'].numpy(), m.experts.gate_up['scale'].numpy(),
                       m.experts.down['q'].numpy(), m.experts.down['scale'].numpy()),
                      [(getattr(m.shared_expert, p).q.numpy(), getattr(m.shared_expert, p).scale.numpy())
                       for p in ('gate_proj', 'up_proj', 'down_proj')],
                      m.shared_expert_gate.weight.detach().float().numpy().reshape(1, -1),
                      (layer.self_attn.o_proj.q.numpy(), layer.self_attn.o_proj.scale.numpy())))
    activation = 'w8a8' if T == 1 else 'w8a16'
    assert install(model, activation=activation, device='cuda') == {'blocks': 2, 'linears': 2}
    x = O.to_bf16(r.standard_normal((T, H), dtype=np.float32))
    x2 = O.to_bf16(r.standard_normal((T, 2 * H), dtype=np.float32))
    for layer, (bank, shared, gate_w, (oq, os_)) in zip(model.layers, truth):
        xd = torch.from_numpy(x).to(torch.bfloat16).cuda()
        out = layer.mlp(xd.reshape(1, T, H))
        y = layer.self_attn.o_proj(torch.from_numpy(x2).to(torch.bfloat16).cuda())
        torch.cuda.synchronize()
        logits = F.linear(xd, layer.mlp.gate.weight).float().cpu().numpy()
        ids, w = O.route(logits, TOP)
        if T == 1:
            ref = O.decode_block(x, ids, w, bank, shared, O.to_bf16(gate_w), activation, 'bf16')
        else:
            ref = O.moe_block(x, w, ids, bank, shared, O.to_bf16(gate_w), 'bf16')
        got = out.float().cpu().numpy().reshape(T, H)
        assert np.abs(got - ref).max() / np.abs(ref).max() < 1e-2
        ref_y = O.linear_w8a16(x2, oq, os_, 'bf16')
        got_y = y.float().cpu().numpy()
        assert np.abs(got_y - ref_y).max() / np.abs(ref_y).max() < 1e-2
