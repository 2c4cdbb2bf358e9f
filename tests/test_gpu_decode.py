"""GPU parity of the one-token decode chain (lmoe_decode_moe) against the
oracle's restatement of the reference decode branch (int8.py:158-187 with
w8a8.grouped_linear installed by cli.py:37-39, or int8.grouped_linear) plus
the HF shared expert and gate.

Tolerance: 1e-2 max-abs-normalised against the oracle;
the W8A8 routed GEMVs are exact integer dots, so the remaining differences
come from the W8A16 shared-expert sums and fp32 exp in silu/sigmoid.
"""
import numpy as np
import pytest
import torch

from helpers import BF16, F16, act, rand_q, rel_maxabs, rng, to_dev, to_np
from oracle import oracle as O

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module', autouse=True)
def _cuda():
    if not torch.cuda.is_available():
        pytest.skip('needs a CUDA device')
    from localmoe35ba3b_b200 import _native
    _native.lib()
    yield
    torch.cuda.synchronize()
    _native.check_device_errors()


def _case(seed, E, H, I, top, dtype):
    r = rng(seed)
    logits = r.standard_normal((1, E), dtype=np.float32) + O.zipf_bias(E, r)[None]
    ids, w = O.route(logits, top)
    qg, sg = rand_q(r, (E, 2 * I, H))
    qd, sd = rand_q(r, (E, H, I))
    shared = [rand_q(r, (I, H)), rand_q(r, (I, H)), rand_q(r, (H, I))]
    gate_w = act(r, (1, H), dtype, 0.02)
    x = act(r, (1, H), dtype)
    res = act(r, (1, H), dtype)
    return x, ids, w, (qg, sg, qd, sd), shared, gate_w, res


def _dev(case, dtype):
    x, ids, w, bank, shared, gate_w, res = case
    return (to_dev(x, dtype), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda(),
            [torch.from_numpy(b).cuda() for b in bank],
            [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for q, s in shared], to_dev(gate_w, dtype),
            to_dev(res, dtype))


@pytest.mark.parametrize('dtype', [BF16, F16])
@pytest.mark.parametrize('activation', ['w8a8', 'w8a16'])
@pytest.mark.parametrize('E,H,I,top', [(256, 2048, 512, 8), (16, 384, 256, 4)])
def test_decode_block_vs_oracle(dtype, activation, E, H, I, top):
    from localmoe35ba3b_b200.runtime import decode
    case = _case(31 + E, E, H, I, top, dtype)
    x, ids, w, bank, shared, gate_w, res = case
    xd, idd, wd, bd, shd, gd, rd = _dev(case, dtype)
    out = decode.decode_block(xd, wd, idd, bd, shared=shd, shared_gate_weight=gd, residual=rd, activation=activation)
    torch.cuda.synchronize()
    blk = O.decode_block(x, ids, w, bank, shared, gate_w, activation, dtype)
    ref = O.round_to(res + blk, dtype)
    assert rel_maxabs(to_np(out), ref) < 1e-2
    assert (to_np(out) == ref).mean() > 0.5


@pytest.mark.parametrize('activation', ['w8a8', 'w8a16'])
def test_decode_routed_exact_order(activation):
    """Routed part only: ids given out of order and with the expert ids' slots
    shuffled; the table must follow ascending expert ids (int8.py:170-179)."""
    from localmoe35ba3b_b200.operators.int8 import Int8Experts
    E, H, I, top = 64, 512, 256, 8
    case = _case(77, E, H, I, top, BF16)
    x, ids, w, bank, _, _, _ = case
    ids = ids[:, ::-1].copy()
    w = w[:, ::-1].copy()
    xd, idd, wd = to_dev(x, BF16), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda()
    bd = [torch.from_numpy(b).cuda() for b in bank]
    mod = Int8Experts(*bd, activation=activation)
    out = mod(xd, idd, wd)
    torch.cuda.synchronize()
    ref = O.decode_routed(x, ids, w, bank, activation, BF16)
    assert rel_maxabs(to_np(out).reshape(-1), ref.reshape(-1)) < 1e-2
    if activation == 'w8a8':
        # exact integer GEMV dots, exact ordered combine: only silu may differ
        assert (to_np(out).reshape(-1) == ref.reshape(-1)).mean() > 0.9


def test_int8_experts_prefill_matches_routed_moe():
    from localmoe35ba3b_b200.operators.int8 import Int8Experts
    r = rng(5)
    T, E, H, I, top = 40, 32, 512, 256, 8
    logits = r.standard_normal((T, E), dtype=np.float32)
    ids, w = O.route(logits, top)
    qg, sg = rand_q(r, (E, 2 * I, H))
    qd, sd = rand_q(r, (E, H, I))
    x = act(r, (T, H), BF16)
    mod = Int8Experts(*[torch.from_numpy(b).cuda() for b in (qg, sg, qd, sd)])
    out = mod(to_dev(x, BF16), torch.from_numpy(ids).cuda(), torch.from_numpy(w).cuda())
    torch.cuda.synchronize()
    ref = O.routed_moe(x, w, ids, (qg, sg, qd, sd), BF16)
    assert rel_maxabs(to_np(out), ref) < 1e-2


def test_decode_graph_capture_replays_identically():
    """The chain has no host synchronisation: a captured graph replays to the
    eager result bit for bit, with new router inputs copied into the static
    buffers between replays."""
    from localmoe35ba3b_b200.runtime import decode
    E, H, I, top = 256, 2048, 512, 8
    case = _case(91, E, H, I, top, BF16)
    xd, idd, wd, bd, shd, gd, rd = _dev(case, BF16)
    eager = decode.decode_block(xd, wd, idd, bd, shared=shd, shared_gate_weight=gd, residual=rd).clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        decode.decode_block(xd, wd, idd, bd, shared=shd, shared_gate_weight=gd, residual=rd)  # warm the workspace
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        out = decode.decode_block(xd, wd, idd, bd, shared=shd, shared_gate_weight=gd, residual=rd)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize()
    assert torch.equal(out, eager)
    # a different routing row through the same graph
    case2 = _case(92, E, H, I, top, BF16)
    idd.copy_(torch.from_numpy(case2[1]).cuda())
    wd.copy_(torch.from_numpy(case2[2]).cuda())
    g.replay()
    torch.cuda.synchronize()
    ref2 = decode.decode_block(xd, wd, idd, bd, shared=shd, shared_gate_weight=gd, residual=rd)
    torch.cuda.synchronize()
    assert torch.equal(out, ref2)
    del g


def test_decode_layer_graph_capture():
    """A whole one-token layer in one CUDA graph: a dense Int8Linear (an o_proj of
    [H, H]), the router's bf16 logits and its softmax / top-k / renormalise, and the
    MoE block with its gated shared expert and the residual -- no host
    synchronisation anywhere (the reference syncs per layer, int8.py:160).  For two
    token rows copied into the static input, every stage of a replay equals the
    eager library call on the graph's own input to that stage, bit for bit (the
    logits are cuBLAS's and are checked only through the stages that read them), and
    the layer matches the oracle on the graph's routing."""
    from localmoe35ba3b_b200.operators import int8
    from localmoe35ba3b_b200.runtime import block, decode
    E, H, I, top = 256, 2048, 512, 8
    case = _case(93, E, H, I, top, BF16)
    _, _, _, bank, shared, gate_w, _ = case
    xd, _, _, bd, shd, gd, _ = _dev(case, BF16)
    r = rng(94)
    qo_np, so_np = rand_q(r, (H, H))
    qo, so = torch.from_numpy(qo_np).cuda(), torch.from_numpy(so_np).cuda()
    router = to_dev(act(r, (E, H), BF16, 0.02), BF16)
    x = xd.clone()  # the graph's static input row

    def layer():
        h = int8.linear(x, qo, so)
        logits = torch.nn.functional.linear(h, router)
        w, ids = block.topk_from_logits(logits, top)
        y = decode.decode_block(h, w, ids, bd, shared=shd, shared_gate_weight=gd, residual=x)
        return h, logits, w, ids, y

    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        layer()  # warm the workspaces and the library handles outside the capture
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        h, logits, w, ids, y = layer()
    for seed in (95, 96):
        x_np = act(rng(seed), (1, H), BF16)
        x.copy_(to_dev(x_np, BF16))
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(h, int8.linear(x, qo, so))
        w2, ids2 = block.topk_from_logits(logits, top)
        assert torch.equal(w, w2) and torch.equal(ids, ids2)
        y2 = decode.decode_block(h, w, ids, bd, shared=shd, shared_gate_weight=gd, residual=x)
        torch.cuda.synchronize()
        assert torch.equal(y, y2)
        h_np = to_np(h)
        assert rel_maxabs(h_np, O.linear_w8a16(x_np, qo_np, so_np, BF16)) < 1e-2
        blk = O.decode_block(h_np, ids.cpu().numpy(), w.cpu().numpy(), bank, shared, gate_w, 'w8a8', BF16)
        assert rel_maxabs(to_np(y), O.round_to(x_np + blk, BF16)) < 1e-2
    del g


def test_decode_bad_expert_id_sets_error_bit():
    """An id outside [0, E) is caught by the table kernel's own bounds check:
    it raises the device error bit and reads expert 0 instead."""
    from localmoe35ba3b_b200 import _native as N
    from localmoe35ba3b_b200.runtime import decode
    E, H, I, top = 16, 384, 256, 4
    case = _case(13, E, H, I, top, BF16)
    xd, idd, wd, bd, _, _, _ = _dev(case, BF16)
    idd[0, 1] = E + 3
    out = decode.decode_block(xd, wd, idd, bd)
    torch.cuda.synchronize()
    assert torch.isfinite(out.float()).all()
    with pytest.raises(N.NativeError, match='0x2'):
        N.check_device_errors()
