"""Expert-parallel layer on the GPU kernels (lmoe_ep_dispatch, lmoe_ep_owner,
lmoe_ep_fold): W ranks emulated on one GPU (the exchanges as segment copies),
one process over NCCL, and two processes on two GPUs when present; plus the
block's no-route slots and its shared-only form."""
import os
import socket

import numpy as np
import pytest
import torch

from helpers import BF16, act, rand_q, rel_maxabs, rng, to_dev, to_np
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


def _case(T=96, E=32, H=512, I=256, top=8):
    r = rng(44)
    logits = r.standard_normal((T, E), dtype=np.float32) + O.zipf_bias(E, r)[None]
    ids, w = O.route(logits, top)
    bank = (*rand_q(r, (E, 2 * I, H)), *rand_q(r, (E, H, I)))
    shared = [rand_q(r, (I, H)), rand_q(r, (I, H)), rand_q(r, (H, I))]
    gate = act(r, (1, H), BF16, 0.02)
    x = act(r, (T, H), BF16)
    res = act(r, (T, H), BF16)
    return x, ids, w, bank, shared, gate, res


def test_shared_only_block_matches_oracle():
    from localmoe35ba3b_b200.runtime import gpu_routes
    x, ids, w, bank, shared, gate, res = _case()
    bd = [torch.from_numpy(b).cuda() for b in bank]
    sh = [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for q, s in shared]
    t = x.shape[0]
    out = gpu_routes.moe_block(to_dev(x, BF16), torch.empty((t, 0), device='cuda'),
                               torch.empty((t, 0), dtype=torch.int64, device='cuda'), bd, shared=sh,
                               shared_gate_weight=to_dev(gate, BF16), residual=to_dev(res, BF16))
    torch.cuda.synchronize()
    sg = O.shared_gate_combine(np.zeros_like(x), O.shared_expert(x, shared, BF16), x, gate, BF16)
    ref = O.round_to(res + sg, BF16)
    assert rel_maxabs(to_np(out), ref) < 1e-2


def _wire_ref(x, ids, w, bank, shared, gate, res, wire):
    """The block with the routed experts reading the dispatched rows: x itself on
    the bf16 wire, round_bf16(q * s) of its W8A8 quantisation on the int8 wire."""
    xr = x if wire == 'bf16' else O.round_to(O.dequant(*O.quantize_act(x)), BF16)
    routed = O.routed_moe(xr, w, ids, bank, BF16)
    return O.round_to(res + O.shared_gate_combine(routed, O.shared_expert(x, shared, BF16), x, gate, BF16), BF16)


def _round_add(a, b):
    return (a.float() + b.float()).to(a.dtype)


def _ep_sequence_gpu(x, w, ids, bank, shared, gate, res, world, wire):
    """The expert-parallel rounding sequence from single-GPU library calls: per rank
    g, the block on the token's routes to g's experts only (the others -1), whose
    ordered combine is that rank's pre-reduced partial; the partials folded in
    ascending rank order for the tokens that have a route there; then the gated
    shared expert (the block with top 0) and the residual."""
    from localmoe35ba3b_b200.operators import w8a8
    from localmoe35ba3b_b200.runtime import gpu_routes
    e_loc = bank[0].shape[0] // world
    xr = x
    if wire == 'int8':
        q, s = w8a8.quantize(x)
        xr = (q.float() * s.repeat_interleave(128, -1)).to(x.dtype)
    acc = torch.zeros_like(x)
    for g in range(world):
        mine = torch.div(ids, e_loc, rounding_mode='floor') == g
        part = gpu_routes.moe_block(xr, torch.where(mine, w, torch.zeros_like(w)),
                                    torch.where(mine, ids, torch.full_like(ids, -1)), bank)
        has = mine.any(1)
        acc[has] = _round_add(acc[has], part[has])
    t = x.shape[0]
    sh = gpu_routes.moe_block(x, torch.empty((t, 0), device=x.device), torch.empty((t, 0), dtype=torch.int64,
                                                                                  device=x.device),
                              bank, shared=shared, shared_gate_weight=gate)
    return _round_add(res, _round_add(acc, sh))


def _emulate_ranks(x, w, ids, bank, shared, gate, res, world, wire):
    """The GPU expert-parallel layer of `world` ranks run one after another on one
    GPU: rank r owns tokens [r*T/world, (r+1)*T/world) and experts [r*E/world, ...);
    the two all-to-all exchanges are segment copies between the ranks' buffers."""
    from localmoe35ba3b_b200.runtime import ep
    T, H = x.shape
    E, I = bank[0].shape[0], bank[2].shape[2]
    tr, e_loc = T // world, E // world
    L = [ep.GpuLayer(tr, ids.shape[1], E, world, H, I, x.dtype, x.device, wire, transport='nccl')
         for _ in range(world)]
    sl = [slice(r * tr, (r + 1) * tr) for r in range(world)]
    for r in range(world):
        L[r].dispatch(x[sl[r]].contiguous(), w[sl[r]].contiguous(), ids[sl[r]].contiguous())
    seg = (L[0].cap + 1) * L[0].row_bytes
    recv = [torch.empty_like(l.send) for l in L]
    for d in range(world):
        for s in range(world):
            recv[d][s * seg:(s + 1) * seg] = L[s].send[d * seg:(d + 1) * seg]
    for d in range(world):
        L[d].recv = recv[d]
        L[d].owner(x[sl[d]].contiguous(), [b[d * e_loc:(d + 1) * e_loc].contiguous() for b in bank], shared)
    cap = L[0].cap
    back = [torch.empty_like(l.partial) for l in L]
    for s in range(world):
        for d in range(world):
            back[s][d * cap:(d + 1) * cap] = L[d].partial[s * cap:(s + 1) * cap]
    outs = []
    for s in range(world):
        L[s].back = back[s]
        outs.append(L[s].fold(x[sl[s]].contiguous(), gate, res[sl[s]].contiguous()))
    return torch.cat(outs)


@pytest.mark.parametrize('world', [1, 2, 4, 8])
@pytest.mark.parametrize('wire', ['bf16', 'int8'])
def test_expert_parallel_layer_emulated_ranks(world, wire):
    """All W ranks of the GPU expert-parallel layer (dispatch, owner, fold kernels)
    on one GPU: bit-exact against the EP rounding sequence built from the
    single-GPU block, and within 1e-2 of the oracle."""
    from localmoe35ba3b_b200 import _native
    x, ids, w, bank, shared, gate, res = _case(T=192)
    bd = [torch.from_numpy(b).cuda() for b in bank]
    sh = [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for q, s in shared]
    xd, rd, gd = to_dev(x, BF16), to_dev(res, BF16), to_dev(gate, BF16)
    wd, idd = torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda()
    got = _emulate_ranks(xd, wd, idd, bd, sh, gd, rd, world, wire)
    want = _ep_sequence_gpu(xd, wd, idd, bd, sh, gd, rd, world, wire)
    torch.cuda.synchronize()
    _native.check_device_errors()
    assert torch.equal(got.float(), want.float())
    assert rel_maxabs(to_np(got), _wire_ref(x, ids, w, bank, shared, gate, res, wire)) < 1e-2


@pytest.mark.parametrize('transport', ['nccl', 'p2p'])
def test_expert_parallel_layer_world1_equals_block(transport):
    """At world 1 (one process) the layer's sequence is the block's own: the result
    equals gpu_routes.moe_block bit for bit, with either transport (the direct one
    stores to and waits on this rank's own buffers and flags), over several layers
    (the flag epochs advance)."""
    import torch.distributed as dist
    from localmoe35ba3b_b200.runtime import ep, gpu_routes
    x, ids, w, bank, shared, gate, res = _case()
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('nccl', rank=0, world_size=1)
    try:
        bd = [torch.from_numpy(b).cuda() for b in bank]
        sh = [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for q, s in shared]
        xd, wd, idd, gd, rd = (to_dev(x, BF16), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(),
                               to_dev(gate, BF16), to_dev(res, BF16))
        outs = [ep.moe_forward_gpu(xd, wd, idd, bank[0].shape[0], bd, sh, gd, residual=rd, transport=transport)
                for _ in range(3)]
        blk = gpu_routes.moe_block(xd, wd, idd, bd, shared=sh, shared_gate_weight=gd, residual=rd)
        torch.cuda.synchronize()
        from localmoe35ba3b_b200 import _native
        _native.check_device_errors()
    finally:
        ep._layers.clear()
        dist.destroy_process_group()
    for out in outs:
        assert torch.equal(out.float(), blk.float())


def _ep2_worker(rank, wire, transport, port, out_dir):
    import torch.distributed as dist
    from localmoe35ba3b_b200.runtime import ep
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    torch.cuda.set_device(rank)
    dist.init_process_group('nccl', rank=rank, world_size=2)
    try:
        x, ids, w, bank, shared, gate, res = _case()
        t = x.shape[0] // 2
        sl = slice(rank * t, (rank + 1) * t)  # each rank owns half of the tokens
        e_loc = bank[0].shape[0] // 2
        lb = [torch.from_numpy(b[rank * e_loc:(rank + 1) * e_loc]).cuda() for b in bank]
        sh = [(torch.from_numpy(q).cuda(), torch.from_numpy(s).cuda()) for q, s in shared]
        # three layers in a row (the direct transport's flag epochs advance, its buffers are reused)
        for _ in range(3):
            out = ep.moe_forward_gpu(to_dev(x[sl], BF16), torch.from_numpy(w[sl]).cuda(),
                                     torch.from_numpy(ids[sl]).cuda(), bank[0].shape[0], lb, sh, to_dev(gate, BF16),
                                     residual=to_dev(res[sl], BF16), wire=wire, transport=transport)
        torch.cuda.synchronize()
        from localmoe35ba3b_b200 import _native
        _native.check_device_errors()
        for layer in ep._layers.values():
            layer.close()
        ep._layers.clear()
        np.save(os.path.join(out_dir, f'ep2_{rank}.npy'), to_np(out))
        if rank == 0:
            bd = [torch.from_numpy(b).cuda() for b in bank]
            seq = _ep_sequence_gpu(to_dev(x, BF16), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(), bd,
                                   sh, to_dev(gate, BF16), to_dev(res, BF16), 2, wire)
            np.save(os.path.join(out_dir, 'ep2_seq.npy'), to_np(seq))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs 2 GPUs')
@pytest.mark.parametrize('transport', ['p2p', 'nccl'])
@pytest.mark.parametrize('wire', ['bf16', 'int8'])
def test_expert_parallel_two_gpus_matches_oracle(tmp_path, wire, transport):
    """Two processes, one GPU each, direct NVLink stores or NCCL exchanges: bit-exact
    against the EP sequence built from single-GPU block calls, and within 1e-2 of the
    oracle."""
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_ep2_worker, args=(wire, transport, port, str(tmp_path)), nprocs=2, join=True,
                       start_method='spawn')
    x, ids, w, bank, shared, gate, res = _case()
    ref = _wire_ref(x, ids, w, bank, shared, gate, res, wire)
    got = np.concatenate([np.load(tmp_path / f'ep2_{r}.npy') for r in range(2)])
    assert np.array_equal(got, np.load(tmp_path / 'ep2_seq.npy'))
    assert rel_maxabs(got, ref) < 1e-2


def test_block_skips_no_route_slots():
    """A -1 route id is a padded slot (an expert-parallel owner's received row lists
    only its own experts): it gets no GEMM tile and the ordered combine skips it.  The
    result equals, bit for bit, the block with each -1 slot replaced by a real expert
    at weight 0 (whose route adds round(v * 0) = 0, leaving every bf16 sum unchanged);
    no error bit is set; and it matches the oracle over the valid routes."""
    from localmoe35ba3b_b200 import _native
    from localmoe35ba3b_b200.runtime import gpu_routes
    x, ids, w, bank, shared, gate, res = _case(T=150)
    r = rng(45)
    ids = ids.copy()
    w = w.copy()
    drop = r.random(ids.shape) < 0.55
    drop[7] = True          # a row with no route at all
    ids[drop] = -1
    w[drop] = 0.0
    bd = [torch.from_numpy(b).cuda() for b in bank]
    _native.check_device_errors()
    got = gpu_routes.moe_block(to_dev(x, BF16), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(), bd)
    filled = np.where(drop, (np.arange(ids.shape[1])[None, :] * 5 + 3) % bank[0].shape[0], ids)
    same = gpu_routes.moe_block(to_dev(x, BF16), torch.from_numpy(w).cuda(), torch.from_numpy(filled).cuda(), bd)
    torch.cuda.synchronize()
    assert int(_native.error_word('cuda').item()) == 0
    assert torch.equal(got.view(torch.int16), same.view(torch.int16))
    got = to_np(got)
    assert np.all(got[7] == 0)
    ref = np.zeros_like(got)
    for t in range(x.shape[0]):
        keep = ~drop[t]
        if keep.any():
            ref[t] = O.routed_moe(x[t:t + 1], w[t:t + 1, keep], ids[t:t + 1, keep], bank, BF16)[0]
    assert rel_maxabs(got, ref) < 1e-2
