"""Expert-parallel path on the GPU kernels, one process (world size 1 over NCCL):
route rows through gpu_routes.moe_block with one route per row, the shared
expert through the same library call with no routed experts (top 0)."""
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


@pytest.mark.parametrize('wire', ['bf16', 'int8'])
def test_expert_parallel_world1_matches_oracle(wire):
    import torch.distributed as dist
    from localmoe35ba3b_b200.runtime import ep
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
        out = ep.moe_forward(to_dev(x, BF16), torch.from_numpy(w).cuda(), torch.from_numpy(ids).cuda(), bank[0].shape[0],
                             ep.gpu_local_moe(bd), ep.gpu_shared_part(bd, sh, to_dev(gate, BF16)),
                             residual=to_dev(res, BF16), wire=wire)
        torch.cuda.synchronize()
    finally:
        dist.destroy_process_group()
    assert rel_maxabs(to_np(out), _wire_ref(x, ids, w, bank, shared, gate, res, wire)) < 1e-2


def _ep2_worker(rank, wire, port, out_dir):
    import torch.distributed as dist
    from localmoe35ba3b_b200.runtime import ep, gpu_routes
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
        out = ep.moe_forward(to_dev(x[sl], BF16), torch.from_numpy(w[sl]).cuda(), torch.from_numpy(ids[sl]).cuda(),
                             bank[0].shape[0], ep.gpu_local_moe(lb), ep.gpu_shared_part(lb, sh, to_dev(gate, BF16)),
                             residual=to_dev(res[sl], BF16), wire=wire)
        torch.cuda.synchronize()
        np.save(os.path.join(out_dir, f'ep2_{rank}.npy'), to_np(out))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason='needs 2 GPUs')
@pytest.mark.parametrize('wire', ['bf16', 'int8'])
def test_expert_parallel_two_gpus_matches_oracle(tmp_path, wire):
    import torch.multiprocessing as mp
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    port = s.getsockname()[1]
    s.close()
    mp.start_processes(_ep2_worker, args=(wire, port, str(tmp_path)), nprocs=2, join=True, start_method='spawn')
    x, ids, w, bank, shared, gate, res = _case()
    ref = _wire_ref(x, ids, w, bank, shared, gate, res, wire)
    got = np.concatenate([np.load(tmp_path / f'ep2_{r}.npy') for r in range(2)])
    assert rel_maxabs(got, ref) < 1e-2


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float16])
@pytest.mark.parametrize('wire', ['bf16', 'int8'])
def test_pack_and_unpack_kernels_match_torch_packing(wire, dtype):
    """lmoe_ep_pack_rows == the torch byte packing of the gathered rows (with the
    library's W8A8 quantiser on the int8 wire), byte for byte; lmoe_ep_unpack_rows ==
    the torch unpacking gathered per route, bit for bit."""
    from localmoe35ba3b_b200.operators.w8a8 import quantize
    from localmoe35ba3b_b200.runtime import ep
    g = torch.Generator(device='cpu').manual_seed(9)
    T, H, top, n = 40, 1024, 8, 77
    x = (torch.randn((T, H), generator=g) * 3).to(dtype).cuda()
    x[3, 128:256] = 0  # an all-zero group: the scale floor
    tok = torch.randint(0, T, (n,), generator=g).cuda()
    rid = torch.randint(-1, 16, (n, top), generator=g, dtype=torch.int32).cuda()
    rw = torch.rand((n, top), generator=g).cuda()
    got = ep.pack_rows_gpu(x, tok, rid, rw, wire)
    want = ep.pack_rows(x[tok].contiguous(), rid, rw, wire, quantize)
    torch.cuda.synchronize()
    assert got.shape == (n, ep.wire_row_bytes(H, top, wire)) and torch.equal(got, want)
    row_of = torch.randint(0, n, (200,), generator=g).cuda()
    rows = ep.unpack_rows_gpu(got, row_of, H, top, wire, dtype)
    ref_rows, ids, w = ep.unpack_rows(want, H, top, wire, dtype)
    torch.cuda.synchronize()
    assert torch.equal(rows.view(torch.int16), ref_rows[row_of].view(torch.int16))
    assert torch.equal(ids, rid) and torch.equal(w, rw)


def test_pack_kernel_flags_a_token_index_out_of_range():
    """The kernel checks each token index before it reads x: an index outside
    [0, tokens) writes zeros and sets LMOE_DEVERR_BAD_INDEX (4)."""
    from localmoe35ba3b_b200 import _native
    from localmoe35ba3b_b200.runtime import ep
    _native.check_device_errors()
    x = torch.ones((4, 256), dtype=torch.bfloat16, device='cuda')
    tok = torch.tensor([0, 4, 2], device='cuda')
    rid = torch.zeros((3, 2), dtype=torch.int32, device='cuda')
    rw = torch.ones((3, 2), device='cuda')
    buf = ep.pack_rows_gpu(x, tok, rid, rw, 'int8')
    rows = ep.unpack_rows_gpu(buf, torch.tensor([0, 1, 2, 3], device='cuda'), 256, 2, 'int8', torch.bfloat16)
    torch.cuda.synchronize()
    assert int(_native.error_word('cuda').item()) == _native.DEVERR_BAD_INDEX
    _native.error_word('cuda').zero_()
    assert torch.all(rows[1] == 0) and torch.all(rows[3] == 0)
    assert torch.all(rows[0] == 1) and torch.all(rows[2] == 1)


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
