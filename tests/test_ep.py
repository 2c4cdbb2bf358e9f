"""Expert parallelism (runtime/ep.py) on CPU ranks over gloo, world sizes 2 and 4.

The orchestration -- send plan, all-to-all of counts, rows and route lists,
route expansion, per-rank ordered pre-reduction, reverse all-to-all, per-token
fold in ascending rank order, gated shared expert, residual -- runs exactly as
on GPUs; the expert compute is the oracle's.  Checked against (a) the
single-device oracle within the 1e-2 bar, and (b) an independent restatement of
the expert-parallel rounding sequence, bit for bit.
"""
import os
import socket

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import oracle as O

E, H, I, TOP, T = 16, 256, 128, 4, 12


def _case(world):
    r = np.random.default_rng(321)
    qg, sg = O.quantize_weight(r.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.02)
    qd, sd = O.quantize_weight(r.standard_normal((E, H, I)).astype(np.float32) * 0.02)
    shared = [O.quantize_weight(r.standard_normal(s).astype(np.float32) * 0.02)
              for s in ((I, H), (I, H), (H, I))]
    gate = O.round_to(r.standard_normal((1, H)).astype(np.float32) * 0.02, 'bf16')
    xs, ids, ws, res = [], [], [], []
    for _ in range(world):
        logits = r.standard_normal((T, E)).astype(np.float32) + O.zipf_bias(E, r)[None]
        i, w = O.route(logits, TOP)
        xs.append(O.round_to(r.standard_normal((T, H)).astype(np.float32), 'bf16'))
        ids.append(i)
        ws.append(w)
        res.append(O.round_to(r.standard_normal((T, H)).astype(np.float32), 'bf16'))
    return (qg, sg, qd, sd), shared, gate, xs, ids, ws, res


def _bf(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


def _worker(rank, world, port, out_dir):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from localmoe35ba3b_b200.runtime import ep
        bank, shared, gate, xs, ids, ws, res = _case(world)
        e_loc = E // world
        lb = [b[rank * e_loc:(rank + 1) * e_loc] for b in bank]

        def local_moe(x_rows, w, i):
            y = O.routed_moe(x_rows.float().numpy(), w.numpy(), i.numpy(), lb, 'bf16')
            return _bf(y)

        def shared_part(x):
            xn = x.float().numpy()
            sh = O.shared_expert(xn, shared, 'bf16')
            return _bf(O.shared_gate_combine(np.zeros_like(xn), sh, xn, gate, 'bf16'))

        out = ep.moe_forward(_bf(xs[rank]), torch.from_numpy(ws[rank]), torch.from_numpy(ids[rank]), E, local_moe,
                             shared_part, residual=_bf(res[rank]))
        np.save(os.path.join(out_dir, f'ep{rank}.npy'), out.float().numpy())
    finally:
        dist.destroy_process_group()


def _ep_sequence(x, w, ids, bank, shared, gate, res, world):
    """The expert-parallel rounding sequence restated on one process."""
    e_loc = E // world
    out = np.zeros((T, H), dtype=np.float32)
    for t in range(T):
        acc = np.zeros(H, dtype=np.float32)
        for g in range(world):
            sel = [k for k in range(TOP) if ids[t, k] // e_loc == g]
            if not sel:
                continue
            part = np.zeros(H, dtype=np.float32)
            for k in sorted(sel, key=lambda k: ids[t, k]):
                e = int(ids[t, k])
                v = O.routed_moe(x[t:t + 1], w[t:t + 1, k:k + 1], np.array([[0]]),
                                 [b[e:e + 1] for b in bank], 'bf16')[0]
                part = O.round_to(part + v, 'bf16')
            acc = O.round_to(acc + part, 'bf16')
        out[t] = acc
    sh = O.shared_gate_combine(np.zeros_like(x), O.shared_expert(x, shared, 'bf16'), x, gate, 'bf16')
    return O.round_to(res + O.round_to(out + sh, 'bf16'), 'bf16')


def _free_port():
    s = socket.socket()
    s.bind(('127.0.0.1', 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_plan_groups_rows_by_rank():
    from localmoe35ba3b_b200.runtime import ep
    ids = torch.tensor([[0, 9, 3, 12], [15, 14, 13, 12], [1, 2, 3, 4]])
    w = torch.tensor([[.4, .3, .2, .1], [.25, .25, .25, .25], [.1, .2, .3, .4]])
    tok, counts, rid, rw = ep.plan(ids, w, 16, 2)
    assert counts.tolist() == [2, 2]
    assert tok.tolist() == [0, 2, 0, 1]
    assert rid.tolist() == [[0, -1, 3, -1], [1, 2, 3, 4], [-1, 1, -1, 4], [7, 6, 5, 4]]
    assert rw[0].tolist() == pytest.approx([.4, 0, .2, 0])


def test_plan_four_ranks():
    from localmoe35ba3b_b200.runtime import ep
    ids = torch.tensor([[0, 9, 3, 12], [15, 14, 13, 12], [1, 2, 3, 4]])
    w = torch.tensor([[.4, .3, .2, .1], [.25, .25, .25, .25], [.1, .2, .3, .4]])
    tok, counts, rid, rw = ep.plan(ids, w, 16, 4)
    # 4 experts per rank: token 0 -> ranks {0, 2, 3}, token 1 -> {3}, token 2 -> {0, 1}
    assert counts.tolist() == [2, 1, 1, 2]
    assert tok.tolist() == [0, 2, 2, 0, 0, 1]
    assert rid.tolist() == [[0, -1, 3, -1], [1, 2, 3, -1], [-1, -1, -1, 0],
                            [-1, 1, -1, -1], [-1, -1, -1, 0], [3, 2, 1, 0]]
    assert rw[1].tolist() == pytest.approx([.1, .2, .3, 0])
    assert rw[5].tolist() == pytest.approx([.25] * 4)
    with pytest.raises(ValueError):
        ep.plan(ids, w, 16, 3)


@pytest.mark.parametrize('world', [2, 4])
def test_expert_parallel_matches_oracle(tmp_path, world):
    port = _free_port()
    mp.start_processes(_worker, args=(world, port, str(tmp_path)), nprocs=world, join=True, start_method='spawn')
    bank, shared, gate, xs, ids, ws, res = _case(world)
    for rank in range(world):
        got = np.load(tmp_path / f'ep{rank}.npy')
        single = O.round_to(res[rank] + O.moe_block(xs[rank], ws[rank], ids[rank], bank, shared, gate, 'bf16'), 'bf16')
        err = np.abs(got - single).max() / np.abs(single).max()
        assert err < 1e-2, err
        exact = _ep_sequence(xs[rank], ws[rank], ids[rank], bank, shared, gate, res[rank], world)
        assert np.array_equal(got, exact)
