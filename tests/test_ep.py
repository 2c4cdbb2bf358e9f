"""Expert parallelism (runtime/ep.py) on CPU ranks over gloo, world sizes 2 and 4,
with the bf16 and the int8 (W8A8-quantised) dispatch wire.

The orchestration -- send plan, all-to-all of the counts and of the packed rows
(payload, route ids, route weights), per-rank ordered pre-reduction, reverse
all-to-all, per-token fold in ascending rank order, gated shared expert,
residual -- runs as on GPUs; the expert compute is the oracle's, one route per
row, pre-reduced by ``ep.prereduced`` (on GPUs the routed block's own ordered
combine does that step).  Checked against (a) the single-device oracle within
the 1e-2 bar, and (b) an independent restatement of the expert-parallel rounding
sequence, bit for bit.
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


def _case(world, skew=False):
    """Seeded layer and per-rank tokens; ``skew`` routes every token to rank 0's
    experts only (the other ranks then receive no rows at all)."""
    r = np.random.default_rng(321)
    qg, sg = O.quantize_weight(r.standard_normal((E, 2 * I, H)).astype(np.float32) * 0.02)
    qd, sd = O.quantize_weight(r.standard_normal((E, H, I)).astype(np.float32) * 0.02)
    shared = [O.quantize_weight(r.standard_normal(s).astype(np.float32) * 0.02)
              for s in ((I, H), (I, H), (H, I))]
    gate = O.round_to(r.standard_normal((1, H)).astype(np.float32) * 0.02, 'bf16')
    xs, ids, ws, res = [], [], [], []
    for _ in range(world):
        logits = r.standard_normal((T, E)).astype(np.float32) + O.zipf_bias(E, r)[None]
        if skew:
            logits[:, :E // world] += 30.0
        i, w = O.route(logits, TOP)
        xs.append(O.round_to(r.standard_normal((T, H)).astype(np.float32), 'bf16'))
        ids.append(i)
        ws.append(w)
        res.append(O.round_to(r.standard_normal((T, H)).astype(np.float32), 'bf16'))
    return (qg, sg, qd, sd), shared, gate, xs, ids, ws, res


def _bf(a):
    return torch.from_numpy(np.asarray(a, dtype=np.float32)).to(torch.bfloat16)


def _wire_quantize(rows):
    q, s = O.quantize_act(rows.float().numpy())
    return torch.from_numpy(q), torch.from_numpy(s)


def _worker(rank, world, wire, port, out_dir, skew=False):
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=world)
    try:
        from localmoe35ba3b_b200.runtime import ep
        bank, shared, gate, xs, ids, ws, res = _case(world, skew)
        e_loc = E // world
        lb = [b[rank * e_loc:(rank + 1) * e_loc] for b in bank]

        def route_fn(x_rows, w, i):
            y = O.routed_moe(x_rows.float().numpy(), w.numpy(), i.numpy(), lb, 'bf16')
            return _bf(y)
        local_moe = ep.prereduced(route_fn)

        def shared_part(x):
            xn = x.float().numpy()
            sh = O.shared_expert(xn, shared, 'bf16')
            return _bf(O.shared_gate_combine(np.zeros_like(xn), sh, xn, gate, 'bf16'))

        out = ep.moe_forward(_bf(xs[rank]), torch.from_numpy(ws[rank]), torch.from_numpy(ids[rank]), E, local_moe,
                             shared_part, residual=_bf(res[rank]), wire=wire, quantize=_wire_quantize)
        np.save(os.path.join(out_dir, f'ep{rank}.npy'), out.float().numpy())
    finally:
        dist.destroy_process_group()


def _ep_sequence(x, w, ids, bank, shared, gate, res, world, wire='bf16'):
    """The expert-parallel rounding sequence restated on one process; with the
    int8 wire the routed experts read round_bf16(q * s) of the W8A8 quantisation."""
    xr = x if wire == 'bf16' else O.round_to(O.dequant(*O.quantize_act(x)), 'bf16')
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
                v = O.routed_moe(xr[t:t + 1], w[t:t + 1, k:k + 1], np.array([[0]]),
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


def test_wire_rows_round_trip():
    from localmoe35ba3b_b200.runtime import ep
    # H = 2048, top 8: 4096 + 64 bytes on the bf16 wire, 2048 + 64 + 64 on the int8 wire
    assert ep.wire_row_bytes(2048, 8, 'bf16') == 4160
    assert ep.wire_row_bytes(2048, 8, 'int8') == 2176
    with pytest.raises(ValueError):
        ep.wire_row_bytes(2048, 8, 'fp8')
    r = np.random.default_rng(5)
    x = _bf(r.standard_normal((7, H)) * 3)
    rid = torch.tensor(r.integers(-1, 8, (7, TOP)), dtype=torch.int32)
    rw = torch.tensor(r.random((7, TOP)), dtype=torch.float32)
    buf = ep.pack_rows(x, rid, rw, 'bf16')
    assert buf.dtype == torch.uint8 and buf.shape == (7, ep.wire_row_bytes(H, TOP, 'bf16'))
    rows, ids, w = ep.unpack_rows(buf, H, TOP, 'bf16', torch.bfloat16)
    assert torch.equal(rows, x) and torch.equal(ids, rid) and torch.equal(w, rw)
    buf = ep.pack_rows(x, rid, rw, 'int8', _wire_quantize)
    assert buf.shape == (7, ep.wire_row_bytes(H, TOP, 'int8'))
    rows, ids, w = ep.unpack_rows(buf, H, TOP, 'int8', torch.bfloat16)
    want = O.round_to(O.dequant(*O.quantize_act(x.float().numpy())), 'bf16')
    assert np.array_equal(rows.float().numpy(), want)
    assert torch.equal(ids, rid) and torch.equal(w, rw)
    empty = torch.empty((0, ep.wire_row_bytes(H, TOP, 'int8')), dtype=torch.uint8)
    rows, ids, w = ep.unpack_rows(empty, H, TOP, 'int8', torch.bfloat16)
    assert rows.shape == (0, H) and ids.shape == (0, TOP) and w.shape == (0, TOP)


@pytest.mark.parametrize('wire', ['bf16', 'int8'])
@pytest.mark.parametrize('world', [2, 4])
def test_expert_parallel_matches_oracle(tmp_path, world, wire):
    port = _free_port()
    mp.start_processes(_worker, args=(world, wire, port, str(tmp_path)), nprocs=world, join=True,
                       start_method='spawn')
    bank, shared, gate, xs, ids, ws, res = _case(world)
    for rank in range(world):
        got = np.load(tmp_path / f'ep{rank}.npy')
        single = O.round_to(res[rank] + O.moe_block(xs[rank], ws[rank], ids[rank], bank, shared, gate, 'bf16'), 'bf16')
        err = np.abs(got - single).max() / np.abs(single).max()
        assert err < 1e-2, err
        exact = _ep_sequence(xs[rank], ws[rank], ids[rank], bank, shared, gate, res[rank], world, wire)
        assert np.array_equal(got, exact)


def test_expert_parallel_ranks_without_rows(tmp_path):
    """Every token routes to rank 0's experts: rank 1 receives no rows, sends all of its
    rows to rank 0 and gets them back pre-reduced; bit-exact as above."""
    world = 2
    port = _free_port()
    mp.start_processes(_worker, args=(world, 'bf16', port, str(tmp_path), True), nprocs=world, join=True,
                       start_method='spawn')
    bank, shared, gate, xs, ids, ws, res = _case(world, skew=True)
    assert all((i < E // world).all() for i in ids)
    for rank in range(world):
        got = np.load(tmp_path / f'ep{rank}.npy')
        exact = _ep_sequence(xs[rank], ws[rank], ids[rank], bank, shared, gate, res[rank], world)
        assert np.array_equal(got, exact)


def _leaving_worker(rank, port, out_dir):
    """Rank 1 leaves between layers (exits without joining the layer's exchange);
    rank 0 runs the layer and must see an error from its collective, not hang."""
    import datetime
    os.environ['MASTER_ADDR'] = '127.0.0.1'
    os.environ['MASTER_PORT'] = str(port)
    dist.init_process_group('gloo', rank=rank, world_size=2, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        os._exit(0)
    from localmoe35ba3b_b200.runtime import ep
    bank, shared, gate, xs, ids, ws, res = _case(2)

    def route_fn(x_rows, w, i):
        return _bf(O.routed_moe(x_rows.float().numpy(), w.numpy(), i.numpy(), [b[:E // 2] for b in bank], 'bf16'))
    try:
        ep.moe_forward(_bf(xs[0]), torch.from_numpy(ws[0]), torch.from_numpy(ids[0]), E, ep.prereduced(route_fn))
        result = 'not detected'
    except RuntimeError as e:
        result = 'detected: ' + str(e).splitlines()[0][:200]
    with open(os.path.join(out_dir, 'leave.txt'), 'w') as f:
        f.write(result)
    os._exit(0)


def test_rank_that_leaves_is_detected_by_the_next_exchange(tmp_path):
    """Failure detection on the host: the surviving rank's next all-to-all ends with a
    RuntimeError (closed peer or the process group's 10 s timeout) instead of waiting
    for good."""
    import time
    port = _free_port()
    t0 = time.time()
    mp.start_processes(_leaving_worker, args=(port, str(tmp_path)), nprocs=2, join=True, start_method='spawn')
    assert (tmp_path / 'leave.txt').read_text().startswith('detected')
    assert time.time() - t0 < 120
