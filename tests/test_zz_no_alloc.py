"""The allocation-free MoE entry point (lmoe_routed_moe_noalloc).

Some callers cannot allocate device memory where they run the expert block:
host runtimes that hand out device memory only from their own fixed arena,
and C/FFI hosts with no device allocator.  lmoe_routed_moe_noalloc takes its
scratch from a fixed-size device array inside the library instead of a
caller-provided workspace.

This test calls it through the C ABI several times in a row -- a large case,
a small one, the large one again -- so every call after the first runs on
scratch that an earlier call of a different size left behind, and checks each
result against the ordinary entry point lmoe_routed_moe on the same inputs,
within the bf16 tolerance the other tests use and bit for bit (both run the
same kernels).  It also checks that a call too large for the fixed scratch is
refused.  The file name makes pytest collect it last.
"""
import ctypes

import numpy as np
import pytest
import torch

from helpers import act, rand_q, rel_maxabs, rng
from oracle import oracle as O

pytestmark = pytest.mark.gpu


def _case(r, T, E, H, I, top):
    ids, w = O.route(r.standard_normal((T, E), dtype=np.float32) + O.zipf_bias(E, r)[None], top)
    qg, sg = rand_q(r, (E, 2 * I, H))
    qd, sd = rand_q(r, (E, H, I))
    shared = [rand_q(r, (I, H)), rand_q(r, (I, H)), rand_q(r, (H, I))]
    gate = act(r, (1, H), 'bf16', 0.02)
    x = act(r, (T, H), 'bf16')

    def d(a, bf=False):
        t = torch.from_numpy(np.ascontiguousarray(a))
        return (t.bfloat16() if bf else t).cuda()

    return dict(x=d(x, True), w=d(w), ids=d(ids), bank=[d(qg), d(sg), d(qd), d(sd)],
                shared=[d(a) for pair in shared for a in pair], gate=d(gate, True), T=T, E=E, H=H, I=I, top=top)


def _args(c, out):
    from localmoe35ba3b_b200 import _native as N
    return [N.ptr(c['x']), N.ptr(c['w']), N.ptr(c['ids']), c['T'], c['top'], *[N.ptr(t) for t in c['bank']],
            c['E'], c['H'], c['I'], *[N.ptr(t) for t in c['shared']], N.ptr(c['gate']), None, N.ptr(out),
            N.BF16]


def _reference_entry(c):
    from localmoe35ba3b_b200 import _native as N
    lib = N.lib()
    out = torch.empty_like(c['x'])
    ws = torch.empty(lib.lmoe_moe_workspace_size(c['T'], c['top'], c['E'], c['H'], c['I']), dtype=torch.uint8,
                     device='cuda')
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    rc = lib.lmoe_routed_moe(*_args(c, out), N.ptr(ws), N.ptr(err), None, N.stream())
    assert rc == 0
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return out


def test_noalloc_matches_allocating_entry_point_large_small_large():
    if not torch.cuda.is_available():
        pytest.skip('needs a CUDA device')
    from localmoe35ba3b_b200 import _native as N
    lib = N.lib()
    r = rng(2024)
    big, small = _case(r, 128, 64, 2048, 512, 8), _case(r, 96, 32, 512, 256, 8)
    cases = [big, small, big]
    refs = [_reference_entry(c) for c in cases]
    err = torch.zeros(1, dtype=torch.int32, device='cuda')
    for c, ref in zip(cases, refs):
        out = torch.empty_like(c['x'])
        rc = lib.lmoe_routed_moe_noalloc(*_args(c, out), N.ptr(err), N.stream())
        assert rc == 0
        torch.cuda.synchronize()
        assert int(err.item()) == 0
        got = out.float().cpu().numpy()
        want = ref.float().cpu().numpy()
        assert rel_maxabs(got, want) < 1e-2
        assert np.array_equal(got, want)


def test_noalloc_refuses_calls_beyond_its_scratch():
    if not torch.cuda.is_available():
        pytest.skip('needs a CUDA device')
    from localmoe35ba3b_b200 import _native as N
    lib = N.lib()
    T = 256
    assert lib.lmoe_moe_workspace_size(T, 8, 256, 2048, 512) > lib.lmoe_routed_moe_noalloc_limit()
    p = ctypes.c_void_p(16)
    rc = lib.lmoe_routed_moe_noalloc(p, p, p, T, 8, p, p, p, p, 256, 2048, 512, *([None] * 7), None, p, N.BF16,
                                     None, N.stream())
    assert rc == N.ERR_UNSUPPORTED
