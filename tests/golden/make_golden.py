"""Generate golden vectors by running the reference's own code on CPU.

Run once, in a container that has the reference checkout (not on the GPU box):

    python tests/golden/make_golden.py /path/to/reference

What runs: ``qwen35_deploy.convert.quantize`` and
``qwen35_deploy.operators.routing.plan_routes`` (plain torch on CPU),
``qwen35_deploy.runtime.gpu_routes.plan`` (torch + its Triton ``_table``
kernel), and the Triton kernels ``int8._linear``, ``int8._grouped_linear``,
``int8._ordered_reduce``, ``w8a8._quant``, ``w8a8._linear``,
``prefill._routed``/``_reduce`` (through ``prefill.routed_moe``) and
``gpu_routes.routed_moe`` -- all under ``TRITON_INTERPRET=1``.

Two interpreter gaps are bridged without touching the reference's source:
* Triton's interpreter has no binding for ``libdevice.nearbyint`` used by
  ``w8a8._quant``; the kernel's module-level ``libdevice`` name is pointed at a
  shim whose ``nearbyint`` is NumPy's round-half-even ``rint`` (the same
  IEEE operation).
* ``gpu_routes.plan`` rejects non-CUDA ids; the ids are passed as a tensor
  subclass whose ``device.type`` reads ``'cuda'`` while the data stays on CPU.
The interpreter's ``tl.dot`` is wrong for bf16 operands and its fp32->bf16
store conversion truncates (GPU Triton rounds to nearest even), so every
kernel whose output rounding matters is pinned with fp16 activations and
outputs (which the reference accepts: ``int8.py:27``); bf16 runs the same code
paths, and the oracle's bf16 rounding is pinned against torch's conversion.

Inputs are regenerated from NumPy seeds by ``tests/golden/inputs.py`` (shared
with the tests), so the fixtures hold outputs plus input checksums only.
"""
import os
import sys
import types

os.environ['TRITON_INTERPRET'] = '1'
HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, HERE)

import numpy as np  # noqa: E402
import torch  # noqa: E402

import inputs as gi  # noqa: E402


def _t(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    return t if dtype is None else t.to(dtype)


def _np(t):
    t = t.detach().cpu()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    if t.dtype == torch.float16:
        return t.numpy().view(np.uint16)
    return t.numpy()


class _FakeCudaDevice(str):
    type = 'cuda'


class _CudaLooking(torch.Tensor):
    """CPU tensor whose ``.device.type`` reads 'cuda' (for gpu_routes.plan)."""
    @property
    def device(self):
        return _FakeCudaDevice('cpu')


def main(ref_root):
    sys.path.insert(0, ref_root)
    import triton.language as tl
    from triton.runtime.interpreter import TensorHandle
    from qwen35_deploy.convert import quantize
    from qwen35_deploy.operators import int8, w8a8, routing
    from qwen35_deploy.runtime import prefill, gpu_routes

    def nearbyint(x, **_):
        return tl.core.tensor(TensorHandle(np.rint(x.handle.data), x.handle.dtype.scalar), x.type)
    w8a8._quant.fn.__globals__['libdevice'] = types.SimpleNamespace(nearbyint=nearbyint)

    out = {}
    # ---- a15 weight quantiser: the reference's own known-answer case + random
    w = torch.linspace(-1, 1, 256).reshape(2, 128).bfloat16()
    q, s, _, _ = quantize(w)
    out['wq_known_q'], out['wq_known_s'] = _np(q), _np(s)
    wr = gi.weight_quant_input()
    q, s, _, _ = quantize(_t(wr))
    out['wq_rand_q'], out['wq_rand_s'] = _np(q), _np(s)

    # ---- a5 activation quantiser (bf16 input)
    xa = gi.act_quant_input()
    xt = torch.from_numpy(xa.view(np.int16)).view(torch.bfloat16)
    rows, k = xt.shape
    qq = torch.empty(rows, k, dtype=torch.int8)
    ss = torch.empty(rows, k // 128, dtype=torch.float32)
    w8a8._quant[(rows, k // 128)](xt, qq, ss, k)
    out['aq_q'], out['aq_s'] = _np(qq), _np(ss)

    # ---- a1 dense W8A16 linear (fp16), both tile shapes of int8.linear
    x, q, s = gi.linear_inputs()
    xh = torch.from_numpy(x.view(np.float16))
    m, kk = xh.shape
    n = q.shape[0]
    for bm, bn in ((16, 32), (32, 64)):
        y = torch.empty(m, n, dtype=torch.float16)
        int8._linear[((m + bm - 1) // bm, (n + bn - 1) // bn)](xh, _t(q), _t(s), y, m, n, kk, BM=bm, BN=bn)
        out[f'lin_y_{bm}x{bn}'] = _np(y)

    # ---- a4 / a6 table-driven decode GEMV
    g = gi.grouped_inputs()
    qb, sb, qd, sd = (_t(a) for a in (g['qg'], g['sg'], g['qd'], g['sd']))
    rowsel = g['experts']
    table = torch.tensor([[qb[e].data_ptr(), sb[e].data_ptr(), qd[e].data_ptr(), sd[e].data_ptr(), slot]
                          for e, slot in zip(rowsel, g['slots'])], dtype=torch.int64)
    E = len(rowsel)
    xs_h = torch.from_numpy(g['x_shared'].view(np.float16))
    xn_h = torch.from_numpy(g['x_rows'].view(np.float16))
    ng, nd = qb.shape[1], qd.shape[1]
    out['gl16_gu'] = _np(int8.grouped_linear(xs_h, table, E, ng, 0, True))
    out['gl16_dn'] = _np(int8.grouped_linear(xn_h, table, E, nd, 2, False))
    # W8A8: reference quantiser then the reference int8 GEMV (bf16 inputs)
    xs_b = torch.from_numpy(g['x_shared_bf16'].view(np.int16)).view(torch.bfloat16)
    xn_b = torch.from_numpy(g['x_rows_bf16'].view(np.int16)).view(torch.bfloat16)
    for tag, xin, nn, field, shared in (('gu', xs_b, ng, 0, True), ('dn', xn_b, nd, 2, False)):
        qx, sx = _quant_cpu(w8a8, xin)
        y = torch.empty((E, nn), dtype=torch.float16)
        w8a8._linear[(E, (nn + 31) // 32)](qx, sx, table, y, nn, xin.shape[-1], field, shared)
        out[f'gl8_{tag}'] = _np(y)

    # ---- a7 ordered combine (fp16)
    v, slots, wts = gi.reduce_inputs()
    vt = torch.from_numpy(v)
    tab = torch.zeros((len(slots), 5), dtype=torch.int64)
    tab[:, 4] = torch.from_numpy(slots)
    y = torch.empty(v.shape[1], dtype=torch.float16)
    int8._ordered_reduce[((v.shape[1] + 255) // 256,)](vt, tab, _t(wts), y, v.shape[1], len(slots))
    out['ored_y'] = _np(y)

    # ---- a8 / a9 routing metadata
    for name, (ids, experts) in gi.route_cases().items():
        ids_t = _t(ids)
        positions, segments = routing.plan_routes(ids_t, experts)
        out[f'{name}_positions'] = _np(positions)
        out[f'{name}_segments'] = np.asarray(segments, dtype=np.int64).reshape(-1, 3)
        for bm in (16, 32):
            pos, table, ordered, sl = gpu_routes.plan(ids_t.as_subclass(_CudaLooking), experts, bm)
            out[f'{name}_bm{bm}_pos'] = _np(pos.as_subclass(torch.Tensor))
            out[f'{name}_bm{bm}_table'] = _np(table.as_subclass(torch.Tensor))
            out[f'{name}_bm{bm}_ordered'] = _np(ordered.as_subclass(torch.Tensor))
            out[f'{name}_bm{bm}_slots'] = _np(sl.as_subclass(torch.Tensor))

    # ---- a10-a13 routed prefill FFN (fp16): CPU-plan and GPU-plan variants
    r = gi.routed_inputs()
    xh = torch.from_numpy(r['x'].view(np.float16))
    banks = [_t(r['qg']), _t(r['sg']), _t(r['qd']), _t(r['sd'])]
    ids_t = _t(r['ids'])
    wts = _t(r['weights'])
    out['rmoe_cpuplan'] = _np(prefill.routed_moe(xh, wts, ids_t, banks))
    out['rmoe_cpuplan_large'] = _np(prefill.routed_moe(xh, wts, ids_t, banks, large_tile=True))
    res = gpu_routes.routed_moe(xh, wts, ids_t.as_subclass(_CudaLooking), banks)
    out['rmoe_gpuplan'] = _np(res.as_subclass(torch.Tensor))
    # stage outputs straight from the reference kernels
    pos, table, ordered, sl = gpu_routes.plan(ids_t.as_subclass(_CudaLooking), banks[0].shape[0], 16)
    pos, table = pos.as_subclass(torch.Tensor), table.as_subclass(torch.Tensor)
    routes = ids_t.numel()
    gu = torch.empty((routes, banks[0].shape[1]), dtype=torch.float16)
    prefill._routed[(len(table), (gu.shape[1] + 31) // 32)](
        xh, banks[0], banks[1], pos, table, gu, gu.shape[1], xh.shape[1], True,
        banks[0].stride(0), banks[1].stride(0), BM=16, BN=32)
    out['rmoe_gu'] = _np(gu)

    out['input_checksums'] = gi.checksums()
    np.savez_compressed(os.path.join(HERE, 'golden.npz'), **out)
    print('wrote', len(out), 'arrays to', os.path.join(HERE, 'golden.npz'))


def _quant_cpu(w8a8, x):
    """``w8a8.quantize`` minus its ``is_cuda`` guard: same allocation and launch."""
    k = x.shape[-1]
    q = torch.empty_like(x, dtype=torch.int8)
    s = torch.empty((x.shape[0], k // 128), dtype=torch.float32)
    w8a8._quant[(x.shape[0], k // 128)](x, q, s, k)
    return q, s


if __name__ == '__main__':
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get('REFERENCE_ROOT', ''))
