"""CPU-only checks of the boundary: the C-ABI library loads and exports every
symbol the header declares, host-only entry points answer, and the Python
operators keep the reference's validation errors.  No kernel is launched."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, 'include', 'localmoe_b200.h')


def header_symbols():
    text = open(HEADER).read()
    return re.findall(r'LMOE_API\s+(?:int64_t|int)\s+(lmoe_\w+)\s*\(', text)


def test_header_declares_entry_points():
    names = header_symbols()
    assert len(names) >= 10
    assert len(set(names)) == len(names)


def test_library_exports_every_declared_symbol():
    from localmoe35ba3b_b200 import _native
    lib = ctypes.CDLL(_native.LIB_PATH)
    for name in header_symbols():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    from localmoe35ba3b_b200 import _native
    assert set(header_symbols()) == set(_native.SIGNATURES)
    _native.lib()  # sets argtypes for all; raises on a missing symbol


def test_host_only_entry_points():
    from localmoe35ba3b_b200 import _native
    lib = _native.lib()
    assert lib.lmoe_abi_version() == 3
    a = lib.lmoe_route_meta_size(2048, 8, 256)
    b = lib.lmoe_route_meta_size(4096, 8, 256)
    assert 0 < a < b and a % 256 == 0
    ws = lib.lmoe_moe_workspace_size(2048, 8, 256, 2048, 512)
    # hidden [(R+T), I] + down [(R+T), H] in bf16 dominate
    assert ws >= (16384 + 2048) * (512 + 2048) * 2
    assert lib.lmoe_plan_workspace_size(2048, 8, 256) >= 16384 * 4


def test_c_abi_rejects_bad_geometry_without_launching():
    from localmoe35ba3b_b200 import _native
    lib = _native.lib()
    p = ctypes.c_void_p(16)
    assert lib.lmoe_quantize_rows(p, p, p, 4, 100, 0, None) == _native.ERR_INVALID
    assert lib.lmoe_quantize_rows(None, p, p, 4, 128, 0, None) == _native.ERR_INVALID
    assert lib.lmoe_quantize_rows(p, p, p, 4, 128, 7, None) == _native.ERR_INVALID
    assert lib.lmoe_linear_w8a16(p, p, p, p, 4, 64, 100, 0, None, None) == _native.ERR_INVALID
    assert lib.lmoe_grouped_linear_w8a8(p, p, p, 8, 64, 256, 1, 1, 0, None, None, None) == _native.ERR_INVALID
    assert lib.lmoe_plan(p, 16, 8, 0, 16, p, p, p, p, p, None) == _native.ERR_INVALID
    assert lib.lmoe_routed_moe(p, p, p, 16, 8, p, p, p, p, 8, 2048, 100, *([None] * 8), p, 0, p, None,
                               None, None) == _native.ERR_INVALID


def test_ep_layer_sizes_and_validation():
    """The expert-parallel layer's row and workspace sizes; bad geometry, a null
    pointer or a misaligned buffer is refused before any launch."""
    from localmoe35ba3b_b200 import _native
    lib = _native.lib()
    # [payload | ids | weights | ranks] rounded up to 16 bytes
    assert lib.lmoe_ep_layer_row_bytes(2048, 8, _native.WIRE_DTYPE) == 4096 + 96
    assert lib.lmoe_ep_layer_row_bytes(2048, 8, _native.WIRE_INT8) == 2048 + 64 + 96
    assert lib.lmoe_ep_layer_row_bytes(2048, 1, _native.WIRE_INT8) == 2128
    assert lib.lmoe_ep_layer_row_bytes(100, 8, 0) == _native.ERR_INVALID
    assert lib.lmoe_ep_layer_row_bytes(2048, 17, 0) == _native.ERR_INVALID
    assert lib.lmoe_ep_layer_row_bytes(2048, 8, 2) == _native.ERR_INVALID
    pws = lib.lmoe_ep_plan_workspace_size(2048, 8, 256, 4)
    assert pws >= lib.lmoe_route_meta_size(2048, 8, 256) + 2048 * 4 * 4
    ows = lib.lmoe_ep_owner_workspace_size(2048, 8, 256, 8, 2048, 2048, 512)
    routes = 8 * 2048 * 8
    assert ows >= (routes + 2048) * (2048 + 512 + 2048) * 2 + routes * 4 + 8 * 2048 * 8 * 4
    assert lib.lmoe_ep_owner_workspace_size(2048, 8, 256, 3, 2048, 2048, 512) == _native.ERR_INVALID  # 256 % 3
    assert lib.lmoe_ep_owner_workspace_size(2048, 8, 256, 16, 2048, 2048, 512) == _native.ERR_INVALID  # world > 8
    assert lib.lmoe_ep_owner_workspace_size(2048, 8, 256, 2, 1024, 2048, 512) == _native.ERR_INVALID  # cap < tokens
    p = ctypes.c_void_p(256)
    assert lib.lmoe_ep_dispatch(p, p, p, 64, 8, 256, 2, 64, 2000, 0, 0, p, p, None, None, None) == _native.ERR_INVALID
    assert lib.lmoe_ep_dispatch(None, p, p, 64, 8, 256, 2, 64, 2048, 0, 0, p, p, None, None,
                                None) == _native.ERR_INVALID
    assert lib.lmoe_ep_dispatch(ctypes.c_void_p(264), p, p, 64, 8, 256, 2, 64, 2048, 0, 0, p, p, None, None,
                                None) == _native.ERR_INVALID
    assert lib.lmoe_ep_owner(p, p, 64, 8, 256, 2, 64, 2048, 512, 0, p, p, p, p, *([None] * 6), ctypes.c_void_p(272),
                             p, 0, None, None, None, None) == _native.ERR_INVALID  # workspace not 256-byte aligned
    assert lib.lmoe_ep_fold(p, p, p, 64, 8, 256, 2, 64, 2048, 512, None, 1, None, None, p, 0, None, None,
                            None) == _native.ERR_INVALID  # shared expert without the owner workspace
    # the direct transport: a peer table with a rank outside [0, world) or a null buffer is refused
    peers = _native.EpPeers()
    peers.rank = 2
    assert lib.lmoe_ep_dispatch(p, p, p, 64, 8, 256, 2, 64, 2048, 0, 0, None, p, None, ctypes.byref(peers),
                                None) == _native.ERR_INVALID
    peers.rank = 0
    assert lib.lmoe_ep_fold(p, p, p, 64, 8, 256, 2, 64, 2048, 512, p, 1, None, None, p, 0, None,
                            ctypes.byref(peers), None) == _native.ERR_INVALID


def test_operator_validation_errors_match_reference():
    from localmoe35ba3b_b200.operators import int8, routing, w8a8
    from localmoe35ba3b_b200.runtime import gpu_routes
    q = torch.zeros((64, 256), dtype=torch.int8)
    s = torch.zeros((64, 2), dtype=torch.float32)
    with pytest.raises(ValueError, match='W8A16 requires CUDA FP16/BF16 activations'):
        int8.linear(torch.zeros((2, 256), dtype=torch.bfloat16), q, s)
    with pytest.raises(ValueError, match='Expected CUDA rows with K divisible by 128'):
        w8a8.quantize(torch.zeros((2, 256), dtype=torch.bfloat16))
    with pytest.raises(ValueError, match='Expected contiguous CUDA \\[tokens,top_k\\] routing IDs'):
        gpu_routes.plan(torch.zeros((4, 8), dtype=torch.int64), 16, 16)
    with pytest.raises(ValueError, match='Expected nonempty CPU \\[tokens,top_k\\] IDs'):
        routing.plan_routes(torch.zeros((0, 8), dtype=torch.int64), 16)
    with pytest.raises(ValueError, match='Out-of-range expert ID'):
        routing.plan_routes(torch.tensor([[0, 16]]), 16)


def test_no_cpu_fallback_when_library_missing(monkeypatch):
    from localmoe35ba3b_b200 import _native
    monkeypatch.setattr(_native, 'LIB_PATH', os.path.join(ROOT, 'does-not-exist.so'))
    monkeypatch.setattr(_native, '_lib', None)
    with pytest.raises(_native.NativeError, match='no fallback'):
        _native.lib()


def test_bench_reference_arm_json_contract():
    """``bench.py --impl reference`` (no GPU needed) prints one JSON line on our arm's
    metric, unit and workload, with its cpu_baseline and e2e objects."""
    import json
    import subprocess
    import sys
    sys.path.insert(0, ROOT)
    import bench
    out = subprocess.run([sys.executable, os.path.join(ROOT, 'bench.py'), '--impl', 'reference', '--steps', '1',
                          '--warmup', '0'], capture_output=True, text=True, timeout=600, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [l for l in out.stdout.splitlines() if l.startswith('{')]
    assert len(lines) == 1
    d = json.loads(lines[0])
    assert d['impl'] == 'reference' and d['metric'] == bench.METRIC and d['unit'] == bench.UNIT
    assert d['higher_is_better'] is True and d['value'] > 0 and d['n_gpus'] == 1
    assert d['config'] == bench.config(bench.parse([]), 1)
    cb = d['cpu_baseline']
    assert cb['kind'] == 'port' and cb['cores'] >= 1 and cb['value'] == d['value'] and cb['sample']
    assert d['e2e'] == {'value': d['value'], 'unit': d['unit'], 'h2d_bytes_per_step': 0, 'd2h_bytes_per_step': 0}


def test_header_compiles_as_c_and_links(tmp_path):
    """A C host (no C++ and no CUDA headers) compiles against the header, links the
    library and calls its host-only entry points."""
    import shutil
    import subprocess
    gcc = shutil.which('gcc')
    if gcc is None:
        pytest.skip('gcc not available')
    from localmoe35ba3b_b200 import _native
    src = tmp_path / 'host.c'
    src.write_text('''
#include <stdio.h>
#include "localmoe_b200.h"
int main(void) {
  int64_t row = lmoe_ep_layer_row_bytes(2048, 8, LMOE_WIRE_INT8);
  int64_t bad = lmoe_ep_layer_row_bytes(100, 8, LMOE_WIRE_INT8);
  int rc = lmoe_quantize_rows((const void*)16, (int8_t*)16, (float*)16, 4, 100, LMOE_BF16, NULL);
  printf("%d %lld %lld %d\\n", lmoe_abi_version(), (long long)row, (long long)bad, rc);
  return 0;
}
''')
    exe = tmp_path / 'host'
    libdir = os.path.dirname(_native.LIB_PATH)
    cc = subprocess.run([gcc, '-std=c99', '-Wall', '-Werror', '-I', os.path.join(ROOT, 'include'), str(src),
                         '-o', str(exe), '-L', libdir, '-l:' + os.path.basename(_native.LIB_PATH),
                         '-Wl,-rpath,' + libdir], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    assert run.stdout.split() == ['3', '2208', str(_native.ERR_INVALID), str(_native.ERR_INVALID)]
