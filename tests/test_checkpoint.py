"""The converted-checkpoint loader (runtime/checkpoint.py) on a small
conversion written in the reference converter's format (convert.py:60-118):
tensors land unchanged, integrity failures raise as model.py:52-54 does."""
import json
import os

import numpy as np
import pytest
import torch

from helpers import write_conversion


def test_load_moe_layers_roundtrip(tmp_path):
    from localmoe35ba3b_b200.runtime import checkpoint
    truth = write_conversion(str(tmp_path), layers=2, E=8, H=256, I=128, seed=1)
    got = checkpoint.load_moe_layers(tmp_path, device='cpu')
    assert len(got) == 2
    for layer, d in enumerate(got):
        t = truth[layer]
        qg, sg, qd, sd = d['banks']
        assert qg.dtype == torch.int8 and sg.dtype == torch.float32 and qg.is_contiguous()
        assert np.array_equal(qg.numpy(), t['gate_up'][0]) and np.array_equal(sg.numpy(), t['gate_up'][1])
        assert np.array_equal(qd.numpy(), t['down'][0]) and np.array_equal(sd.numpy(), t['down'][1])
        for (q, s), (tq, ts) in zip(d['shared'], t['shared']):
            assert np.array_equal(q.numpy(), tq) and np.array_equal(s.numpy(), ts)
        assert d['router'].dtype == torch.bfloat16 and tuple(d['router'].shape) == (8, 256)
        assert np.array_equal(d['router'].float().numpy(), t['router'])
        assert tuple(d['shared_gate'].shape) == (1, 256)
        assert np.array_equal(d['shared_gate'].float().numpy(), t['shared_gate'])
    # a subset of layers
    only = checkpoint.load_moe_layers(tmp_path, layers=[1], device='cpu', verify=False)
    assert np.array_equal(only[0]['banks'][0].numpy(), truth[1]['gate_up'][0])


def test_integrity_failures(tmp_path):
    from localmoe35ba3b_b200.runtime import checkpoint
    write_conversion(str(tmp_path), layers=1, E=4, H=256, I=128, seed=2)
    records = checkpoint.read_manifest(tmp_path)
    rec = records['model.language_model.layers.0.mlp.experts.down_proj']
    path = tmp_path / rec['file']
    data = bytearray(path.read_bytes())
    data[-1] ^= 0xFF  # same size, different content: caught by the SHA-256 only
    path.write_bytes(bytes(data))
    with pytest.raises(RuntimeError, match='Corrupt artifact'):
        checkpoint.load_moe_layers(tmp_path, device='cpu')
    # without verification the size check alone passes this file
    checkpoint.load_moe_layers(tmp_path, device='cpu', verify=False)
    path.write_bytes(bytes(data[:-8]))  # truncated: caught by the size check
    with pytest.raises(RuntimeError, match='Corrupt artifact'):
        checkpoint.load_moe_layers(tmp_path, device='cpu', verify=False)


def test_incomplete_and_missing(tmp_path):
    from localmoe35ba3b_b200.runtime import checkpoint
    write_conversion(str(tmp_path), layers=1, E=4, H=256, I=128, seed=3)
    m = json.loads((tmp_path / 'manifest.json').read_text())
    m['records'] = [r for r in m['records'] if not r['name'].endswith('shared_expert.up_proj.weight')]
    (tmp_path / 'manifest.json').write_text(json.dumps(m))
    with pytest.raises(RuntimeError, match='Missing tensor'):
        checkpoint.load_moe_layers(tmp_path, device='cpu')
    m['complete'] = False
    (tmp_path / 'manifest.json').write_text(json.dumps(m))
    with pytest.raises(RuntimeError, match='Incomplete conversion'):
        checkpoint.read_manifest(tmp_path)
