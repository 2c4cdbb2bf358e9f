"""Loader for the reference's converted checkpoint, straight into device-resident
MoE banks.

Format (written by qwen35_deploy/convert.py:60-118, read by
qwen35_deploy/model.py:29-64): ``manifest.json`` with ``complete`` and one
record per tensor (``name``, ``file``, ``bytes``, ``sha256``, ``format``); each
record's safetensors file holds ``{'q': int8 [.., N, K], 'scale': fp32
[.., N, K/128]}`` for ``format == 'int8_g128_fp32scale'`` and ``{'weight': ...}``
for ``'original'``.  Expert banks are stacked ``[E, N, K]`` under
``model.language_model.layers.<L>.mlp.experts.{gate_up_proj,down_proj}``.

On a B200 all 40 layers (33.2 GB of banks) stay resident, so the reference's
CPU bank, pinned slabs and GPU LRU (model.py:50-57, int8.py ExpertCache) are not
needed: each file is loaded once onto the device in the layout the kernels read
(no repacking).  Integrity checks follow model.py:52-54: the file size always,
the SHA-256 when ``verify``.
"""
import hashlib
import json
from pathlib import Path

import torch
from safetensors.torch import load_file

PREFIX = 'model.language_model.layers.{}.mlp.'
QUANT = 'int8_g128_fp32scale'


def sha256(path):
    """Hex SHA-256 of a file, streamed in 8 MiB blocks."""
    h = hashlib.sha256()
    with open(path, 'rb') as f:
        for block in iter(lambda: f.read(8 << 20), b''):
            h.update(block)
    return h.hexdigest()


def read_manifest(root):
    root = Path(root)
    manifest = json.loads((root / 'manifest.json').read_text())
    if not manifest.get('complete'):
        raise RuntimeError('Incomplete conversion: ' + str(root))
    return {r['name']: r for r in manifest['records']}


def _load(root, record, device, verify):
    path = Path(root) / record['file']
    if path.stat().st_size != record['bytes'] or (verify and sha256(path) != record['sha256']):
        raise RuntimeError('Corrupt artifact: ' + str(path))
    return load_file(str(path), device=str(device))


def _quant(root, records, name, device, verify):
    r = records.get(name)
    if r is None:
        raise RuntimeError('Missing tensor: ' + name)
    if r['format'] != QUANT:
        raise RuntimeError('Expected an INT8 group-128 tensor: ' + name)
    d = _load(root, r, device, verify)
    return d['q'].contiguous(), d['scale'].contiguous()


def _orig(root, records, name, device, verify, dtype):
    r = records.get(name)
    if r is None:
        raise RuntimeError('Missing tensor: ' + name)
    return _load(root, r, device, verify)['weight'].to(dtype).contiguous()


def load_moe_layer(root, layer, records=None, device='cuda', verify=True, dtype=torch.bfloat16):
    """One layer's MoE tensors: ``{'banks': [qg, sg, qd, sd], 'shared': [(q, s)] * 3
    (gate_proj, up_proj, down_proj), 'shared_gate': [1, H], 'router': [E, H]}``
    on ``device``."""
    records = read_manifest(root) if records is None else records
    p = PREFIX.format(layer)
    qg, sg = _quant(root, records, p + 'experts.gate_up_proj', device, verify)
    qd, sd = _quant(root, records, p + 'experts.down_proj', device, verify)
    if qg.ndim != 3 or qd.ndim != 3 or qg.shape[0] != qd.shape[0] or qg.shape[2] != qd.shape[1] \
            or qg.shape[1] != 2 * qd.shape[2]:
        raise ValueError('Invalid INT8 expert bank geometry')
    shared = [_quant(root, records, p + f'shared_expert.{n}.weight', device, verify)
              for n in ('gate_proj', 'up_proj', 'down_proj')]
    return {'banks': [qg, sg, qd, sd], 'shared': shared,
            'shared_gate': _orig(root, records, p + 'shared_expert_gate.weight', device, verify, dtype).reshape(1, -1),
            'router': _orig(root, records, p + 'gate.weight', device, verify, dtype)}


def load_moe_layers(root, layers=None, device='cuda', verify=True, dtype=torch.bfloat16):
    """Every MoE layer of the conversion (or the given layer indices), each as
    ``load_moe_layer`` returns it."""
    records = read_manifest(root)
    if layers is None:
        found = set()
        for name in records:
            if name.startswith('model.language_model.layers.') and name.endswith('.mlp.experts.gate_up_proj'):
                found.add(int(name.split('.')[3]))
        layers = sorted(found)
    return [load_moe_layer(root, i, records, device, verify, dtype) for i in layers]


def load_blocks(root, top_k=8, layers=None, device='cuda', verify=True, activation='w8a8'):
    """``SparseMoeBlock`` per MoE layer, banks resident on ``device``
    (``top_k`` is the config's num_experts_per_tok)."""
    from .block import SparseMoeBlock
    return [SparseMoeBlock(d['router'], top_k, d['banks'], d['shared'], d['shared_gate'], activation=activation)
            for d in load_moe_layers(root, layers, device, verify)]
