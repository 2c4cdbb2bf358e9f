"""Shared test helpers: seeded weight banks, dtype conversions, tolerances."""
import numpy as np
import torch

from oracle import oracle as O

BF16, F16 = 'bf16', 'f16'
TORCH_DT = {BF16: torch.bfloat16, F16: torch.float16}


def rng(seed):
    return np.random.default_rng(seed)


def rand_q(r, shape):
    """int8 weights in [-127, 127] with realistic absmax-RTN scales."""
    q = r.integers(-127, 128, size=shape, dtype=np.int8)
    k = shape[-1]
    s = (r.uniform(0.5, 1.5, size=shape[:-1] + (k // 128,)) * (0.02 * 3 / 127)).astype(np.float32)
    return q, s


def act(r, shape, dtype, scale=1.0):
    """Activations as float32 values exactly representable in dtype."""
    x = r.standard_normal(shape, dtype=np.float32) * scale
    return O.round_to(x, dtype)


def to_dev(a, dtype=None, device='cuda'):
    """numpy -> torch on device; float32 arrays are cast to the activation dtype."""
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(TORCH_DT[dtype])
    return t.to(device)


def to_np(t):
    return t.detach().float().cpu().numpy()


def ulp_close(got, ref, dtype, ulps=1, frac_exact=0.9, atol_rel=2.0 ** -13):
    """|got - ref| <= ulps * ulp(ref) + atol_rel * max|ref| elementwise, and most
    elements equal.  Used where the reference leaves the fp32 summation order
    to tl.dot: a different order moves the fp32 sum by a few fp32 ulps of the
    summed magnitudes, which the absolute term covers for outputs that
    cancel to near zero."""
    got = np.asarray(got, dtype=np.float32)
    ref = np.asarray(ref, dtype=np.float32)
    mant = 7 if dtype == BF16 else 10
    mag = np.maximum(np.abs(ref), np.float32(2.0 ** -100))
    ulp = np.exp2(np.floor(np.log2(mag)) - mant)
    bad = np.abs(got - ref) > ulps * ulp + atol_rel * float(np.abs(ref).max())
    exact = float((got == ref).mean())
    return (not bad.any()) and exact >= frac_exact, dict(max_ulps=float((np.abs(got - ref) / ulp).max()),
                                                         exact=exact, nbad=int(bad.sum()))


def rel_maxabs(got, ref):
    """max|got - ref| / max|ref| -- the north-star tolerance metric."""
    got = np.asarray(got, dtype=np.float64)
    ref = np.asarray(ref, dtype=np.float64)
    return float(np.abs(got - ref).max() / max(np.abs(ref).max(), 1e-30))


def write_conversion(root, layers, E, H, I, seed=0):
    """A small converted checkpoint in the reference converter's output format
    (convert.py:60-118: per-tensor safetensors files, per-record size and
    SHA-256, manifest.json with complete=True) holding the MoE tensors of
    ``layers`` layers.  Returns {layer: {name suffix: numpy arrays}}."""
    import hashlib
    import json
    import os
    from safetensors.torch import save_file
    r = rng(seed)
    records, truth = [], {}

    def put(name, values, fmt):
        key = hashlib.sha256(name.encode()).hexdigest()[:24]
        path = os.path.join(root, key + '.safetensors')
        save_file({k: torch.from_numpy(np.ascontiguousarray(v)) if isinstance(v, np.ndarray) else v
                   for k, v in values.items()}, path)
        with open(path, 'rb') as f:
            digest = hashlib.sha256(f.read()).hexdigest()
        first = next(iter(values.values()))
        records.append({'name': name, 'shape': list(first.shape), 'file': key + '.safetensors', 'sha256': digest,
                        'bytes': os.path.getsize(path), 'format': fmt})

    for layer in range(layers):
        p = f'model.language_model.layers.{layer}.mlp.'
        t = {}
        t['gate_up'] = rand_q(r, (E, 2 * I, H))
        t['down'] = rand_q(r, (E, H, I))
        t['shared'] = [rand_q(r, (I, H)), rand_q(r, (I, H)), rand_q(r, (H, I))]
        t['shared_gate'] = act(r, (1, H), BF16, 0.02)
        t['router'] = act(r, (E, H), BF16, 0.05)
        put(p + 'experts.gate_up_proj', {'q': t['gate_up'][0], 'scale': t['gate_up'][1]}, 'int8_g128_fp32scale')
        put(p + 'experts.down_proj', {'q': t['down'][0], 'scale': t['down'][1]}, 'int8_g128_fp32scale')
        for n, (q, s) in zip(('gate_proj', 'up_proj', 'down_proj'), t['shared']):
            put(p + f'shared_expert.{n}.weight', {'q': q, 'scale': s}, 'int8_g128_fp32scale')
        put(p + 'shared_expert_gate.weight', {'weight': torch.from_numpy(t['shared_gate']).to(torch.bfloat16)},
            'original')
        put(p + 'gate.weight', {'weight': torch.from_numpy(t['router']).to(torch.bfloat16)}, 'original')
        truth[layer] = t
    with open(os.path.join(root, 'manifest.json'), 'w') as f:
        json.dump({'identity': {'format': 'q36-w8a16-g128-rtn-fp32scale-v1'}, 'records': records, 'complete': True,
                   'bytes': sum(x['bytes'] for x in records)}, f)
    return truth
