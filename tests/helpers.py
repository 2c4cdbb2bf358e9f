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
