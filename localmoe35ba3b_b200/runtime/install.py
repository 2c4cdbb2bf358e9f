"""``install(model)``: put the B200 path into a loaded model through the
reference's own seam, submodule replacement by name.

The reference builds the HF model and then swaps modules by name
(qwen35_deploy/model.py:16-18 ``replace``): every converted 2-D weight becomes an
``Int8Linear`` (:61-62) and every ``mlp.experts`` an ``Int8Experts`` over its host
bank (:67-70); ``--activation w8a8`` (the default) also installs the W8A8 decode
GEMV (cli.py:28,37-39).  ``install`` walks such a model and replaces, by the same
seam:

* each sparse-MoE block -- a module holding ``gate`` (router ``weight [E, H]``,
  ``top_k``), ``experts`` (INT8 banks), ``shared_expert`` (three INT8 linears)
  and ``shared_expert_gate`` (``weight [1, H]``), the HF
  ``Qwen3_5MoeSparseMoeBlock`` the reference keeps -- by one ``SparseMoeBlock``
  whose banks are resident on ``device``;
* every other INT8 linear -- a module holding an int8 ``q [N, K]`` and an fp32
  ``scale [N, K/128]``, the reference's ``Int8Linear`` -- by this package's
  ``Int8Linear`` over the same tensors.

Modules are recognised by what they hold, not by their class, so neither the
reference package nor transformers has to be importable.  Expert banks are read
from the reference's ``Int8Experts`` (``gate_up`` / ``down`` dicts of
``{'q', 'scale'}``, int8.py:127-130) or from this package's ``Int8Experts``.
"""
import torch

from ..operators.int8 import Int8Experts, Int8Linear
from .block import SparseMoeBlock


def _int8_pair(m):
    """``(q, scale)`` of an INT8 group-128 linear, else None."""
    q, s = getattr(m, 'q', None), getattr(m, 'scale', None)
    if not (isinstance(q, torch.Tensor) and isinstance(s, torch.Tensor)):
        return None
    if q.dtype != torch.int8 or q.ndim != 2 or q.shape[1] % 128 or s.dtype != torch.float32:
        return None
    if tuple(s.shape) != (q.shape[0], q.shape[1] // 128):
        return None
    return q, s


def _banks(experts):
    """``[qg, sg, qd, sd]`` of an experts module, else None."""
    if isinstance(experts, Int8Experts):
        return experts.banks()
    gu, dn = getattr(experts, 'gate_up', None), getattr(experts, 'down', None)
    if isinstance(gu, dict) and isinstance(dn, dict) and {'q', 'scale'} <= set(gu) and {'q', 'scale'} <= set(dn):
        return [gu['q'], gu['scale'], dn['q'], dn['scale']]
    return None


def _is_moe_block(m):
    return all(hasattr(m, a) for a in ('gate', 'experts', 'shared_expert', 'shared_expert_gate'))


def _replace(model, name, module):
    parent, _, child = name.rpartition('.')
    setattr(model.get_submodule(parent) if parent else model, child, module)


def _to(t, device):
    return t.to(device).contiguous()


def install(model, activation='w8a8', device='cuda'):
    """Replace ``model``'s sparse-MoE blocks and INT8 linears in place; returns
    ``{'blocks': n, 'linears': m}``.  Raises ``ValueError`` for a block whose
    experts or shared expert are not INT8 group-128 (there is no float path)."""
    if activation not in ('w8a8', 'w8a16'):
        raise ValueError("activation must be 'w8a8' or 'w8a16'")
    if _is_moe_block(model) or _int8_pair(model) is not None:
        raise ValueError('install replaces submodules: pass the model that holds them')
    blocks = [(n, m) for n, m in model.named_modules() if n and _is_moe_block(m)
              and not isinstance(m, SparseMoeBlock)]
    for name, m in blocks:
        banks = _banks(m.experts)
        if banks is None:
            raise ValueError(f'{name}.experts holds no INT8 group-128 banks')
        shared = [_int8_pair(getattr(m.shared_expert, p, None)) for p in ('gate_proj', 'up_proj', 'down_proj')]
        if any(p is None for p in shared):
            raise ValueError(f'{name}.shared_expert is not INT8 group-128')
        router = m.gate.weight.detach()
        blk = SparseMoeBlock(_to(router, device), int(m.gate.top_k), [_to(b, device) for b in banks],
                             [(_to(q, device), _to(s, device)) for q, s in shared],
                             _to(m.shared_expert_gate.weight.detach().to(router.dtype), device),
                             activation=activation)
        _replace(model, name, blk)
    linears = [(n, p) for n, m in model.named_modules() if n and not isinstance(m, Int8Linear)
               for p in [_int8_pair(m)] if p is not None]
    for name, (q, s) in linears:
        _replace(model, name, Int8Linear(_to(q, device), _to(s, device)))
    return {'blocks': len(blocks), 'linears': len(linears)}
