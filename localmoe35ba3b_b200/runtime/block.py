"""The whole sparse-MoE block on the device: router + routed experts + gated
shared expert.

The reference keeps the HF ``Qwen3_5MoeSparseMoeBlock`` and replaces only its
``experts`` submodule and the linears (qwen35_deploy/model.py:57-68), so its
block runs the HF router (``Qwen3_5MoeTopKRouter.forward``,
transformers/models/qwen3_5_moe/modeling_qwen3_5_moe.py:762-770), the experts
and the shared-expert gate and add (:781-792) as separate torch steps, with a
host synchronisation per layer in ``Int8Experts.forward`` (int8.py:160).

``TopKRouter`` mirrors the HF router's interface: the logits are the same bf16
``F.linear`` (a plain library GEMM), the fp32 softmax / top-k / renormalise tail
is one library kernel (``lmoe_router_topk``).  ``SparseMoeBlock`` mirrors the HF
block's ``forward(hidden_states) -> hidden_states``: one token goes through the
graph-capturable decode chain, more tokens through the fused prefill block --
with 64, 128 or 256 experts its router too (``lmoe_moe_block_router``: the
logits on tensor cores, the tail and the metadata's route counts in the same
kernel); the shared expert is folded into the same library call as the routed
experts.
"""
import torch
import torch.nn.functional as F

from .. import _native as N
from .decode import decode_block
from .gpu_routes import moe_block, moe_block_router, router_gemm_ok


def topk_from_logits(logits, top_k, return_probs=False):
    """fp32 softmax / top-k / renormalise of ``logits [T, E]`` (FP16/BF16, on
    the GPU; hf :765-769): ``(weights fp32 [T, top_k], ids int64 [T, top_k])``,
    ids in descending probability with ties to the lower expert id (the set
    ``torch.topk`` returns), and the fp32 softmax first when ``return_probs``."""
    if not logits.is_cuda or logits.dtype not in (torch.float16, torch.bfloat16) or logits.ndim != 2:
        raise ValueError('Expected CUDA FP16/BF16 router logits [tokens, experts]')
    t, e = logits.shape
    if not 1 <= top_k <= min(32, e):
        raise ValueError('top_k must be in [1, min(32, experts)]')
    logits = logits.contiguous()
    w = torch.empty((t, top_k), dtype=torch.float32, device=logits.device)
    ids = torch.empty((t, top_k), dtype=torch.int64, device=logits.device)
    probs = torch.empty((t, e), dtype=torch.float32, device=logits.device) if return_probs else None
    N.call('lmoe_router_topk', N.ptr(logits), t, e, top_k, N.ptr(w), N.ptr(ids), N.ptr(probs),
           N.dtype_code(logits.dtype), N.stream(logits.device))
    return (probs, w, ids) if return_probs else (w, ids)


def route(x, weight, top_k, return_probs=False):
    """HF router on ``x [T, H]`` with the gate ``weight [E, H]``: the bf16
    logits ``F.linear(x, weight)`` (hf :764), then ``topk_from_logits``."""
    if not x.is_cuda or x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError('Expected CUDA FP16/BF16 hidden states')
    if x.ndim != 2 or weight.ndim != 2 or weight.shape[1] != x.shape[1]:
        raise ValueError('Router weight must be [experts, hidden]')
    return topk_from_logits(F.linear(x, weight.to(x.dtype)), top_k, return_probs)


class TopKRouter(torch.nn.Module):
    """Drop-in for HF ``Qwen3_5MoeTopKRouter``: ``forward(hidden_states)``
    returns ``(router_logits, router_scores, router_indices)`` as HF does
    (the first is the fp32 softmax, the second the renormalised top-k fp32)."""

    def __init__(self, weight, top_k):
        super().__init__()
        self.weight = torch.nn.Parameter(weight, requires_grad=False)
        self.top_k = top_k
        self.num_experts, self.hidden_dim = weight.shape

    def forward(self, hidden_states):
        x = hidden_states.reshape(-1, self.hidden_dim)
        return route(x, self.weight, self.top_k, return_probs=True)


class SparseMoeBlock(torch.nn.Module):
    """Drop-in for HF ``Qwen3_5MoeSparseMoeBlock``: ``forward(hidden_states
    [B, S, H]) -> [B, S, H]`` = routed experts + round(sigmoid(gate(x))) *
    shared_expert(x), with the converted INT8 banks
    ``banks = [qg [E, 2I, H], sg, qd [E, H, I], sd]`` and the shared expert as
    three ``(q, scale)`` pairs (gate_proj, up_proj, down_proj)."""

    def __init__(self, router_weight, top_k, banks, shared, shared_gate_weight, activation='w8a8'):
        super().__init__()
        if activation not in ('w8a8', 'w8a16'):
            raise ValueError("activation must be 'w8a8' or 'w8a16'")
        self.gate = TopKRouter(router_weight, top_k)
        for i, t in enumerate(banks):
            self.register_buffer(f'bank{i}', t, persistent=False)
        for i, (q, s) in enumerate(shared):
            self.register_buffer(f'shared_q{i}', q, persistent=False)
            self.register_buffer(f'shared_s{i}', s, persistent=False)
        self.register_buffer('shared_gate_weight', shared_gate_weight.reshape(1, -1), persistent=False)
        self.activation = activation  # decode arithmetic of the routed experts (cli.py:37-39)

    @property
    def banks(self):
        return [self.bank0, self.bank1, self.bank2, self.bank3]

    @property
    def shared(self):
        return [(self.shared_q0, self.shared_s0), (self.shared_q1, self.shared_s1), (self.shared_q2, self.shared_s2)]

    def forward(self, hidden_states, residual=None):
        shape = hidden_states.shape
        x = hidden_states.reshape(-1, shape[-1])
        if x.shape[0] == 0:
            return hidden_states.clone()
        res = residual.reshape(-1, shape[-1]) if residual is not None else None
        if x.shape[0] > 1 and router_gemm_ok(x, self.gate.weight, self.gate.top_k):
            # prefill: router (tensor-core logits + tail + route counts) and experts in one call
            y, _, _ = moe_block_router(x, self.gate.weight, self.gate.top_k, self.banks, shared=self.shared,
                                       shared_gate_weight=self.shared_gate_weight, residual=res)
            return y.reshape(shape)
        w, ids = route(x, self.gate.weight, self.gate.top_k)
        if x.shape[0] == 1:
            y = decode_block(x, w, ids, self.banks, shared=self.shared, shared_gate_weight=self.shared_gate_weight,
                             residual=res, activation=self.activation)
        else:
            y = moe_block(x, w, ids, self.banks, shared=self.shared, shared_gate_weight=self.shared_gate_weight,
                          residual=res)
        return y.reshape(shape)
