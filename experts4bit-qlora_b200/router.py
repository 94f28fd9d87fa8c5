"""Fused router (R1): fp32 logits, deterministic top-k and the routing epilogue on the GPU.

``route`` computes what transformers' ``OlmoeTopKRouter`` / ``Qwen3MoeTopKRouter`` /
``MixtralTopKRouter`` compute (``softmax(x . W_r^T)`` in fp32, top-k, optional
renorm), with the reference's deterministic tie rule -- stable descending
order, ties to the lower expert id (experts4bit_qlora/engines/cpu_router.py:100-119) --
and gpt-oss's top-k-then-softmax variant.
"""
from __future__ import annotations

import torch
import torch.nn as nn

from . import _native as N
from . import ops

KINDS = {"softmax_then_topk": N.SOFTMAX_THEN_TOPK, "topk_then_softmax": N.TOPK_THEN_SOFTMAX}


def route(hidden_states: torch.Tensor, router_weight: torch.Tensor, top_k: int,
          kind: str = "softmax_then_topk", norm_topk_prob: bool = False, return_logits: bool = False):
    """Returns ``(top_k_weights f32 [T,k], top_k_index i64 [T,k])`` (plus fp32 logits)."""
    x = hidden_states.reshape(-1, hidden_states.shape[-1])
    if x.dtype not in (torch.bfloat16, torch.float16):
        x = x.to(torch.bfloat16)
    return ops.router_topk(x, router_weight, top_k, KINDS[kind], norm_topk_prob, return_logits)


class TopKRouter(nn.Module):
    """Router module with a ``[E, H]`` weight; ``forward`` returns ``(weights, index)``."""

    def __init__(self, hidden_dim: int, num_experts: int, top_k: int, norm_topk_prob: bool = False,
                 kind: str = "softmax_then_topk", dtype=torch.bfloat16, device=None):
        super().__init__()
        self.top_k, self.num_experts, self.norm_topk_prob, self.kind = top_k, num_experts, norm_topk_prob, kind
        self.weight = nn.Parameter(torch.zeros(num_experts, hidden_dim, dtype=dtype, device=device),
                                   requires_grad=False)

    def forward(self, hidden_states):
        return route(hidden_states, self.weight, self.top_k, self.kind, self.norm_topk_prob)
