"""``ExpertsLoRA``: per-expert LoRA adapters over a frozen ``ExpertsNbit`` base,
drop-in for ``experts4bit_qlora.lora.ExpertsLoRA`` (experts4bit_qlora/lora.py:131-460).

Same parameters (``gate_up_lora_A [E,r,H]``, ``gate_up_lora_B [E,n1,r]``,
``down_lora_A [E,r,I]``, ``down_lora_B [E,H,r]``), initialisation (A ~ N(0, 1/r),
B = 0), delta ``scaling * (x . A^T) . B^T`` added BEFORE the activation, and the
same no-grad decode fast path. The reference's bitsandbytes 4-bit GEMV route
(``lora.py:258-327``) is not reproduced: under ``enable_fast`` the whole layer,
decode included, runs through the fused CUDA path instead.
"""
from __future__ import annotations

import os

import torch
import torch.nn as nn
import torch.nn.functional as F


def _decode_fastpath_enabled() -> bool:
    """``E4B_DECODE_FASTPATH=0`` disables the single-token loop (``lora.py:92-94``)."""
    return os.environ.get("E4B_DECODE_FASTPATH", "1") != "0"


def _epilogue(base, proj):
    """The base's own activation (``lora.py:102-128``): ``_apply_gate`` if the base has one,
    else ``act(gate) * up`` with gate = first half, else ``act(proj)``."""
    hook = getattr(base, "_apply_gate", None)
    if hook is not None:
        out = hook(proj)
        return out if out.dtype == proj.dtype else out.to(proj.dtype)
    if base.has_gate:
        gate, up = proj.chunk(2, dim=-1)
        return base.act_fn(gate) * up
    return base.act_fn(proj)


class ExpertsLoRA(nn.Module):
    def __init__(self, base, r: int = 8, alpha: int = 16, dtype: torch.dtype = torch.float32):
        super().__init__()
        self.base = base
        for p in self.base.parameters():
            p.requires_grad_(False)
        if r < 1:
            raise ValueError(f"ExpertsLoRA needs rank r >= 1, got r={r}; leave B at zero for a no-op adapter")
        self.r = r
        self.scaling = alpha / r
        self._delegate_ok = None
        num_experts = base.num_experts
        gate_up_out, hidden = base._gate_up_shape
        _, intermediate = base._down_shape
        self.gate_up_lora_A = nn.Parameter(torch.empty(num_experts, r, hidden, dtype=dtype))
        self.gate_up_lora_B = nn.Parameter(torch.zeros(num_experts, gate_up_out, r, dtype=dtype))
        self.down_lora_A = nn.Parameter(torch.empty(num_experts, r, intermediate, dtype=dtype))
        self.down_lora_B = nn.Parameter(torch.zeros(num_experts, hidden, r, dtype=dtype))
        nn.init.normal_(self.gate_up_lora_A, std=1.0 / r)
        nn.init.normal_(self.down_lora_A, std=1.0 / r)

    def _delegate_to_base(self) -> bool:
        """Hand the whole forward to the base when an engine ([fast], pipelined or hot
        residency) is attached to it and the adapter is identically zero (``lora.py:181-214``)."""
        if torch.is_grad_enabled() or self.training:
            return False
        base = self.base
        if all(getattr(base, a, None) is None for a in ("_e4b_fast_ref", "_e4b_pipe_ref", "_e4b_hot_ref")):
            return False
        return self._adapter_is_zero()

    def _adapter_is_zero(self) -> bool:
        cached = self._delegate_ok
        if cached is None:
            cached = bool(not self.gate_up_lora_B.any().item() and not self.down_lora_B.any().item())
            self._delegate_ok = cached
        return cached

    def _load_from_state_dict(self, *args, **kwargs):
        self._delegate_ok = None
        return super()._load_from_state_dict(*args, **kwargs)

    def train(self, mode: bool = True):
        self._delegate_ok = None
        return super().train(mode)

    def _lora(self, x, A, B):
        """``lora.py:251-256``: in the adapter dtype, cast back to ``x.dtype``."""
        return (self.scaling * F.linear(F.linear(x.to(A.dtype), A), B)).to(x.dtype)

    def forward(self, hidden_states, top_k_index, top_k_weights):
        base = self.base
        input_dtype = hidden_states.dtype
        compute_dtype = base.compute_dtype if base.compute_dtype is not None else hidden_states.dtype
        hidden_states = hidden_states.to(compute_dtype)
        if self._delegate_to_base():
            return base(hidden_states, top_k_index, top_k_weights).to(input_dtype)
        if (hidden_states.shape[0] == 1 and not torch.is_grad_enabled() and not self.training
                and _decode_fastpath_enabled()):
            return self._forward_decode(hidden_states, top_k_index, top_k_weights, compute_dtype, input_dtype)
        final = torch.zeros_like(hidden_states, dtype=torch.float32)
        with torch.no_grad():
            expert_mask = F.one_hot(top_k_index, num_classes=base.num_experts).permute(2, 1, 0)
            expert_hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero(as_tuple=False).view(-1)
        for expert_idx in expert_hit:
            top_k_pos, token_idx = torch.where(expert_mask[expert_idx])
            x = hidden_states[token_idx]
            proj = base._project(base.gate_up_proj, base.gate_up_absmax, base._gate_up_shape, expert_idx, x,
                                 compute_dtype) + self._lora(x, self.gate_up_lora_A[expert_idx],
                                                             self.gate_up_lora_B[expert_idx])
            cur = _epilogue(base, proj)
            cur = base._project(base.down_proj, base.down_absmax, base._down_shape, expert_idx, cur,
                                compute_dtype) + self._lora(cur, self.down_lora_A[expert_idx],
                                                            self.down_lora_B[expert_idx])
            cur = cur * top_k_weights[token_idx, top_k_pos, None]
            final.index_add_(0, token_idx, cur.to(final.dtype))
        return final.to(input_dtype)

    def _forward_decode(self, hidden_states, top_k_index, top_k_weights, compute_dtype, input_dtype):
        """Single-token no-grad loop over the token's k experts (``lora.py:409-460``)."""
        base = self.base
        final = torch.zeros_like(hidden_states, dtype=torch.float32)
        for j in range(top_k_index.shape[1]):
            e = top_k_index[0, j]
            proj = base._project(base.gate_up_proj, base.gate_up_absmax, base._gate_up_shape, e, hidden_states,
                                 compute_dtype) + self._lora(hidden_states, self.gate_up_lora_A[e],
                                                             self.gate_up_lora_B[e])
            cur = _epilogue(base, proj)
            cur = base._project(base.down_proj, base.down_absmax, base._down_shape, e, cur, compute_dtype) + \
                self._lora(cur, self.down_lora_A[e], self.down_lora_B[e])
            final += (cur * top_k_weights[0, j]).to(final.dtype)
        return final.to(input_dtype)
