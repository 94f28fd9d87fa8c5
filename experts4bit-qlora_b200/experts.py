"""``ExpertsNbit`` / ``Experts4bit``: the fused-expert storage module, drop-in for
``experts4bit_qlora._vendor.experts`` (experts4bit_qlora/_vendor/experts.py:123-530).

Same constructor, ``from_float``, parameter/buffer names and shapes, and
``_extra_state`` schema 1, so reference checkpoints load unchanged. The NF4
codec is this library's (``e4b_nf4_quantize`` / ``e4b_nf4_dequantize``), not
bitsandbytes'. ``forward`` is the reference's per-expert dequantize-then-linear
loop (the semantics ``enable_fast`` falls back to, and the training path);
``enable_fast`` rebinds it to the fused CUDA layer.

Storage schemes built here: ``nf4`` and the 16-bit passthroughs ``bf16`` /
``fp16``. The reference's other codebooks (``fp4``, ``int8``, ``fp8``) are
accepted as names but refused at construction.
"""
from __future__ import annotations

import functools
from collections.abc import Callable
from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F_nn

from . import ops

_SCHEME_BITS = {"nf4": 4, "fp4": 4, "int8": 8, "fp8": 8, "bf16": 16, "fp16": 16}
_PASSTHROUGH_DTYPES = {"bf16": torch.bfloat16, "fp16": torch.float16}
_BUILT_SCHEMES = ("nf4", "bf16", "fp16")
_EXTRA_STATE_SCHEMA = 1
_QUANT_TYPE_ALIASES = {"bfloat16": "bf16", "float16": "fp16"}

# The 16 NF4 values (QLoRA, arXiv:2305.14314, Appendix E).
NF4_CODE = (
    -1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
    -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
    0.07958029955625534, 0.16093020141124725, 0.24611230194568634, 0.33791524171829224,
    0.44070982933044434, 0.5626170039176941, 0.7229568362236023, 1.0,
)


def normalize_quant_type(quant_type, allowed: tuple = tuple(_SCHEME_BITS)) -> str:
    """Canonical scheme name (``_vendor/experts.py:42-58``): case/whitespace-insensitive,
    ``bfloat16``/``float16`` aliases. Raises ``ValueError`` naming the allowed set."""
    if not isinstance(quant_type, str):
        raise ValueError(f"quant_type must be one of {allowed}, got {type(quant_type).__name__}")
    q = quant_type.strip().lower()
    q = _QUANT_TYPE_ALIASES.get(q, q)
    if q not in allowed:
        hint = f" (normalized from {quant_type!r})" if q != quant_type else ""
        raise ValueError(f"quant_type must be one of {allowed}, got {q!r}{hint}")
    return q


def _build_code(quant_type: str, device) -> Optional[torch.Tensor]:
    if quant_type == "nf4":
        return torch.tensor(NF4_CODE, dtype=torch.float32, device=device if device is not None else "cpu")
    return None


class _FrozenLinearRecomputeBackward(torch.autograd.Function):
    """``F.linear`` against a frozen dequantized weight that is re-dequantized in
    backward instead of being saved (``_vendor/experts.py:80-120``)."""

    @staticmethod
    def forward(ctx, x, dequant_fn):
        ctx.dequant_fn = dequant_fn
        return F_nn.linear(x, dequant_fn())

    @staticmethod
    def backward(ctx, grad_output):
        grad_x = None
        if ctx.needs_input_grad[0]:
            try:
                weight = ctx.dequant_fn()
            except Exception as e:
                packed = ctx.dequant_fn.args[0] if getattr(ctx.dequant_fn, "args", None) else None
                if isinstance(packed, torch.Tensor) and packed.numel() == 0:
                    raise RuntimeError(
                        "backward re-dequantization read an evicted expert (0-element placeholder); "
                        "the packed storage must be resident when backward runs") from e
                raise
            grad_x = grad_output @ weight
        return grad_x, None


class ExpertsNbit(nn.Module):
    """Low-bit storage for fused MoE expert weights ``[E, out, in]``.

    Args mirror the reference: ``num_experts, hidden_dim, intermediate_dim,
    has_gate=True, activation=None (SiLU), compute_dtype=None, quant_type="nf4",
    blocksize=64, device=None``.
    """

    _ALLOWED_QUANT_TYPES: tuple = tuple(_SCHEME_BITS)
    _EXTRA_STATE_FIELDS = ("quant_type", "blocksize", "has_gate", "num_experts", "hidden_dim", "intermediate_dim")

    def __init__(self, num_experts: int, hidden_dim: int, intermediate_dim: int, has_gate: bool = True,
                 activation: Optional[Callable[[torch.Tensor], torch.Tensor]] = None,
                 compute_dtype: Optional[torch.dtype] = None, quant_type: str = "nf4", blocksize: int = 64,
                 device=None):
        super().__init__()
        quant_type = normalize_quant_type(quant_type, allowed=type(self)._ALLOWED_QUANT_TYPES)
        if quant_type not in _BUILT_SCHEMES:
            raise NotImplementedError(
                f"quant_type {quant_type!r} is not built in experts4bit-b200; its storage schemes are "
                f"{_BUILT_SCHEMES}")
        self.bits = _SCHEME_BITS[quant_type]
        if self.bits < 16:
            if blocksize != 64:
                raise NotImplementedError("experts4bit-b200 builds NF4 with blocksize 64 only")
            for name, in_features in (("hidden_dim", hidden_dim), ("intermediate_dim", intermediate_dim)):
                if in_features % blocksize != 0:
                    raise ValueError(
                        f"{name} ({in_features}) must be divisible by blocksize ({blocksize}) "
                        "so per-expert quantization blocks align with expert boundaries")
        self.num_experts = num_experts
        self.hidden_dim = hidden_dim
        self.intermediate_dim = intermediate_dim
        self.has_gate = has_gate
        self.act_fn = activation if activation is not None else F_nn.silu
        self.compute_dtype = compute_dtype
        self.quant_type = quant_type
        self.blocksize = blocksize
        gate_up_out = 2 * intermediate_dim if has_gate else intermediate_dim
        self._gate_up_shape = (gate_up_out, hidden_dim)
        self._down_shape = (hidden_dim, intermediate_dim)
        gate_up_numel = gate_up_out * hidden_dim
        down_numel = hidden_dim * intermediate_dim
        if self.bits == 16:
            sd = _PASSTHROUGH_DTYPES[quant_type]
            gu = torch.empty(num_experts, gate_up_numel, dtype=sd, device=device)
            dn = torch.empty(num_experts, down_numel, dtype=sd, device=device)
        else:
            gu = torch.empty(num_experts, gate_up_numel // 2, dtype=torch.uint8, device=device)
            dn = torch.empty(num_experts, down_numel // 2, dtype=torch.uint8, device=device)
        self.gate_up_proj = nn.Parameter(gu, requires_grad=False)
        self.down_proj = nn.Parameter(dn, requires_grad=False)
        if self.bits < 16:
            self.register_buffer("gate_up_absmax", torch.empty(num_experts, gate_up_numel // blocksize,
                                                               dtype=torch.float32, device=device))
            self.register_buffer("down_absmax", torch.empty(num_experts, down_numel // blocksize,
                                                            dtype=torch.float32, device=device))
        else:
            self.register_buffer("gate_up_absmax", None)
            self.register_buffer("down_absmax", None)
        self.register_buffer("code", _build_code(quant_type, device), persistent=False)

    # -- checkpoint metadata (_vendor/experts.py:280-327) ----------------------
    def get_extra_state(self) -> dict:
        state = {"schema": _EXTRA_STATE_SCHEMA}
        state.update({k: getattr(self, k) for k in self._EXTRA_STATE_FIELDS})
        return state

    def set_extra_state(self, state) -> None:
        if state is None:
            return
        if not isinstance(state, dict) or not isinstance(state.get("schema"), int):
            raise ValueError(f"unrecognized ExpertsNbit extra state: {type(state).__name__}")
        if state["schema"] > _EXTRA_STATE_SCHEMA:
            raise ValueError(f"checkpoint carries ExpertsNbit metadata schema {state['schema']}; this build "
                             f"understands <= {_EXTRA_STATE_SCHEMA}")
        bad = {k: (state[k], getattr(self, k)) for k in self._EXTRA_STATE_FIELDS
               if k in state and state[k] != getattr(self, k)}
        if bad:
            detail = ", ".join(f"{k}: checkpoint={c!r} vs module={m!r}" for k, (c, m) in bad.items())
            raise ValueError("checkpoint/module config mismatch — re-instantiate the module with the "
                             f"checkpoint's construction arguments ({detail})")

    def _load_from_state_dict(self, state_dict, prefix, *args, **kwargs):
        state_dict.setdefault(prefix + "_extra_state", None)
        super()._load_from_state_dict(state_dict, prefix, *args, **kwargs)

    # -- construction ----------------------------------------------------------
    @classmethod
    def from_float(cls, gate_up_proj: torch.Tensor, down_proj: torch.Tensor, has_gate: bool = True,
                   activation=None, compute_dtype=None, quant_type: str = "nf4", blocksize: int = 64):
        """Quantize full-precision stacks ``gate_up [E, n1, H]`` and ``down [E, H, I]``
        (``_vendor/experts.py:329-396``) on their own device."""
        if gate_up_proj.dim() != 3 or down_proj.dim() != 3:
            raise ValueError("gate_up_proj and down_proj must be 3D [num_experts, out, in] tensors")
        num_experts, gate_up_out, hidden_dim = gate_up_proj.shape
        intermediate_dim = down_proj.shape[2]
        expected = 2 * intermediate_dim if has_gate else intermediate_dim
        if down_proj.shape[0] != num_experts or down_proj.shape[1] != hidden_dim or gate_up_out != expected:
            raise ValueError(
                f"inconsistent expert stacks for has_gate={has_gate}: expected gate_up_proj "
                f"[num_experts, {'2*intermediate' if has_gate else 'intermediate'}, hidden] and "
                f"down_proj [num_experts, hidden, intermediate] (layout [num_experts, out, in]), "
                f"got gate_up_proj {tuple(gate_up_proj.shape)} vs down_proj {tuple(down_proj.shape)} "
                "— is one of them transposed / stored [num_experts, in, out]?")
        module = cls(num_experts, hidden_dim, intermediate_dim, has_gate=has_gate, activation=activation,
                     compute_dtype=compute_dtype if compute_dtype is not None else gate_up_proj.dtype,
                     quant_type=quant_type, blocksize=blocksize, device=gate_up_proj.device)
        gp, ga = module._quantize_stack(gate_up_proj)
        dp, da = module._quantize_stack(down_proj)
        module.gate_up_proj = nn.Parameter(gp, requires_grad=False)
        module.down_proj = nn.Parameter(dp, requires_grad=False)
        module.gate_up_absmax = ga
        module.down_absmax = da
        return module

    def _quantize_stack(self, weights: torch.Tensor):
        """Whole-stack quantization: blocks never straddle experts, so this equals the
        reference's per-expert loop (``_vendor/experts.py:398-426``) byte for byte."""
        E = weights.shape[0]
        if self.bits == 16:
            return weights.reshape(E, -1).to(_PASSTHROUGH_DTYPES[self.quant_type]).contiguous(), None
        packed, absmax = ops.nf4_quantize(weights.reshape(E, -1), self.blocksize)
        return packed.view(E, -1), absmax.view(E, -1)

    def _dequantize_expert(self, packed, absmax, shape, expert_idx, dtype) -> torch.Tensor:
        """One expert ``[out, in]`` in ``dtype`` (``_vendor/experts.py:428-457``)."""
        if self.bits == 16:
            return packed[expert_idx].reshape(shape).to(dtype)
        return ops.nf4_dequantize(packed[expert_idx], absmax[expert_idx], shape, dtype)

    def _project(self, packed, absmax, shape, expert_idx, x, compute_dtype):
        dequant_fn = functools.partial(self._dequantize_expert, packed, absmax, shape, expert_idx, compute_dtype)
        return _FrozenLinearRecomputeBackward.apply(x, dequant_fn)

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        """The reference per-expert loop (``_vendor/experts.py:468-516``)."""
        input_dtype = hidden_states.dtype
        compute_dtype = self.compute_dtype if self.compute_dtype is not None else hidden_states.dtype
        hidden_states = hidden_states.to(compute_dtype)
        final_hidden_states = torch.zeros_like(hidden_states, dtype=torch.float32)
        with torch.no_grad():
            expert_mask = F_nn.one_hot(top_k_index, num_classes=self.num_experts).permute(2, 1, 0)
            expert_hit = torch.greater(expert_mask.sum(dim=(-1, -2)), 0).nonzero(as_tuple=False).view(-1)
        for expert_idx in expert_hit:
            top_k_pos, token_idx = torch.where(expert_mask[expert_idx])
            current_state = hidden_states[token_idx]
            proj = self._project(self.gate_up_proj, self.gate_up_absmax, self._gate_up_shape, expert_idx,
                                 current_state, compute_dtype)
            if self.has_gate:
                gate, up = proj.chunk(2, dim=-1)
                current_hidden = self.act_fn(gate) * up
            else:
                current_hidden = self.act_fn(proj)
            current_hidden = self._project(self.down_proj, self.down_absmax, self._down_shape, expert_idx,
                                           current_hidden, compute_dtype)
            current_hidden = current_hidden * top_k_weights[token_idx, top_k_pos, None]
            final_hidden_states.index_add_(0, token_idx, current_hidden.to(final_hidden_states.dtype))
        return final_hidden_states.to(input_dtype)


class Experts4bit(ExpertsNbit):
    """The fixed-4-bit specialization (``_vendor/experts.py:519-530``)."""

    _ALLOWED_QUANT_TYPES = ("nf4", "fp4")
