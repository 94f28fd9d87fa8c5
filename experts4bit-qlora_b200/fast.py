"""``enable_fast`` / ``disable_fast`` / ``fast_available``: drop-in for
``experts4bit_qlora.engines.fast`` (experts4bit_qlora/engines/fast.py:66-423).

Patching semantics are the reference's: the instance ``forward`` of every
eligible ``ExpertsLoRA`` wrapper and bare ``ExpertsNbit`` is rebound, the
original kept on ``_e4b_fast_ref``; a wrapped base is skipped; custom forwards
are skipped unless they expose ``_apply_gate``; the fused forwards fall back
to the stored reference forward exactly where the reference does (grad
required, wrapper in training mode, compute dtype not bf16/fp16, 0-element
storage). The fused forward itself is one ``e4b_moe_forward`` call: device
permutation, grouped NF4 GEMMs with SwiGLU and LoRA fused, deterministic
combine -- no host synchronisation, so it can be captured in a CUDA graph.

The fused kernels' epilogue is SiLU(gate)*up (or SiLU for ``has_gate=False``). A
base with another activation or an ``_apply_gate`` hook (a clamped SwiGLU, say)
takes the epilogue route, as the reference does (engines/fast.py:137-156, :320-347):
the grouped gate_up GEMM without an epilogue, the base's own ``_epilogue`` in
torch, the grouped down GEMM, the fixed-order combine.
"""
from __future__ import annotations

import os
from typing import Optional

import torch

from . import _native
from . import ops

_CHECK = os.environ.get("E4B_CHECK_ERRORS", "0") == "1"


def fast_available() -> bool:
    """True iff libe4b.so loads and CUDA is up (``fast.py:66-72``)."""
    return _native.available() and torch.cuda.is_available()


def _eligible_fp8(mod) -> Optional[str]:
    """Eligibility of an ``ExpertsFp8Blocks`` stack for the fused FP8 path."""
    n1, k1 = mod._gate_up_shape
    n2, k2 = mod._down_shape
    if n1 % 128 or k1 % 128 or n2 % 128 or k2 % 128 or (mod.has_gate and (n1 // 2) % 128):
        return "FP8 dims not multiples of the 128x128 scale tile"
    if mod.num_experts > 1024:
        return "more than 1024 experts"
    if not mod.gate_up_proj.is_cuda:
        return "storage not on CUDA"
    if getattr(mod, "act_fn", None) is not torch.nn.functional.silu:
        return "activation is not SiLU"
    return None


def _eligible_mxfp4(mod) -> Optional[str]:
    """Eligibility of an MXFP4 stack for the fused MXFP4 layer (bf16 tensor-core GEMMs)."""
    if mod.hidden_dim % 128 or mod.intermediate_dim % 128:
        return "MXFP4 dims not multiples of 128"
    if mod.num_experts > 1024:
        return "more than 1024 experts"
    if not mod.gate_up_proj.is_cuda:
        return "storage not on CUDA"
    if not _fused_epilogue(mod):
        return "custom activation: the MXFP4 layer fuses SiLU(gate)*up / SiLU only"
    return None


def _eligible(mod) -> Optional[str]:
    """None if ``mod`` can take the fused path, else the reason (``fast.py:75-97``)."""
    if getattr(mod, "quant_type", None) == "fp8_block128":
        return _eligible_fp8(mod)
    if getattr(mod, "_e4b_mxfp4_arena", False):
        return _eligible_mxfp4(mod)
    if getattr(mod, "bits", None) != 4 or getattr(mod, "quant_type", None) != "nf4":
        return "storage is not nf4-4bit"
    if getattr(mod, "blocksize", None) != 64:
        return f"blocksize {getattr(mod, 'blocksize', None)} != 64"
    n1, k1 = mod._gate_up_shape
    n2, k2 = mod._down_shape
    if k1 % 64 or k2 % 64:
        return "K not divisible by 64"
    if mod.num_experts > 1024:
        return "more than 1024 experts"
    if not mod.gate_up_proj.is_cuda:
        return "storage not on CUDA"
    return None


def _fused_epilogue(base) -> bool:
    """Whether the kernels' own epilogue is the base's: SiLU(gate)*up / SiLU, no hook."""
    return not hasattr(base, "_apply_gate") and getattr(base, "act_fn", None) is torch.nn.functional.silu


def _run_epilogue_route(base, hs, top_k_index, top_k_weights, input_dtype, wrapper=None):
    """The layer for a base whose activation the kernels do not fuse (``fast.py:137-156`` and
    ``:214-257``): device permutation, grouped gate_up GEMM without an epilogue (+ the adapter's
    delta), the base's own ``_epilogue``, grouped down GEMM (+ delta), the fixed-order combine."""
    from .lora import _epilogue
    T, H = hs.shape
    k = top_k_index.shape[1]
    E = base.num_experts
    n1, _ = base._gate_up_shape
    n2, k2 = base._down_shape
    idx = top_k_index.long().contiguous()
    order, inv, offsets = ops.permute(idx, E)
    rows = torch.div(order, k, rounding_mode="floor")  # source token of every expert-sorted row
    up = ops.grouped_nf4_gemm(hs, base.gate_up_proj.view(E, n1, H // 2), base.gate_up_absmax.view(E, n1, H // 64),
                              offsets, a_rows=rows)
    sizes = None
    if wrapper is not None:  # the adapter per expert segment (host sizes, as the reference's loop)
        sizes = (offsets[1:] - offsets[:-1]).tolist()
        a_cat = hs.index_select(0, rows.long())
        off = 0
        for e, n in enumerate(sizes):
            if n:
                up[off:off + n] += wrapper._lora(a_cat[off:off + n], wrapper.gate_up_lora_A[e],
                                                 wrapper.gate_up_lora_B[e])
                off += n
    h = _epilogue(base, up).contiguous()
    down = ops.grouped_nf4_gemm(h, base.down_proj.view(E, n2, k2 // 2), base.down_absmax.view(E, n2, k2 // 64),
                                offsets)
    if wrapper is not None:
        off = 0
        for e, n in enumerate(sizes):
            if n:
                down[off:off + n] += wrapper._lora(h[off:off + n], wrapper.down_lora_A[e], wrapper.down_lora_B[e])
                off += n
    return ops.combine(down, inv, top_k_weights.contiguous(), T, k, out_dtype=input_dtype)


def _grad_needed(mod, hidden_states) -> bool:
    return torch.is_grad_enabled() and (hidden_states.requires_grad
                                        or any(p.requires_grad for p in mod.parameters()))


def _run(base, hidden_states, top_k_index, top_k_weights, compute_dtype, input_dtype, lora=None, wrapper=None):
    hs = hidden_states if hidden_states.dtype == compute_dtype else hidden_states.to(compute_dtype)
    if not _fused_epilogue(base):
        return _run_epilogue_route(base, hs.contiguous(), top_k_index, top_k_weights, input_dtype, wrapper)
    return ops.moe_forward(hs, top_k_index, top_k_weights, base.gate_up_proj, base.gate_up_absmax,
                           base.down_proj, base.down_absmax, base.num_experts, base.intermediate_dim,
                           has_gate=base.has_gate, out_dtype=input_dtype, lora=lora, check_errors=_CHECK)


def fused_experts_forward(mod, hidden_states, top_k_index, top_k_weights):
    """Fused inference forward of a bare ``ExpertsNbit`` (``fast.py:100-160``)."""
    if _grad_needed(mod, hidden_states):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    compute_dtype = mod.compute_dtype if mod.compute_dtype is not None else hidden_states.dtype
    if compute_dtype not in (torch.bfloat16, torch.float16):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    return _run(mod, hidden_states, top_k_index, top_k_weights, compute_dtype, hidden_states.dtype)


def fused_fp8_experts_forward(mod, hidden_states, top_k_index, top_k_weights):
    """Fused inference forward of an ``ExpertsFp8Blocks`` stack (bf16 or fp16 compute)."""
    if _grad_needed(mod, hidden_states):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    compute_dtype = mod.compute_dtype if mod.compute_dtype is not None else hidden_states.dtype
    if compute_dtype not in (torch.bfloat16, torch.float16) or mod.gate_up_proj.numel() == 0:
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    hs = hidden_states if hidden_states.dtype == compute_dtype else hidden_states.to(compute_dtype)
    gs, ds = mod.scale_values()
    return ops.moe_forward(hs, top_k_index, top_k_weights, mod.gate_up_proj, gs, mod.down_proj, ds,
                           mod.num_experts, mod.intermediate_dim, has_gate=mod.has_gate,
                           out_dtype=hidden_states.dtype, check_errors=_CHECK,
                           weight_format=_native.FMT_FP8_BLOCK128)


def fused_mxfp4_experts_forward(mod, hidden_states, top_k_index, top_k_weights):
    """Fused inference forward of MXFP4 stacks (``engines/nvme_experts.py:769-868``): bf16
    compute and no autograd graph, else the module's reference forward."""
    if _grad_needed(mod, hidden_states):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    compute_dtype = mod.compute_dtype if mod.compute_dtype is not None else hidden_states.dtype
    if compute_dtype is not torch.bfloat16 or mod.gate_up_proj.numel() == 0:
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    return ops.moe_forward(hidden_states.to(torch.bfloat16), top_k_index, top_k_weights, mod.gate_up_proj,
                           mod.gate_up_absmax, mod.down_proj, mod.down_absmax, mod.num_experts,
                           mod.intermediate_dim, has_gate=mod.has_gate, out_dtype=hidden_states.dtype,
                           check_errors=_CHECK, weight_format=_native.FMT_MXFP4)


def fused_experts_lora_forward(mod, hidden_states, top_k_index, top_k_weights):
    """Fused inference forward of an ``ExpertsLoRA`` wrapper (``fast.py:163-257``):
    the adapter deltas run inside the grouped GEMMs, before the activation."""
    base = mod.base
    if _grad_needed(mod, hidden_states):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    if mod.training:
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    compute_dtype = base.compute_dtype if base.compute_dtype is not None else hidden_states.dtype
    if compute_dtype not in (torch.bfloat16, torch.float16):
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    if base.gate_up_proj.numel() == 0 or base.down_proj.numel() == 0:
        return mod._e4b_fast_ref(hidden_states, top_k_index, top_k_weights)
    lora = (mod.gate_up_lora_A, mod.gate_up_lora_B, mod.down_lora_A, mod.down_lora_B, mod.scaling)
    return _run(base, hidden_states, top_k_index, top_k_weights, compute_dtype, hidden_states.dtype, lora, mod)


def enable_fast(model, verbose: bool = False) -> int:
    """Patch every eligible module under ``model``; returns the patch count (``fast.py:281-411``)."""
    from .experts import Experts4bit, ExpertsNbit
    from .fp8_experts import ExpertsFp8Blocks
    from .lora import ExpertsLoRA

    stock_forwards = {ExpertsNbit.forward, Experts4bit.forward}
    mods = list(model.modules()) if hasattr(model, "modules") else [model]
    patched = 0
    wrapped_bases = {id(m.base) for m in mods if isinstance(m, ExpertsLoRA)}
    for mod in mods:
        if not isinstance(mod, ExpertsLoRA):
            continue
        if type(mod).forward is not ExpertsLoRA.forward:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: custom forward")
            continue
        reason = _eligible(mod.base)
        if reason is None and getattr(mod.base, "_e4b_mxfp4_arena", False):
            reason = "MXFP4 base: the fused MXFP4 layer takes no adapters"
        if reason is not None:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: {reason}")
            continue
        if type(mod.base).forward not in stock_forwards and not hasattr(mod.base, "_apply_gate"):
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: base {type(mod.base).__name__} has a custom forward")
            continue
        if hasattr(mod, "_e4b_fast_ref"):
            continue
        mod._e4b_fast_ref = mod.forward
        mod.forward = fused_experts_lora_forward.__get__(mod)
        patched += 1
    for mod in mods:
        if not isinstance(mod, ExpertsFp8Blocks) or type(mod).forward is not ExpertsFp8Blocks.forward:
            continue
        reason = _eligible(mod)
        if reason is not None:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: {reason}")
            continue
        if hasattr(mod, "_e4b_fast_ref"):
            continue
        mod._e4b_fast_ref = mod.forward
        mod.forward = fused_fp8_experts_forward.__get__(mod)
        patched += 1
    for mod in mods:
        if not isinstance(mod, ExpertsNbit):
            continue
        if id(mod) in wrapped_bases:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: wrapped by a patched ExpertsLoRA "
                      "(its forward is never called)")
            continue
        if type(mod).forward not in stock_forwards and not hasattr(mod, "_apply_gate"):
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: custom forward")
            continue
        reason = _eligible(mod)
        if reason is not None:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: {reason}")
            continue
        for attr, what in (("_hot_residency", "hot_residency"), ("_e4b_cold_ref", "cold engine"),
                           ("_e4b_pipe_ref", "pipelined residency"), ("_e4b_mxfp4_ref", "mxfp4 NVMe residency")):
            if hasattr(mod, attr):
                if verbose:
                    print(f"[e4b.fast] skip {type(mod).__name__}: {what} enabled — disable it first")
                break
        else:
            if hasattr(mod, "_e4b_fast_ref"):
                continue
            mod._e4b_fast_ref = mod.forward
            fwd = fused_mxfp4_experts_forward if getattr(mod, "_e4b_mxfp4_arena", False) else fused_experts_forward
            mod.forward = fwd.__get__(mod)
            patched += 1
    if patched and getattr(model, "training", False):
        import warnings
        warnings.warn(
            f"[e4b.fast] model is in TRAINING mode: fused_experts_lora_forward falls back to the reference "
            f"path while `training` is set, so all {patched} patch(es) will be bypassed. Call model.eval() "
            "before inference.", RuntimeWarning, stacklevel=2)
    return patched


def disable_fast(model) -> int:
    """Undo ``enable_fast``; returns the number of modules restored (``fast.py:414-423``)."""
    mods = model.modules() if hasattr(model, "modules") else [model]
    restored = 0
    for mod in mods:
        if hasattr(mod, "_e4b_fast_ref"):
            mod.forward = mod._e4b_fast_ref
            del mod._e4b_fast_ref
            restored += 1
    _native.check_errors()  # a device error the fused calls recorded surfaces here at the latest
    return restored
