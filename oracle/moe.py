"""CPU restatement of the reference's fused-expert forward (test infrastructure only).

Every function cites the reference code it restates (paths relative to the
experts4bit-qlora project root). All of it runs on CPU with torch/numpy.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from .nf4 import dequantize_nf4, dequantize_nf4_f32

SOFTMAX_THEN_TOPK = "softmax_then_topk"   # OLMoE / Qwen3-MoE / Mixtral
TOPK_THEN_SOFTMAX = "topk_then_softmax"   # gpt-oss


# --------------------------------------------------------------------------- #
# Storage helpers
# --------------------------------------------------------------------------- #
def dequant_expert(packed, absmax, e, shape, dtype=torch.bfloat16, blocksize=64):
    """``ExpertsNbit._dequantize_expert`` for NF4 (``_vendor/experts.py:428-457``)."""
    return dequantize_nf4(packed[e].numpy(), absmax[e].numpy(), shape, dtype, blocksize)


def dequant_stack_f32(packed, absmax, shape, blocksize=64):
    """Whole-stack fp32 dequant ``[E, out, in]``; equals per-expert dequant
    (``tests/test_fused_train_parity.py:227-281`` pins this identity)."""
    E = packed.shape[0]
    f = dequantize_nf4_f32(packed.numpy().reshape(-1), absmax.numpy().reshape(-1), blocksize)
    return torch.from_numpy(f).reshape(E, *shape)


# --------------------------------------------------------------------------- #
# Router (engines/cpu_router.py:100-119; transformers OlmoeTopKRouter.forward)
# --------------------------------------------------------------------------- #
def router_logits_f32(x, router_weight):
    """fp32 logits ``x . W_r^T`` with fp32 inputs and accumulation. ``router_weight`` is ``[E, H]``."""
    return x.float() @ router_weight.float().t()


def deterministic_topk(logits32, k):
    """Stable descending sort, ties to the LOWER expert id (``cpu_router.py:100-104``)."""
    vals, idx = torch.sort(logits32, dim=-1, descending=True, stable=True)
    return vals[:, :k], idx[:, :k]


def route_on_host(logits32, k, kind=SOFTMAX_THEN_TOPK, norm_topk_prob=False):
    """Routing epilogue (``cpu_router.py:107-119``): returns (weights fp32 [T,k], idx i64 [T,k])."""
    top_logits, top_idx = deterministic_topk(logits32, k)
    if kind == SOFTMAX_THEN_TOPK:
        probs = torch.softmax(logits32, dim=-1)
        w = probs.gather(-1, top_idx)
        if norm_topk_prob:
            w = w / w.sum(dim=-1, keepdim=True)
    else:
        w = torch.softmax(top_logits, dim=-1)
    return w, top_idx


# --------------------------------------------------------------------------- #
# Permutation and combine of the fused driver (engines/fast.py)
# --------------------------------------------------------------------------- #
def permute(top_k_index, num_experts):
    """``fast.py:126-133``: stable expert-major order of the flat (token, slot) pairs.

    Returns ``order, token_rows, top_pos, counts, offsets`` (offsets has E+1 entries).
    """
    k = top_k_index.shape[1]
    flat = top_k_index.reshape(-1).long()
    order = torch.argsort(flat, stable=True)
    token_rows = order // k
    top_pos = order - token_rows * k
    counts = torch.bincount(flat, minlength=num_experts)
    offsets = torch.zeros(num_experts + 1, dtype=torch.long)
    offsets[1:] = torch.cumsum(counts, 0)
    return order, token_rows, top_pos, counts, offsets


def scatter_combine(down, w_sorted, order, tokens, k, out_dtype):
    """``fast.py:260-278``: unique writes into ``[T*k, H]`` fp32, then a fixed-order k-sum."""
    hidden = down.shape[1]
    buf = torch.zeros(tokens * k, hidden, dtype=torch.float32)
    buf[order] = down.to(torch.float32) * w_sorted[:, None]
    return buf.view(tokens, k, hidden).sum(1).to(out_dtype)


# --------------------------------------------------------------------------- #
# The reference per-expert loop (_vendor/experts.py:468-516) and its LoRA
# wrapper (lora.py:329-407), in the reference's own dtypes.
# --------------------------------------------------------------------------- #
def _epilogue(proj, has_gate=True):
    """``lora.py:125-128``: ``silu(gate) * up`` with gate = first half."""
    if has_gate:
        gate, up = proj.chunk(2, dim=-1)
        return F.silu(gate) * up
    return F.silu(proj)


def _lora(x, A, B, scaling):
    """``lora.py:251-256``: ``scaling * ((x . A^T) . B^T)`` in the adapter dtype, cast back."""
    return (scaling * F.linear(F.linear(x.to(A.dtype), A), B)).to(x.dtype)


def reference_forward(st, hidden_states, top_k_index, top_k_weights, compute_dtype=None, lora=None):
    """The reference loop over hit experts.

    ``st`` is a dict with ``gate_up_packed, gate_up_absmax, down_packed,
    down_absmax, E, H, I, has_gate``. ``lora`` (optional) is a dict with
    ``gate_up_A, gate_up_B, down_A, down_B, scaling``. Without ``lora`` this
    restates ``ExpertsNbit.forward``; with it, ``ExpertsLoRA.forward``'s mask
    path (which has the same summation order).
    """
    E, H, I, has_gate = st["E"], st["H"], st["I"], st.get("has_gate", True)
    gu_shape = (2 * I if has_gate else I, H)
    dn_shape = (H, I)
    input_dtype = hidden_states.dtype
    cdt = compute_dtype if compute_dtype is not None else input_dtype
    hs = hidden_states.to(cdt)
    final = torch.zeros_like(hs, dtype=torch.float32)
    with torch.no_grad():
        mask = F.one_hot(top_k_index.long(), num_classes=E).permute(2, 1, 0)
        hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero(as_tuple=False).view(-1)
        for e in hit.tolist():
            pos, tok = torch.where(mask[e])
            x = hs[tok]
            w_gu = expert_weight(st, "gate_up", e, cdt)
            proj = F.linear(x, w_gu)
            if lora is not None:
                proj = proj + _lora(x, lora["gate_up_A"][e], lora["gate_up_B"][e], lora["scaling"])
            h = _epilogue(proj, has_gate)
            w_dn = expert_weight(st, "down", e, cdt)
            d = F.linear(h, w_dn)
            if lora is not None:
                d = d + _lora(h, lora["down_A"][e], lora["down_B"][e], lora["scaling"])
            d = d * top_k_weights[tok, pos, None]
            final.index_add_(0, tok, d.to(final.dtype))
    return final.to(input_dtype)


def fp32_oracle(st, hidden_states, top_k_index, top_k_weights, lora=None, w_cache=None):
    """fp32 forward over the same dequantized NF4 values (``tests/test_fast.py:49-68``),
    optionally with the LoRA deltas in fp32. Returns fp32 ``[T, H]``.

    ``w_cache`` (optional dict) memoises the fp32 dequantized stacks across calls.
    """
    E, H, I, has_gate = st["E"], st["H"], st["I"], st.get("has_gate", True)
    gu_shape = (2 * I if has_gate else I, H)
    dn_shape = (H, I)
    if w_cache is not None and "gu" in w_cache:
        W_gu, W_dn = w_cache["gu"], w_cache["dn"]
    elif st.get("format", "nf4") == "fp8":
        W_gu = torch.stack([expert_weight(st, "gate_up", e, torch.float32) for e in range(E)])
        W_dn = torch.stack([expert_weight(st, "down", e, torch.float32) for e in range(E)])
        if w_cache is not None:
            w_cache["gu"], w_cache["dn"] = W_gu, W_dn
    else:
        W_gu = dequant_stack_f32(st["gate_up_packed"], st["gate_up_absmax"], gu_shape)
        W_dn = dequant_stack_f32(st["down_packed"], st["down_absmax"], dn_shape)
        if w_cache is not None:
            w_cache["gu"], w_cache["dn"] = W_gu, W_dn
    x = hidden_states.float()
    out = torch.zeros(x.shape[0], H, dtype=torch.float32)
    idx = top_k_index.long()
    for e in range(E):
        tok, pos = torch.where(idx == e)
        if not len(tok):
            continue
        h = x[tok] @ W_gu[e].t()
        if lora is not None:
            s = lora["scaling"]
            h = h + s * ((x[tok] @ lora["gate_up_A"][e].float().t()) @ lora["gate_up_B"][e].float().t())
        h = _epilogue(h, has_gate)
        d = h @ W_dn[e].t()
        if lora is not None:
            d = d + s * ((h @ lora["down_A"][e].float().t()) @ lora["down_B"][e].float().t())
        out.index_add_(0, tok, d * top_k_weights[tok, pos, None].float())
    return out


def fused_driver_forward(st, hidden_states, top_k_index, top_k_weights, compute_dtype=torch.bfloat16, lora=None):
    """``fast.py:100-160`` / ``:163-257`` with the grouped GEMM restated as a
    per-segment bf16 dequant-matmul. Pins the permutation and combine semantics."""
    E, H, I, has_gate = st["E"], st["H"], st["I"], st.get("has_gate", True)
    gu_shape = (2 * I if has_gate else I, H)
    dn_shape = (H, I)
    input_dtype = hidden_states.dtype
    hs = hidden_states.to(compute_dtype)
    T, k = top_k_index.shape
    order, token_rows, top_pos, counts, offsets = permute(top_k_index, E)
    a_cat = hs.index_select(0, token_rows)
    up = torch.empty(a_cat.shape[0], gu_shape[0], dtype=compute_dtype)
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            w = dequant_expert(st["gate_up_packed"], st["gate_up_absmax"], e, gu_shape, torch.float32)
            up[lo:hi] = (a_cat[lo:hi].float() @ w.t()).to(compute_dtype)
            if lora is not None:
                up[lo:hi] += _lora(a_cat[lo:hi], lora["gate_up_A"][e], lora["gate_up_B"][e], lora["scaling"])
    h = _epilogue(up, has_gate).contiguous()
    down = torch.empty(a_cat.shape[0], H, dtype=compute_dtype)
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        if hi > lo:
            w = dequant_expert(st["down_packed"], st["down_absmax"], e, dn_shape, torch.float32)
            down[lo:hi] = (h[lo:hi].float() @ w.t()).to(compute_dtype)
            if lora is not None:
                down[lo:hi] += _lora(h[lo:hi], lora["down_A"][e], lora["down_B"][e], lora["scaling"])
    w = top_k_weights[token_rows, top_pos].to(torch.float32)
    return scatter_combine(down, w, order, T, k, input_dtype)


# --------------------------------------------------------------------------- #
# FP8 e4m3 with 128x128 block scales (formats/fp8_blocks.py:60-128)
# --------------------------------------------------------------------------- #
def fp8_scale_values(scale):
    """e8m0 bytes -> fp32 multipliers ``2**(b-127)`` (``fp8_blocks.py:44-60``, ``_scale_values``);
    a float tensor already holds the values."""
    scale = torch.as_tensor(scale)
    if scale.dtype in (torch.uint8, torch.int8):
        return torch.exp2((scale.view(torch.uint8).to(torch.int32) - 127).float())
    return scale.float()


def fp8_block_dequant(weight_u8, scale, block=128, dtype=torch.bfloat16):
    """``dequantize_fp8_blocks`` (``fp8_blocks.py:60-128``). Aligned shapes
    (``:104-121``): ``bf16(e4m3) * bf16(scale)`` in ``dtype``, i.e. the scale rounded to
    ``dtype`` and one rounding of the product; ragged shapes (``:126-127``):
    ``(fp32(e4m3) * scale).to(dtype)``."""
    w = torch.as_tensor(weight_u8).view(torch.float8_e4m3fn).float()
    out, inn = w.shape
    s = fp8_scale_values(scale)
    if out % block == 0 and inn % block == 0:
        s = s.to(dtype).float()
    s = s.repeat_interleave(block, 0)[:out].repeat_interleave(block, 1)[:, :inn]
    return (w * s).to(dtype)


def expert_weight(st, which, e, dtype):
    """Dequantized ``[out, in]`` weight of expert ``e`` (``which`` = "gate_up" | "down") of a
    stack dict: NF4 (``format`` absent or "nf4") or FP8 blocks (``format`` == "fp8")."""
    E, H, I, has_gate = st["E"], st["H"], st["I"], st.get("has_gate", True)
    shape = ((2 * I if has_gate else I), H) if which == "gate_up" else (H, I)
    if st.get("format", "nf4") == "fp8":
        return fp8_block_dequant(st[which + "_w"][e].reshape(shape), st[which + "_scale"][e], dtype=dtype)
    return dequant_expert(st[which + "_packed"], st[which + "_absmax"], e, shape, dtype)


def rel_errors(got, ref):
    """(max-abs-diff / max|ref|, mean|diff| / mean|ref|): the norm-relative metrics the
    parity tests use (``tests/test_fast.py:43-46`` for the max form)."""
    g, r = got.float(), ref.float()
    d = (g - r).abs()
    return (d.max() / r.abs().max().clamp_min(1e-30)).item(), (d.mean() / r.abs().mean().clamp_min(1e-30)).item()


def np_bf16(x):
    """bf16 tensor -> numpy uint16 view (for fixtures)."""
    return x.contiguous().view(torch.int16).numpy().view(np.uint16)
