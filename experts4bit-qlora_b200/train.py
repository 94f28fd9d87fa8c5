"""``enable_fast_train`` / ``disable_fast_train``: the differentiable expert path of an
``ExpertsLoRA`` layer, drop-in for ``experts4bit_qlora.engines.fast.enable_fast_train``
(experts4bit_qlora/engines/fast.py:453-675).

``enable_fast`` is inference-only (it falls back whenever a gradient is needed); this
patches the ``ExpertsLoRA`` wrapper itself so a training step reaches the library with
gradients on. The composition is the reference's (fast.py:453-552): the frozen NF4
projection and the trainable ``scaling * B(Ax)`` delta are added to the same
pre-activation, then SiLU(gate)*up, then the down projection with its own delta, then
the top-k-weighted scatter in fp32.

Forward: the device permutation (``e4b_permute``) and the grouped NF4 GEMMs
(``e4b_grouped_nf4_gemm``: tcgen05 tiles at prefill sizes) for both frozen
projections; the adapter products per expert.

Backward: the input gradients of the frozen projections, ``dL/dh = dD . W_down`` and
``dL/dx = dP . W_gate_up``, run on the library's dgrad kernel with ``dgrad=True``
(``e4b_grouped_nf4_dgrad``: tcgen05 tiles, each weight tile decoded into shared memory,
nothing materialised), else on one decode of each stack per backward (``e4b_nf4_dequantize``,
freed after the step) and batched GEMMs. The SwiGLU forward and backward, the combine and its
row gradients are single library kernels; the rank-r adapter products and the four adapter
gradients run on the library's segment kernels over the expert-sorted rows (fp32, no padding;
ranks up to 16, larger ranks as batched GEMMs over padded segments).

Numerics: bf16 compute with fp32 adapter math, as ``ExpertsLoRA.forward``; the
frozen projections accumulate in fp32 on fp16 operands (the NF4 value is exact in
fp16), and experts are summed in group-sorted order, so the path matches the
reference loop within the bf16 noise floor, not bit for bit (the reference's
parity contract, tests/test_fused_train_parity.py:46-80).
"""
from __future__ import annotations

import types
from typing import Optional

import torch
import torch.nn.functional as F

from . import _native as N
from . import ops


class _Segments:
    """Expert-sorted rows as a padded batch ``[Ea, L, C]``: active expert i's rows at [i, 0:count)."""

    def __init__(self, offsets_host, R, device):
        counts = [offsets_host[e + 1] - offsets_host[e] for e in range(len(offsets_host) - 1)]
        self.experts = [e for e, c in enumerate(counts) if c > 0]
        self.counts = [counts[e] for e in self.experts]
        self.L = max(self.counts) if self.counts else 0
        self.Ea = len(self.experts)
        # flat padded position of sorted row j: i * L + (j - start_i)
        pos = []
        for i, e in enumerate(self.experts):
            pos.append((i * self.L - offsets_host[e], offsets_host[e], offsets_host[e + 1]))
        shift = torch.zeros(R, dtype=torch.int64)
        for d, a, b in pos:
            shift[a:b] = d
        self.pos = (torch.arange(R, dtype=torch.int64) + shift).to(device, non_blocking=True)
        self.eid = torch.tensor(self.experts, dtype=torch.int64).to(device, non_blocking=True)

    def pad(self, x):
        """``[R, C]`` -> ``[Ea, L, C]`` (padding rows are zero)."""
        out = torch.zeros(self.Ea * self.L, x.shape[1], dtype=x.dtype, device=x.device)
        out.index_copy_(0, self.pos, x)
        return out.view(self.Ea, self.L, -1)

    def unpad(self, xp):
        """``[Ea, L, C]`` -> ``[R, C]`` in row order."""
        return xp.reshape(self.Ea * self.L, -1).index_select(0, self.pos)


class _Adapters:
    """The rank-r adapter products over expert-sorted rows. Ranks up to 16 run on the library's
    segment kernels (fp32, no padding: ``e4b_lora_rank_down`` / ``_rank_up`` / ``_outer``); larger
    ranks as batched GEMMs over the segments padded to the longest."""

    def __init__(self, offs_host, R, dev, rank):
        self.kernels = rank <= 16
        self.rank = rank
        if self.kernels:
            self.tiles = ops.RowTiles(offs_host, dev)
        else:
            self.seg = _Segments(offs_host, R, dev)

    def down_A(self, X, A):
        """``X[row] . A_e^T`` -> [R, r] (A [E, r, K])."""
        E, r, K = A.shape
        if self.kernels:
            return ops.lora_rank_down(X, A, (r * K, K, 1), r, self.tiles)
        s = self.seg
        return s.unpad(torch.bmm(s.pad(X).to(A.dtype), A[s.eid].transpose(1, 2))).float()

    def down_B(self, X, B):
        """``X[row] . B_e`` -> [R, r] (B [E, N, r])."""
        E, Nn, r = B.shape
        if self.kernels:
            return ops.lora_rank_down(X, B, (Nn * r, 1, r), r, self.tiles)
        s = self.seg
        return s.unpad(torch.bmm(s.pad(X).to(B.dtype), B[s.eid])).float()

    def add_up_B(self, Y, B, out, scale):
        """``out[row] += scale * Y[row] . B_e^T`` (B [E, N, r]); 16-bit ``out`` takes the delta
        rounded to its dtype."""
        E, Nn, r = B.shape
        if self.kernels:
            return ops.lora_rank_up(Y, B, (Nn * r, 1, r), Nn, self.tiles, out, scale)
        s = self.seg
        d = s.unpad(scale * torch.bmm(s.pad(Y).to(B.dtype), B[s.eid].transpose(1, 2)))
        return out + (d.to(out.dtype) if out.dtype != torch.float32 else d.float())

    def add_up_A(self, Y, A, out, scale):
        """``out[row] += scale * Y[row] . A_e`` (A [E, r, K], fp32 ``out``)."""
        E, r, K = A.shape
        if self.kernels:
            return ops.lora_rank_up(Y, A, (r * K, K, 1), K, self.tiles, out, scale)
        s = self.seg
        return out + s.unpad(scale * torch.bmm(s.pad(Y).to(A.dtype), A[s.eid])).float()

    def grad_B(self, P, Y, like, scale):
        """dL/dB: ``G_e[n, j] = scale * sum over e's rows of P[row, n] * Y[row, j]`` (like B [E, N, r])."""
        E, Nn, r = like.shape
        if self.kernels:
            G = torch.zeros(E, Nn, r, dtype=torch.float32, device=P.device)
            return ops.lora_outer(P, Y, self.tiles, G, (Nn * r, r, 1), scale).to(like.dtype)
        s = self.seg
        g = scale * torch.bmm(s.pad(P).to(like.dtype).transpose(1, 2), s.pad(Y).to(like.dtype))
        full = torch.zeros_like(like)
        full[s.eid] = g.to(like.dtype)
        return full

    def grad_A(self, Y, P, like, scale):
        """dL/dA: ``G_e[j, k] = scale * sum over e's rows of Y[row, j] * P[row, k]`` (like A [E, r, K])."""
        E, r, K = like.shape
        if self.kernels:
            G = torch.zeros(E, r, K, dtype=torch.float32, device=P.device)
            return ops.lora_outer(P, Y, self.tiles, G, (r * K, 1, K), scale).to(like.dtype)
        s = self.seg
        g = scale * torch.bmm(s.pad(Y).to(like.dtype).transpose(1, 2), s.pad(P).to(like.dtype))
        full = torch.zeros_like(like)
        full[s.eid] = g.to(like.dtype)
        return full


class _FusedExpertsLoRATrain(torch.autograd.Function):
    @staticmethod
    def forward(ctx, hidden, top_k_weights, A_gu, B_gu, A_dn, B_dn, lora_mod, top_k_index):
        base = lora_mod.base
        E, H, I = base.num_experts, base.hidden_dim, base.intermediate_dim
        n1 = 2 * I if base.has_gate else I
        s = float(lora_mod.scaling)
        T, k = top_k_index.shape
        dev = hidden.device
        order, inv, offsets = ops.permute(top_k_index, E)
        order = order.long()
        token_rows = order // k
        offs_host = offsets.tolist()  # one host sync, as the reference's sizes .tolist()
        R = T * k
        ad = _Adapters(offs_host, R, dev, A_gu.shape[1])
        gu_p = base.gate_up_proj.view(E, n1, H // 2)
        gu_a = base.gate_up_absmax.view(E, n1, H // 64)
        dn_p = base.down_proj.view(E, H, I // 2)
        dn_a = base.down_absmax.view(E, H, I // 64)
        x = hidden.index_select(0, token_rows)                       # [R, H] compute dtype
        proj = ops.grouped_nf4_gemm(hidden, gu_p, gu_a, offsets, a_rows=token_rows.to(torch.int32))
        # adapter delta of gate_up in fp32, rounded to the compute dtype and added to the projection
        xa_gu = ad.down_A(x, A_gu)                                    # [R, r] fp32
        proj = ad.add_up_B(xa_gu, B_gu, proj, s)
        h = ops.swiglu_forward(proj, base.has_gate)                   # [R, I], act rounded as lora._epilogue
        down = ops.grouped_nf4_gemm(h.contiguous(), dn_p, dn_a, offsets)
        xa_dn = ad.down_A(h, A_dn)                                    # [R, r] fp32
        down = ad.add_up_B(xa_dn, B_dn, down, s)                      # [R, H] compute dtype
        w_rows = top_k_weights.reshape(-1)[order].float()
        # weighted rows summed per token over its k slots in slot order, fp32 (no atomics)
        out = ops.combine(down, inv, top_k_weights.float(), T, k, torch.float32)
        ctx.lora_mod = lora_mod
        ctx.ad = ad
        ctx.offs_host = offs_host
        ctx.meta = (T, k, E, H, I, n1, s)
        ctx.save_for_backward(token_rows, order, inv, proj, h, down, xa_gu, xa_dn, w_rows, x, A_gu, B_gu, A_dn, B_dn,
                              offsets)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        (token_rows, order, inv, proj, h, down, xa_gu, xa_dn, w_rows, x, A_gu, B_gu, A_dn, B_dn,
         offsets) = ctx.saved_tensors
        lora_mod, ad = ctx.lora_mod, ctx.ad
        base = lora_mod.base
        T, k, E, H, I, n1, s = ctx.meta
        cdt = proj.dtype
        R = T * k
        # dL/d down rows (grad_out[token] * w) and dL/d w_rows (grad_out[token] . down), one pass
        dd, d_w = ops.combine_row_grads(grad_out, token_rows, w_rows, down)
        grad_w = torch.zeros(T * k, dtype=torch.float32, device=grad_out.device)
        grad_w[order] = d_w
        dgrad = getattr(lora_mod, "_e4b_dgrad", False)
        seg = None
        if dgrad and ops.dgrad_eligible(H, I):
            # dL/dh of the frozen down projection on the tensor cores, nothing decoded to memory
            dh = ops.grouped_nf4_dgrad(dd, base.down_proj.view(E, H, I // 2), base.down_absmax.view(E, H, I // 64),
                                       offsets)                         # [R, I] fp32
        else:
            # the frozen stack decoded once for this backward (compute dtype, freed on return)
            seg = _Segments(ctx.offs_host, R, dd.device)
            W_dn = ops.nf4_dequantize(base.down_proj, base.down_absmax, (E, H, I), cdt)
            dh = seg.unpad(torch.bmm(seg.pad(dd), W_dn if seg.Ea == E else W_dn[seg.eid]).float())
            del W_dn
        t_dn = ad.down_B(dd, B_dn)                                      # [R, r] fp32
        gB_dn = ad.grad_B(dd, xa_dn, B_dn, s)                           # [E, H, r]
        gA_dn = ad.grad_A(t_dn, h, A_dn, s)                             # [E, r, I]
        dh = ad.add_up_A(t_dn, A_dn, dh, s)                             # [R, I] fp32
        dproj = ops.swiglu_backward(proj, dh, base.has_gate)            # SiLU(gate) * up, in the compute dtype
        if dgrad and ops.dgrad_eligible(n1, H):
            dx = ops.grouped_nf4_dgrad(dproj, base.gate_up_proj.view(E, n1, H // 2),
                                       base.gate_up_absmax.view(E, n1, H // 64), offsets)  # [R, H] fp32
        else:
            seg = seg or _Segments(ctx.offs_host, R, dd.device)
            W_gu = ops.nf4_dequantize(base.gate_up_proj, base.gate_up_absmax, (E, n1, H), cdt)
            dx = seg.unpad(torch.bmm(seg.pad(dproj), W_gu if seg.Ea == E else W_gu[seg.eid]).float())
            del W_gu
        t_gu = ad.down_B(dproj, B_gu)                                   # [R, r] fp32
        gB_gu = ad.grad_B(dproj, xa_gu, B_gu, s)                        # [E, n1, r]
        gA_gu = ad.grad_A(t_gu, x, A_gu, s)                             # [E, r, H]
        dx = ad.add_up_A(t_gu, A_gu, dx, s)                             # [R, H] fp32
        grad_hidden = ops.combine(dx, inv, None, T, k, torch.float32)  # slot order, no atomics
        return grad_hidden.to(cdt), grad_w.view(T, k), gA_gu, gB_gu, gA_dn, gB_dn, None, None


def fused_experts_train_forward(lora_mod, hidden_states, top_k_index, top_k_weights):
    """Training-capable fused forward of an ``ExpertsLoRA`` (``fast.py:453-552``)."""
    base = lora_mod.base
    input_dtype = hidden_states.dtype
    compute_dtype = base.compute_dtype if base.compute_dtype is not None else input_dtype
    if compute_dtype not in (torch.bfloat16, torch.float16) or not hidden_states.is_cuda:
        return lora_mod._e4b_train_ref(hidden_states, top_k_index, top_k_weights)
    hs = hidden_states.to(compute_dtype).contiguous()
    idx = top_k_index.contiguous().long()
    out = _FusedExpertsLoRATrain.apply(hs, top_k_weights, lora_mod.gate_up_lora_A, lora_mod.gate_up_lora_B,
                                       lora_mod.down_lora_A, lora_mod.down_lora_B, lora_mod, idx)
    return out.to(input_dtype)


def _train_ineligible(mod) -> Optional[str]:
    from .fast import _eligible, _fused_epilogue
    reason = _eligible(mod.base)
    if reason is not None:
        return reason
    if getattr(mod.base, "_e4b_mxfp4_arena", False):
        return "MXFP4 storage has no training path"
    if not _fused_epilogue(mod.base):
        return "the training backward differentiates SiLU(gate)*up only (custom activation or _apply_gate)"
    if getattr(mod.base, "quant_type", None) == "fp8_block128":
        return "FP8 block storage has no training path"
    H, I = mod.base.hidden_dim, mod.base.intermediate_dim
    if H % 64 or I % 64:
        return "hidden and intermediate sizes must be multiples of 64"
    return None


def enable_fast_train(model, verbose: bool = False, dgrad: bool = False) -> int:
    """Route ``ExpertsLoRA`` training through the fused path; returns the patch count
    (``fast.py:555-660``). ``dgrad=True`` takes the input gradients of both frozen projections
    through the library's dgrad kernel (``e4b_grouped_nf4_dgrad``: tcgen05, weights decoded
    tile by tile, nothing materialised), as the reference's option selects its single-launch
    dgrad kernel; ``dgrad=False`` decodes each frozen stack once per backward and runs the
    products as batched GEMMs over the experts' row segments."""
    from .experts import Experts4bit, ExpertsNbit
    from .lora import ExpertsLoRA

    if not N.available():
        if verbose:
            print("[e4b.fast] libe4b.so is not built: no fused training path")
        return 0
    stock = {ExpertsNbit.forward, Experts4bit.forward}
    mods = list(model.modules()) if hasattr(model, "modules") else [model]
    patched = 0
    for mod in mods:
        if not isinstance(mod, ExpertsLoRA):
            continue
        if hasattr(mod, "_e4b_train_ref"):
            if getattr(mod, "_e4b_dgrad", False) != dgrad:
                import warnings
                warnings.warn(
                    f"[e4b.fast] enable_fast_train(dgrad={dgrad}) on a module already patched with "
                    f"dgrad={getattr(mod, '_e4b_dgrad', False)}: the existing patch is kept. Call "
                    "disable_fast_train first to change it.", RuntimeWarning, stacklevel=2)
            continue
        if type(mod.base).forward not in stock and not hasattr(mod.base, "_apply_gate"):
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: base {type(mod.base).__name__} has a custom forward")
            continue
        reason = _train_ineligible(mod)
        if reason is not None:
            if verbose:
                print(f"[e4b.fast] skip {type(mod).__name__}: {reason}")
            continue
        mod._e4b_train_ref = mod.forward
        mod._e4b_dgrad = dgrad
        mod.forward = types.MethodType(
            lambda self, hs, tki, tkw: fused_experts_train_forward(self, hs, tki, tkw), mod)
        patched += 1
    if verbose:
        print(f"[e4b.fast] fused TRAINING path on {patched} ExpertsLoRA module(s)")
    return patched


def disable_fast_train(model) -> int:
    """Undo ``enable_fast_train`` (``fast.py:663-675``); returns the number restored."""
    n = 0
    mods = model.modules() if hasattr(model, "modules") else [model]
    for mod in mods:
        ref = getattr(mod, "_e4b_train_ref", None)
        if ref is not None:
            mod.forward = ref
            del mod._e4b_train_ref
            if hasattr(mod, "_e4b_dgrad"):
                del mod._e4b_dgrad
            n += 1
    return n
