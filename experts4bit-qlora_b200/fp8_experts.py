"""``ExpertsFp8Blocks``: fused expert stacks stored as block-scaled FP8 (e4m3).

The storage is DeepSeek's (formats/fp8_blocks.py:1-128 of the reference):
``float8_e4m3fn`` bytes ``[E, out, in]`` with one scale per ``[128, 128]`` tile,
``[E, ceil(out/128), ceil(in/128)]``, either e8m0 exponent bytes (``uint8``,
value ``2**(b-127)``) or fp32 multipliers. The reference decodes such weights
with ``dequantize_fp8_blocks`` and has no fused expert path for them; this
module defines that path with the reference's per-expert loop semantics
(_vendor/experts.py:468-516) over ``dequantize_fp8_blocks`` weights:
``W = bf16(fp32(w) * scale)`` (the scale rounded to bf16 first on 128-aligned
shapes), bf16 matmuls, fp32 accumulation of the weighted expert outputs.

``forward`` is that loop (the fallback and training path); ``enable_fast``
rebinds it to ``e4b_moe_forward`` with ``E4B_FMT_FP8_BLOCK128``, which keeps the
weights at full precision (fp32(w) * scale) and, like the NF4 path, fp16
intermediates: closer to the fp32 result than the loop's bf16 rounding.
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn
import torch.nn.functional as F_nn

from . import ops

BLOCK = 128
E4M3_MAX = 448.0


def scale_values(scale: torch.Tensor) -> torch.Tensor:
    """fp32 multipliers of a scale tensor: e8m0 bytes (uint8/int8) -> ``2**(b-127)``,
    float tensors as they are (``fp8_blocks.py:44-60``)."""
    if scale.dtype in (torch.uint8, torch.int8):
        return torch.exp2((scale.view(torch.uint8).to(torch.int32) - 127).float())
    return scale.float()


def quantize_fp8_blocks(w: torch.Tensor, scale_format: str = "e8m0"):
    """``[..., out, in]`` -> (e4m3 bytes ``uint8 [..., out, in]``, scales ``[..., to, ti]``).

    Per 128x128 tile: ``amax / 448`` as an fp32 scale, or rounded up to a power of two
    and stored as its e8m0 byte. ``w / scale`` then rounds to e4m3 (never above 448)."""
    if scale_format not in ("e8m0", "fp32"):
        raise ValueError("scale_format must be 'e8m0' or 'fp32'")
    *lead, out, inn = w.shape
    to, ti = (out + BLOCK - 1) // BLOCK, (inn + BLOCK - 1) // BLOCK
    wf = w.float()
    pad = torch.zeros(*lead, to * BLOCK, ti * BLOCK, dtype=torch.float32, device=w.device)
    pad[..., :out, :inn] = wf
    amax = pad.view(*lead, to, BLOCK, ti, BLOCK).abs().amax(dim=(-3, -1)).clamp_min(1e-30)
    if scale_format == "e8m0":
        e = torch.ceil(torch.log2(amax / E4M3_MAX)).clamp(-127, 127).to(torch.int32)
        scale = (e + 127).to(torch.uint8)
        sv = torch.exp2(e.float())
    else:
        sv = amax / E4M3_MAX
        scale = sv
    full = sv.repeat_interleave(BLOCK, -2)[..., :out, :].repeat_interleave(BLOCK, -1)[..., :inn]
    q = (wf / full).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    return q.contiguous(), scale.contiguous()


def dequantize_fp8_blocks(w_u8: torch.Tensor, scale: torch.Tensor, dtype=torch.bfloat16) -> torch.Tensor:
    """``[out, in]`` e4m3 bytes + tile scales -> ``dtype`` (formats/fp8_blocks.py:60-128).
    CUDA tensors go through ``e4b_fp8_block_dequantize``; CPU tensors through torch."""
    if w_u8.is_cuda:
        return ops.fp8_block_dequantize(w_u8, scale_values(scale), dtype)
    w = w_u8.view(torch.float8_e4m3fn).float()
    out, inn = w.shape
    s = scale_values(scale)
    if out % BLOCK == 0 and inn % BLOCK == 0:
        s = s.to(dtype).float()
    s = s.repeat_interleave(BLOCK, 0)[:out].repeat_interleave(BLOCK, 1)[:, :inn]
    return (w * s).to(dtype)


class ExpertsFp8Blocks(nn.Module):
    """Block-scaled FP8 expert stacks ``gate_up [E, n1, H]``, ``down [E, H, I]``.

    Parameters: ``gate_up_proj`` / ``down_proj`` (uint8 e4m3 bytes, frozen);
    buffers ``gate_up_scale`` / ``down_scale`` (uint8 e8m0 or fp32). Forward signature
    and output dtype as ``ExpertsNbit``."""

    def __init__(self, num_experts: int, hidden_dim: int, intermediate_dim: int, has_gate: bool = True,
                 activation=None, compute_dtype: Optional[torch.dtype] = torch.bfloat16,
                 scale_dtype: torch.dtype = torch.uint8, device=None):
        super().__init__()
        self.num_experts, self.hidden_dim, self.intermediate_dim = num_experts, hidden_dim, intermediate_dim
        self.has_gate = has_gate
        self.act_fn = activation if activation is not None else F_nn.silu
        self.compute_dtype = compute_dtype
        self.quant_type = "fp8_block128"
        self.bits = 8
        self.block_size = BLOCK
        n1 = 2 * intermediate_dim if has_gate else intermediate_dim
        self._gate_up_shape = (n1, hidden_dim)
        self._down_shape = (hidden_dim, intermediate_dim)
        tiles = lambda o, i: ((o + BLOCK - 1) // BLOCK, (i + BLOCK - 1) // BLOCK)  # noqa: E731
        self.gate_up_proj = nn.Parameter(torch.empty(num_experts, n1, hidden_dim, dtype=torch.uint8, device=device),
                                         requires_grad=False)
        self.down_proj = nn.Parameter(torch.empty(num_experts, hidden_dim, intermediate_dim, dtype=torch.uint8,
                                                  device=device), requires_grad=False)
        self.register_buffer("gate_up_scale", torch.empty(num_experts, *tiles(n1, hidden_dim), dtype=scale_dtype,
                                                          device=device))
        self.register_buffer("down_scale", torch.empty(num_experts, *tiles(hidden_dim, intermediate_dim),
                                                       dtype=scale_dtype, device=device))

    @classmethod
    def from_float(cls, gate_up_proj: torch.Tensor, down_proj: torch.Tensor, has_gate: bool = True,
                   activation=None, compute_dtype=torch.bfloat16, scale_format: str = "e8m0"):
        E, n1, H = gate_up_proj.shape
        I = down_proj.shape[2]
        if down_proj.shape[:2] != (E, H) or n1 != (2 * I if has_gate else I):
            raise ValueError("expected gate_up [E, n1, H] and down [E, H, I] stacks ([E, out, in])")
        gq, gs = quantize_fp8_blocks(gate_up_proj, scale_format)
        dq, ds = quantize_fp8_blocks(down_proj, scale_format)
        m = cls(E, H, I, has_gate, activation, compute_dtype, gs.dtype, device=gate_up_proj.device)
        m.gate_up_proj = nn.Parameter(gq, requires_grad=False)
        m.down_proj = nn.Parameter(dq, requires_grad=False)
        m.gate_up_scale = gs
        m.down_scale = ds
        return m

    @classmethod
    def from_checkpoint(cls, gate_up_w, gate_up_scale, down_w, down_scale, has_gate: bool = True, **kw):
        """From stored tensors: e4m3 weights (float8_e4m3fn or uint8) and their tile scales."""
        E, n1, H = gate_up_w.shape
        I = down_w.shape[2]
        m = cls(E, H, I, has_gate, scale_dtype=gate_up_scale.dtype if gate_up_scale.element_size() != 1
                else torch.uint8, device=gate_up_w.device, **kw)
        as_u8 = lambda t: t.view(torch.uint8) if t.element_size() == 1 else t  # noqa: E731
        m.gate_up_proj = nn.Parameter(as_u8(gate_up_w).contiguous(), requires_grad=False)
        m.down_proj = nn.Parameter(as_u8(down_w).contiguous(), requires_grad=False)
        m.gate_up_scale = as_u8(gate_up_scale).contiguous()
        m.down_scale = as_u8(down_scale).contiguous()
        return m

    def scale_values(self):
        """fp32 multipliers of both scale stacks (what the fused kernels read)."""
        return scale_values(self.gate_up_scale).contiguous(), scale_values(self.down_scale).contiguous()

    def dequantize_expert(self, which: str, e: int, dtype=torch.bfloat16) -> torch.Tensor:
        w = self.gate_up_proj if which == "gate_up" else self.down_proj
        s = self.gate_up_scale if which == "gate_up" else self.down_scale
        return dequantize_fp8_blocks(w[e], s[e], dtype)

    def forward(self, hidden_states: torch.Tensor, top_k_index: torch.Tensor,
                top_k_weights: torch.Tensor) -> torch.Tensor:
        """The per-expert loop (``_vendor/experts.py:468-516``) over dequantized FP8 weights."""
        input_dtype = hidden_states.dtype
        cdt = self.compute_dtype if self.compute_dtype is not None else input_dtype
        hs = hidden_states.to(cdt)
        final = torch.zeros_like(hs, dtype=torch.float32)
        with torch.no_grad():
            mask = F_nn.one_hot(top_k_index, num_classes=self.num_experts).permute(2, 1, 0)
            hit = torch.greater(mask.sum(dim=(-1, -2)), 0).nonzero(as_tuple=False).view(-1)
        for e in hit.tolist():
            pos, tok = torch.where(mask[e])
            x = hs[tok]
            proj = F_nn.linear(x, self.dequantize_expert("gate_up", e, cdt))
            if self.has_gate:
                g, u = proj.chunk(2, dim=-1)
                h = self.act_fn(g) * u
            else:
                h = self.act_fn(proj)
            d = F_nn.linear(h, self.dequantize_expert("down", e, cdt))
            d = d * top_k_weights[tok, pos, None]
            final.index_add_(0, tok, d.to(final.dtype))
        return final.to(input_dtype)

    def extra_repr(self) -> str:
        return (f"num_experts={self.num_experts}, hidden_dim={self.hidden_dim}, "
                f"intermediate_dim={self.intermediate_dim}, has_gate={self.has_gate}, storage=fp8_e4m3 "
                f"block={BLOCK}, scale={self.gate_up_scale.dtype}")
