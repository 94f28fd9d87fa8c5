"""MXFP4 expert weights: ``dequantize_mxfp4``, drop-in for
``experts4bit_qlora.formats.mxfp4.dequantize_mxfp4`` (formats/mxfp4.py:35-105).

Blocks ``uint8 [..., rows, G, B]`` hold two e2m1 codes per byte (low nibble first),
scales ``[..., rows, G]`` one e8m0 exponent per block; the result is the dense
``[..., G*2B, rows]`` tensor (trailing pair transposed) the reference returns, bit for
bit. Storage of another dtype label (``int8`` blocks, ``float8_e8m0fnu`` scales) is
reinterpreted as bytes, never value-cast, as the reference does. CUDA tensors go through
``e4b_mxfp4_dequantize``, CPU tensors through ``e4b_mxfp4_dequantize_host``.
"""
from __future__ import annotations

import torch

from . import _native as N
from .experts import ExpertsNbit

FP4_VALUES = (
    0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
    -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0,
)


def dequantize_mxfp4(blocks: torch.Tensor, scales: torch.Tensor, *, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
    if blocks.shape[:-1] != scales.shape:
        raise ValueError(
            f"blocks.shape[:-1]={tuple(blocks.shape[:-1])} != scales.shape={tuple(scales.shape)}")
    if blocks.ndim < 3:
        raise ValueError(
            f"blocks must be [..., rows, G, B] with at least one leading row axis; got {tuple(blocks.shape)}")
    if scales.device != blocks.device:
        raise ValueError(f"scales are on {scales.device} but blocks on {blocks.device}")
    if blocks.dtype != torch.uint8:
        blocks = blocks.view(torch.uint8)
    if scales.dtype != torch.uint8:
        scales = scales.view(torch.uint8)
    *prefix, rows, G, B = blocks.shape
    P = 1
    for d in prefix:
        P *= d
    K = G * 2 * B
    b = blocks.contiguous()
    s = scales.contiguous()
    out = torch.empty(*prefix, K, rows, dtype=dtype, device=blocks.device)
    L = N.lib()
    if blocks.is_cuda:
        N.check(L.e4b_mxfp4_dequantize(b.data_ptr(), s.data_ptr(), P, rows, G, B, out.data_ptr(), N.dtype_code(dtype),
                                       N.stream_handle(blocks.device)), "e4b_mxfp4_dequantize")
    else:
        N.check(L.e4b_mxfp4_dequantize_host(b.data_ptr(), s.data_ptr(), P, rows, G, B, out.data_ptr(),
                                            N.dtype_code(dtype)), "e4b_mxfp4_dequantize_host")
    return out


# --------------------------------------------------------------------------- #
# MXFP4 expert stacks and their fused layer
# --------------------------------------------------------------------------- #
def quantize_mxfp4(w: torch.Tensor):
    """``[..., rows, K]`` (K % 32 == 0) -> (codes ``uint8 [..., rows, K/2]`` low nibble first,
    e8m0 scales ``uint8 [..., rows, K/32]``). Per 32-element block the scale is the smallest power
    of two with ``amax / scale <= 6`` (e8m0 ``s = ceil(log2(amax / 6)) + 127``), and each value
    takes the nearest e2m1 code of ``w / scale`` (ties to the lower code index). For building
    test and benchmark stacks; checkpoints arrive already quantized."""
    *lead, rows, K = w.shape
    if K % 32:
        raise ValueError(f"K ({K}) must be a multiple of 32")
    wf = w.float().reshape(*lead, rows, K // 32, 32)
    amax = wf.abs().amax(-1).clamp_min(1e-38)
    e = torch.ceil(torch.log2(amax / 6.0)).clamp(-127, 127)
    s = (e + 127).to(torch.uint8)
    y = wf / torch.exp2(e)[..., None]
    table = torch.tensor(FP4_VALUES, dtype=torch.float32, device=w.device)
    codes = (y[..., None] - table).abs().argmin(-1).to(torch.uint8)  # first minimum: the lower code
    codes = codes.reshape(*lead, rows, K // 2, 2)
    packed = codes[..., 0] | (codes[..., 1] << 4)
    return packed.contiguous(), s.contiguous()


def _decode_rows(packed: torch.Tensor, scales: torch.Tensor, rows: int, K: int, dtype) -> torch.Tensor:
    """``[rows, K]`` of one expert from its ``[rows*K/2]`` codes and ``[rows*K/32]`` scales
    (``dequantize_mxfp4`` gives ``[K, rows]``; transposed back)."""
    blocks = packed.reshape(rows, K // 32, 16)
    return dequantize_mxfp4(blocks, scales.reshape(rows, K // 32), dtype=dtype).t()


class ExpertsMxfp4(ExpertsNbit):
    """MXFP4 expert stacks with the ``ExpertsNbit`` interface (the reference's MXFP4 arena
    module, engines/nvme_experts.py:700-760): ``gate_up_proj`` / ``down_proj`` hold e2m1 codes
    ``uint8 [E, out*in/2]`` (low nibble first), ``gate_up_absmax`` / ``down_absmax`` the e8m0
    exponents ``uint8 [E, out*in/32]``. ``forward`` is the reference loop over per-expert
    dequantized weights; ``enable_fast`` routes bf16 inference to the fused layer."""

    _ALLOWED_QUANT_TYPES = ("nf4",)

    def __init__(self, num_experts: int, hidden_dim: int, intermediate_dim: int, has_gate: bool = True,
                 activation=None, compute_dtype=torch.bfloat16, device=None):
        if hidden_dim % 32 or intermediate_dim % 32:
            raise ValueError("MXFP4 needs hidden and intermediate sizes divisible by 32")
        super().__init__(num_experts, hidden_dim, intermediate_dim, has_gate=has_gate, activation=activation,
                         compute_dtype=compute_dtype, quant_type="nf4", blocksize=64, device=device)
        n1 = self._gate_up_shape[0]
        self.gate_up_absmax = torch.empty(num_experts, n1 * hidden_dim // 32, dtype=torch.uint8, device=device)
        self.down_absmax = torch.empty(num_experts, hidden_dim * intermediate_dim // 32, dtype=torch.uint8,
                                       device=device)
        self._e4b_mxfp4_arena = True

    @classmethod
    def from_float(cls, gate_up_proj, down_proj, has_gate: bool = True, activation=None,
                   compute_dtype=torch.bfloat16):
        E, n1, H = gate_up_proj.shape
        I = down_proj.shape[2]
        m = cls(E, H, I, has_gate=has_gate, activation=activation, compute_dtype=compute_dtype,
                device=gate_up_proj.device)
        gp, gs = quantize_mxfp4(gate_up_proj)
        dp, ds = quantize_mxfp4(down_proj)
        m.gate_up_proj = torch.nn.Parameter(gp.reshape(E, -1), requires_grad=False)
        m.down_proj = torch.nn.Parameter(dp.reshape(E, -1), requires_grad=False)
        m.gate_up_absmax = gs.reshape(E, -1)
        m.down_absmax = ds.reshape(E, -1)
        return m

    def _dequantize_expert(self, packed, absmax, shape, expert_idx, dtype) -> torch.Tensor:
        rows, K = shape
        return _decode_rows(packed[expert_idx], absmax[expert_idx], rows, K, dtype).to(dtype)
