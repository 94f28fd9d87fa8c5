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
