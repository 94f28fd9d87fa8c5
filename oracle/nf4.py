"""NF4 codec restated for the oracle (test infrastructure only).

Follows the reference's use of bitsandbytes:
* ``experts4bit_qlora/_vendor/experts.py:408-426`` -- per expert,
  ``quantize_4bit(w[e], blocksize=64, compress_statistics=False, quant_type="nf4")``;
  packed bytes flattened to ``[E, out*in/2]``, absmax to ``[E, out*in/64]`` fp32.
* ``experts4bit_qlora/_vendor/experts.py:447-457`` -- ``dequantize_4bit`` of one
  expert back to ``[out, in]`` in the compute dtype.

The algorithm (QLoRA, arXiv:2305.14314, section 3 and Appendix E):
* codebook: 16 values, normalised quantiles of N(0,1) with an exact zero;
* absmax: per block of 64 consecutive row-major elements, fp32 max |w|;
* quantize: nearest codebook entry of ``w * (1/absmax)``; thresholds are the
  fp32 midpoints ``(c[i] + c[i+1]) * 0.5``; a value exactly on a midpoint goes
  to the LOWER code (this tie rule is this project's choice, unpinned against
  bitsandbytes);
* packing: two codes per byte, the FIRST element in the HIGH nibble;
* dequantize: ``dtype(fp32(code[q]) * absmax)`` with round-to-nearest-even.
"""
from __future__ import annotations

import numpy as np
import torch

# The NF4 table as published in the QLoRA paper (Appendix E). Each value is an
# exact float32.
NF4_CODE = np.array(
    [-1.0, -0.6961928009986877, -0.5250730514526367, -0.39491748809814453,
     -0.28444138169288635, -0.18477343022823334, -0.09105003625154495, 0.0,
     0.07958029955625534, 0.16093020141124725, 0.24611230194568634,
     0.33791524171829224, 0.44070982933044434, 0.5626170039176941,
     0.7229568362236023, 1.0],
    dtype=np.float32,
)

BLOCKSIZE = 64


def nf4_codebook_from_construction(offset: float = 0.9677083) -> np.ndarray:
    """The codebook rebuilt from the paper's construction: 8 positive and 7
    negative normal quantiles between ``offset`` and 0.5, plus an exact zero,
    normalised to [-1, 1]. Used to pin ``NF4_CODE`` independently."""
    from scipy.stats import norm

    pos = norm.ppf(np.linspace(offset, 0.5, 9)[:-1])
    neg = -norm.ppf(np.linspace(offset, 0.5, 8)[:-1])
    v = np.sort(np.concatenate([pos, [0.0], neg]))
    return v / v.max()


def nf4_thresholds() -> np.ndarray:
    """The 15 decision thresholds in fp32: ``(c[i] + c[i+1]) * 0.5``."""
    c = NF4_CODE
    return ((c[:-1] + c[1:]) * np.float32(0.5)).astype(np.float32)


def quantize_nf4(w, blocksize: int = BLOCKSIZE):
    """Quantize a 2-D ``[out, in]`` weight (any float dtype) to NF4.

    Returns ``(packed uint8 [out*in/2], absmax float32 [out*in/blocksize])``.
    """
    a = np.asarray(torch.as_tensor(w).float().contiguous().reshape(-1).numpy(), dtype=np.float32)
    if a.size % blocksize:
        raise ValueError("element count must be a multiple of blocksize")
    blocks = a.reshape(-1, blocksize)
    absmax = np.abs(blocks).max(axis=1).astype(np.float32)
    with np.errstate(divide="ignore"):
        inv = np.where(absmax > 0, np.float32(1.0) / absmax, np.float32(0.0)).astype(np.float32)
    scaled = (blocks * inv[:, None]).astype(np.float32).reshape(-1)
    q = np.searchsorted(nf4_thresholds(), scaled, side="left").astype(np.uint8)
    packed = ((q[0::2] << 4) | q[1::2]).astype(np.uint8)
    return packed, absmax


def unpack_nf4(packed) -> np.ndarray:
    """uint8 bytes -> code indices, first element from the high nibble."""
    p = np.asarray(packed, dtype=np.uint8).reshape(-1)
    out = np.empty(p.size * 2, dtype=np.uint8)
    out[0::2] = p >> 4
    out[1::2] = p & 0xF
    return out


def dequantize_nf4_f32(packed, absmax, blocksize: int = BLOCKSIZE) -> np.ndarray:
    """fp32 ``code[q] * absmax[block]`` (flat)."""
    q = unpack_nf4(packed)
    am = np.asarray(absmax, dtype=np.float32).reshape(-1)
    return (NF4_CODE[q] * np.repeat(am, blocksize)).astype(np.float32)


def dequantize_nf4(packed, absmax, shape, dtype=torch.bfloat16, blocksize: int = BLOCKSIZE) -> torch.Tensor:
    """One matrix dequantized to ``dtype`` (fp32 product, then one RNE cast)."""
    f = torch.from_numpy(dequantize_nf4_f32(packed, absmax, blocksize)).reshape(tuple(shape))
    return f.to(dtype)


def quantize_stack(weights, blocksize: int = BLOCKSIZE):
    """``[E, out, in]`` -> (packed ``[E, out*in/2]`` uint8, absmax ``[E, out*in/bs]`` fp32),
    one independent quantization per expert (``_vendor/experts.py:408-426``)."""
    w = torch.as_tensor(weights)
    packed, absmax = [], []
    for e in range(w.shape[0]):
        p, a = quantize_nf4(w[e], blocksize)
        packed.append(p)
        absmax.append(a)
    return torch.from_numpy(np.stack(packed)), torch.from_numpy(np.stack(absmax))
