"""MXFP4 (OCP Microscaling FP4) restated -- test infrastructure only (a checker, never
the product path).

Follows formats/mxfp4.py:25-105 of the reference (itself a restatement of
transformers' convert_moe_packed_tensors): blocks ``uint8 [..., rows, G, B]`` hold two
e2m1 codes per byte, LOW nibble first; scales ``uint8 [..., rows, G]`` are e8m0
exponents (bias 127), one per block of 2B values; the value is
``ldexp(FP4_VALUES[code], s - 127)`` in fp32 (the exact product, rounded once; 2**128 is not
formed on its own, so zero codes stay signed zeros even for s = 255), rounded once to the output
dtype, and the result has its trailing (rows, K) pair transposed to ``[..., K, rows]``.
Pinned by tests/golden/mxfp4.npz, made by running the reference's function.
"""
from __future__ import annotations

import numpy as np

FP4_VALUES = np.array([0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0,
                       -0.0, -0.5, -1.0, -1.5, -2.0, -3.0, -4.0, -6.0], dtype=np.float32)


def dequantize_mxfp4_f32(blocks: np.ndarray, scales: np.ndarray) -> np.ndarray:
    """fp32 values ``[..., K, rows]`` (K = G * 2B) before the output-dtype rounding."""
    *prefix, rows, G, B = blocks.shape
    lo = FP4_VALUES[blocks & 0x0F]
    hi = FP4_VALUES[blocks >> 4]
    vals = np.empty((*prefix, rows, G, 2 * B), dtype=np.float32)
    vals[..., 0::2] = lo
    vals[..., 1::2] = hi
    exp = (scales.astype(np.int32) - 127)[..., None]
    with np.errstate(over="ignore"):
        # ldexp, as the reference's torch.ldexp: one rounding of the exact product, so 0.5 * 2**128
        # is finite and a zero code stays a signed zero under e8m0 255
        vals = np.ldexp(vals, exp).astype(np.float32)
    vals = vals.reshape(*prefix, rows, G * 2 * B)
    return np.swapaxes(vals, -1, -2).copy()
