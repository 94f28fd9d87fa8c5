"""Regenerate ``fp8_blocks.npz`` by running the REFERENCE's own
``formats.fp8_blocks.dequantize_fp8_blocks`` (pure torch) on seeded inputs.

Run in the build container only (it imports experts4bit-qlora from its source tree):

    python tests/golden/make_fp8_golden.py [/path/to/experts4bit-qlora]

Cases: aligned and ragged shapes; e8m0 scales (uint8 bytes) and arbitrary fp32
scales; bf16, fp16 and fp32 outputs. Inputs are stored beside the outputs.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

# (name, rows, cols, scale kind, out dtype)
CASES = [
    ("aligned_e8m0_bf16", 256, 384, "e8m0", torch.bfloat16),
    ("aligned_f32_bf16", 256, 384, "f32", torch.bfloat16),
    ("aligned_f32_f16", 128, 256, "f32", torch.float16),
    ("aligned_e8m0_f32", 128, 256, "e8m0", torch.float32),
    ("ragged_f32_bf16", 130, 200, "f32", torch.bfloat16),
    ("ragged_e8m0_bf16", 200, 136, "e8m0", torch.bfloat16),
]


def make_inputs(rows, cols, kind, seed):
    g = torch.Generator().manual_seed(seed)
    w = (torch.randn(rows, cols, generator=g) * 64).clamp(-448, 448).to(torch.float8_e4m3fn)
    w_u8 = w.view(torch.uint8)
    w_u8[0, :8] = torch.tensor([0x00, 0x80, 0x01, 0x81, 0x07, 0x08, 0x7E, 0xFE], dtype=torch.uint8)  # zeros, subnormals, max
    tiles = ((rows + 127) // 128, (cols + 127) // 128)
    if kind == "e8m0":
        scale = torch.randint(110, 135, tiles, generator=g, dtype=torch.int32).to(torch.uint8)
    else:
        scale = torch.rand(tiles, generator=g) * 1e-2 + 1e-4
    return w_u8, scale


def main(ref_root):
    repo = os.path.dirname(os.path.dirname(HERE))
    # the package __init__ imports bitsandbytes; the oracle's stand-in satisfies it
    sys.path[:0] = [os.path.join(repo, "oracle", "bnb_shim"), repo, ref_root]
    from experts4bit_qlora.formats.fp8_blocks import dequantize_fp8_blocks

    out = {}
    for i, (name, rows, cols, kind, dt) in enumerate(CASES):
        w_u8, scale = make_inputs(rows, cols, kind, 100 + i)
        y = dequantize_fp8_blocks(w_u8, scale, dtype=dt)
        out[f"{name}__w"] = w_u8.numpy()
        out[f"{name}__scale"] = scale.numpy()
        out[f"{name}__out"] = y.view(torch.int16).numpy() if dt != torch.float32 else y.view(torch.int32).numpy()
    np.savez_compressed(os.path.join(HERE, "fp8_blocks.npz"), **out)
    print("fp8_blocks", sorted({k.split("__")[0] for k in out}))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("E4B_REFERENCE_ROOT", "../reference"))
