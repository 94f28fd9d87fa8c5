"""Regenerate tests/golden/mxfp4.npz by running the REFERENCE's ``dequantize_mxfp4``
(formats/mxfp4.py) on seeded inputs. Run in the build container only (it imports the
reference from its source tree):

    python tests/golden/make_mxfp4_golden.py [/path/to/experts4bit-qlora]

Cases: a gpt-oss-like rank-4 stack ``[E, rows, G, 16]`` and a single rank-3 projection,
with random codes and e8m0 scales over 0..255 (the extremes included; 255 with zero codes,
which the reference turns into NaN), dequantized to
bf16, fp16 and fp32. The outputs are stored as raw bit patterns.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))

CASES = {"stack": (3, 64, 4, 16), "single": (48, 2, 16)}


def inputs(name):
    shape = CASES[name]
    g = np.random.default_rng(7 + len(shape))
    blocks = g.integers(0, 256, size=shape, dtype=np.uint8)
    scales = g.integers(100, 140, size=shape[:-1], dtype=np.uint8)   # realistic weight scales
    flat = scales.reshape(-1)
    flat[:5] = (0, 1, 253, 254, 255)                                 # the extremes; 255 gives 2**128 = inf
    codes = blocks.reshape(-1, shape[-1])
    codes[4, :2] = (0x00, 0x80)                                      # +0 and -0 codes under the inf scale
    return blocks, scales


def main(ref_root: str) -> None:
    repo = os.path.dirname(os.path.dirname(HERE))
    sys.path[:0] = [os.path.join(repo, "oracle", "bnb_shim"), repo, ref_root]  # the package imports bitsandbytes
    from experts4bit_qlora.formats.mxfp4 import dequantize_mxfp4
    out = {}
    for name in CASES:
        blocks, scales = inputs(name)
        out[f"{name}_blocks"], out[f"{name}_scales"] = blocks, scales
        for dt, tag, view in ((torch.bfloat16, "bf16", torch.int16), (torch.float16, "f16", torch.int16),
                              (torch.float32, "f32", torch.int32)):
            y = dequantize_mxfp4(torch.from_numpy(blocks), torch.from_numpy(scales), dtype=dt)
            out[f"{name}_{tag}"] = y.view(view).numpy()
    np.savez_compressed(os.path.join(HERE, "mxfp4.npz"), **out)
    print({k: v.shape for k, v in out.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("E4B_REFERENCE_ROOT", "../reference"))
