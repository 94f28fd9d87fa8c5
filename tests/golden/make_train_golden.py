"""Regenerate the training-path golden fixture by running the REFERENCE's ``ExpertsLoRA``
forward AND backward on CPU (autograd through its own loop and its recompute-backward
frozen projection).

Run in the build container only (it imports experts4bit-qlora from its source tree,
which does not exist on the GPU box):

    python tests/golden/make_train_golden.py [/path/to/experts4bit-qlora]

bitsandbytes is not installed there; ``oracle/bnb_shim`` puts the oracle's NF4 codec
behind its function names, so ``Experts4bit.from_float`` / ``_dequantize_expert`` and
``ExpertsLoRA.forward`` run as shipped. The fixture is the reference parity contract's
own layer (tests/test_fused_train_parity.py:40-110 there): E=8, H=128, I=192, top-2,
``ExpertsLoRA(r=8, alpha=16, dtype=float32)`` with B ~ N(0, 0.02), bf16 compute, 64
tokens, bf16 top-k weights, a fixed random loss weighting. Saved: the quantized stacks,
the adapters, the inputs, and the outputs -- forward, dL/dx, dL/d top_k_weights and the
four adapter gradients.
"""
from __future__ import annotations

import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))

E, HID, INTER, TOP_K, R, T = 8, 128, 192, 2, 8, 64


def _f32(t):
    return t.detach().float().contiguous().numpy()


def main(ref_root: str) -> None:
    sys.path[:0] = [os.path.join(REPO, "oracle", "bnb_shim"), REPO, ref_root]
    from experts4bit_qlora import Experts4bit, ExpertsLoRA

    torch.manual_seed(0)
    gate_up = torch.randn(E, 2 * INTER, HID) * 0.1
    down = torch.randn(E, HID, INTER) * 0.1
    base = Experts4bit.from_float(gate_up, down, quant_type="nf4", compute_dtype=torch.bfloat16)
    mod = ExpertsLoRA(base, r=R, alpha=16, dtype=torch.float32)
    with torch.no_grad():
        for p in (mod.gate_up_lora_B, mod.down_lora_B):
            p.normal_(0, 0.02)
    mod.train()
    torch.manual_seed(1)
    hs = torch.randn(T, HID, dtype=torch.bfloat16)
    idx = torch.randint(0, E, (T, TOP_K))
    wts = torch.rand(T, TOP_K, dtype=torch.bfloat16)
    torch.manual_seed(101)
    loss_w = torch.randn(T, HID)

    x = hs.clone().requires_grad_(True)
    w = wts.clone().requires_grad_(True)
    out = mod(x, idx, w)
    (out.float() * loss_w).sum().backward()
    res = {
        "gate_up_packed": base.gate_up_proj.data.numpy(), "gate_up_absmax": base.gate_up_absmax.numpy(),
        "down_packed": base.down_proj.data.numpy(), "down_absmax": base.down_absmax.numpy(),
        "hs": _f32(hs), "idx": idx.numpy(), "wts": _f32(wts), "loss_w": loss_w.numpy(),
        "out": _f32(out), "dx": _f32(x.grad), "dw": _f32(w.grad),
    }
    for n in ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B"):
        p = getattr(mod, n)
        res[n] = _f32(p)
        res["d_" + n] = _f32(p.grad)
    np.savez_compressed(os.path.join(HERE, "train_lora.npz"), **res)
    print({k: v.shape for k, v in res.items()})


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("E4B_REFERENCE_ROOT", "../reference"))
