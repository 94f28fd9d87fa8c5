"""CPU: this package's ``ExpertsLoRA`` loop -- the reference the GPU training-path parity
test (test_gpu_train.py) compares against -- reproduces the REFERENCE's own ``ExpertsLoRA``
forward and every gradient (dL/dx, dL/d top_k_weights, the four adapter gradients) on the
reference parity contract's fixture. The fixture was made by running the reference's code
(tests/golden/make_train_golden.py) on the same NF4 bytes; the match is bit-exact."""
import os

import numpy as np
import pytest
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
NAMES = ("gate_up_lora_A", "gate_up_lora_B", "down_lora_A", "down_lora_B")


def _rel(got, want):
    return float((got.float() - want.float()).norm() / want.float().norm().clamp_min(1e-12))


def test_lora_loop_forward_and_gradients_match_reference(e4b):
    g = np.load(os.path.join(HERE, "golden", "train_lora.npz"))
    E, n1, H = 8, 384, 128
    I = n1 // 2
    base = e4b.Experts4bit(E, H, I, compute_dtype=torch.bfloat16)
    base.gate_up_proj = torch.nn.Parameter(torch.from_numpy(g["gate_up_packed"]), requires_grad=False)
    base.gate_up_absmax = torch.from_numpy(g["gate_up_absmax"])
    base.down_proj = torch.nn.Parameter(torch.from_numpy(g["down_packed"]), requires_grad=False)
    base.down_absmax = torch.from_numpy(g["down_absmax"])
    mod = e4b.ExpertsLoRA(base, r=8, alpha=16, dtype=torch.float32)
    with torch.no_grad():
        for n in NAMES:
            getattr(mod, n).copy_(torch.from_numpy(g[n]))
    mod.train()
    x = torch.from_numpy(g["hs"]).to(torch.bfloat16).requires_grad_(True)
    w = torch.from_numpy(g["wts"]).to(torch.bfloat16).requires_grad_(True)
    idx = torch.from_numpy(g["idx"])
    out = mod(x, idx, w)
    (out.float() * torch.from_numpy(g["loss_w"])).sum().backward()
    got = {"out": out, "dx": x.grad, "dw": w.grad}
    got.update({"d_" + n: getattr(mod, n).grad for n in NAMES})
    for k, v in got.items():
        ref = torch.from_numpy(g[k])
        assert v.shape == ref.shape, k
        # same bytes, the same bf16 loop and autograd graph: bit for bit
        assert torch.equal(v.detach().float(), ref), (k, _rel(v.detach(), ref))
