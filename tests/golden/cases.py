"""Seeded parity cases shared by the golden-fixture generator and the tests.

Each case is rebuilt from its seed on CPU (torch's CPU generator is
deterministic) and quantized with the oracle codec; the committed fixture
``<name>.npz`` holds sha256 digests of the rebuilt inputs plus the outputs the
reference's own Python produced on them (``make_golden.py``).
"""
from __future__ import annotations

import hashlib

import numpy as np
import torch

from oracle.nf4 import quantize_stack

CASES = ("small", "uneven", "lora_multi", "lora_decode", "lora_bf16_r16", "olmoe_like", "ragged", "nogate")


def _digest(t) -> str:
    a = t.contiguous().view(torch.uint8) if isinstance(t, torch.Tensor) else torch.from_numpy(np.ascontiguousarray(t)).view(torch.uint8)
    return hashlib.sha256(a.numpy().tobytes()).hexdigest()


def _stack(gate_up, down, has_gate=True):
    E, n1, H = gate_up.shape
    I = down.shape[2]
    gp, ga = quantize_stack(gate_up)
    dp, da = quantize_stack(down)
    return {"gate_up_packed": gp, "gate_up_absmax": ga, "down_packed": dp, "down_absmax": da,
            "E": E, "H": H, "I": I, "has_gate": has_gate}


def build(name: str) -> dict:
    """Rebuild case ``name``: dict with st, x, idx, w, k, lora (or None), float weights."""
    lora = None
    router_w = None
    has_gate = True
    if name in ("small", "uneven"):
        # tests/test_fast.py:23-36 (and :110-120 for "uneven")
        E, H, I, k = 4, 128, 64, 2
        T, seed = (16, 0) if name == "small" else (8, 3)
        torch.manual_seed(seed)
        gate_up = torch.randn(E, 2 * I, H, dtype=torch.float32)
        down = torch.randn(E, H, I, dtype=torch.float32)
        x = torch.randn(T, H, dtype=torch.bfloat16)
        logits = torch.randn(T, E)
        top_w, top_i = torch.topk(torch.softmax(logits, -1), k=k, dim=-1)
        w = top_w.to(torch.bfloat16)
        idx = top_i
        if name == "uneven":
            idx = torch.stack([torch.zeros(T, dtype=torch.long), torch.ones(T, dtype=torch.long)], 1)
    elif name in ("lora_multi", "lora_decode", "lora_bf16_r16"):
        # tests/test_fast_lora.py:48-71; the bf16 r=16 variant follows config 3's adapters
        E, H, k = 8, 128, 2
        I = 64 if name == "lora_bf16_r16" else 192
        torch.manual_seed(0)
        gate_up = (torch.randn(E, 2 * I, H) * 0.1)
        down = (torch.randn(E, H, I) * 0.1)
        if name == "lora_bf16_r16":
            r, alpha, adt, std_a, std_b = 16, 16, torch.bfloat16, 0.01, 0.01
        else:
            r, alpha, adt, std_a, std_b = 8, 16, torch.float32, 1.0 / 8, 0.02
        g = torch.Generator().manual_seed(11)
        lora = {
            "gate_up_A": (torch.randn(E, r, H, generator=g) * std_a).to(adt),
            "gate_up_B": (torch.randn(E, 2 * I, r, generator=g) * std_b).to(adt),
            "down_A": (torch.randn(E, r, I, generator=g) * std_a).to(adt),
            "down_B": (torch.randn(E, H, r, generator=g) * std_b).to(adt),
            "scaling": alpha / r, "r": r, "alpha": alpha,
        }
        T = 1 if name == "lora_decode" else (12 if name == "lora_multi" else 24)
        torch.manual_seed(1)
        x = torch.randn(T, H, dtype=torch.bfloat16)
        idx = torch.randint(0, E, (T, k))
        w = torch.rand(T, k, dtype=torch.bfloat16)
    elif name == "olmoe_like":
        # OLMoE fan-out (64 experts, top-8) at small width; router weight [E, H]
        E, H, I, k, T = 64, 128, 64, 8, 5
        g = torch.Generator().manual_seed(0)
        gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
        down = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
        router_w = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        logits = x.float() @ router_w.float().t()
        probs = torch.softmax(logits, -1)
        _, idx = torch.sort(logits, dim=-1, descending=True, stable=True)
        idx = idx[:, :k]
        w = probs.gather(-1, idx)
    elif name == "ragged":
        E, H, I, k, T = 16, 128, 64, 4, 33
        g = torch.Generator().manual_seed(5)
        gate_up = torch.randn(E, 2 * I, H, generator=g) * 0.05
        down = torch.randn(E, H, I, generator=g) * 0.05
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        logits = torch.randn(T, E, generator=g)
        logits[:, [3, 7, 11]] = -1e9            # three cold experts
        logits[:, 0] += 2.0                     # one hot expert
        _, idx = torch.sort(logits, dim=-1, descending=True, stable=True)
        idx = idx[:, :k]
        w = torch.softmax(logits, -1).gather(-1, idx)
    elif name == "nogate":
        # has_gate=False: gate_up is a plain up projection of size I
        E, H, I, k, T = 4, 128, 64, 2, 9
        has_gate = False
        g = torch.Generator().manual_seed(9)
        gate_up = torch.randn(E, I, H, generator=g) * 0.1
        down = torch.randn(E, H, I, generator=g) * 0.1
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        idx = torch.randint(0, E, (T, k), generator=g)
        w = torch.rand(T, k, generator=g)
    else:
        raise KeyError(name)
    st = _stack(gate_up, down, has_gate)
    return {"name": name, "st": st, "x": x, "idx": idx.long(), "w": w, "k": idx.shape[1], "lora": lora,
            "gate_up_f": gate_up, "down_f": down, "router_w": router_w}


def input_digests(case: dict) -> dict:
    st = case["st"]
    d = {f"sha_{k}": _digest(st[k]) for k in ("gate_up_packed", "gate_up_absmax", "down_packed", "down_absmax")}
    d["sha_x"] = _digest(case["x"])
    d["sha_idx"] = _digest(case["idx"])
    d["sha_w"] = _digest(case["w"])
    if case["lora"] is not None:
        for k in ("gate_up_A", "gate_up_B", "down_A", "down_B"):
            d[f"sha_lora_{k}"] = _digest(case["lora"][k])
    return d
