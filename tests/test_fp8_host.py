"""CPU: the FP8 block-scaled storage mode (formats/fp8_blocks.py:60-128 of the
reference) -- the oracle and the module's host dequant pinned bit-exactly to
fixtures produced by the reference's own ``dequantize_fp8_blocks``
(tests/golden/make_fp8_golden.py), the quantizer's invariants, and the module's
reference loop against the oracle loop."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import moe as M

GOLD = os.path.join(os.path.dirname(__file__), "golden", "fp8_blocks.npz")
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _cases():
    d = dict(np.load(GOLD))
    return d, sorted({k.split("__")[0] for k in d})


def _bits(y):
    return y.view(torch.int32).numpy() if y.dtype == torch.float32 else y.view(torch.int16).numpy()


@pytest.mark.parametrize("name", _cases()[1])
def test_oracle_matches_reference_fixture(name):
    d, _ = _cases()
    dt = DT[name.rsplit("_", 1)[1]]
    y = M.fp8_block_dequant(torch.from_numpy(d[name + "__w"]), torch.from_numpy(d[name + "__scale"]), dtype=dt)
    assert np.array_equal(_bits(y), d[name + "__out"])


@pytest.mark.parametrize("name", _cases()[1])
def test_module_host_dequant_matches_reference_fixture(e4b, name):
    from importlib import import_module
    f8 = import_module("experts4bit-qlora_b200.fp8_experts")
    d, _ = _cases()
    dt = DT[name.rsplit("_", 1)[1]]
    y = f8.dequantize_fp8_blocks(torch.from_numpy(d[name + "__w"]), torch.from_numpy(d[name + "__scale"]), dt)
    assert np.array_equal(_bits(y), d[name + "__out"])


@pytest.mark.parametrize("fmt", ["e8m0", "fp32"])
def test_quantizer_invariants(e4b, fmt):
    from importlib import import_module
    f8 = import_module("experts4bit-qlora_b200.fp8_experts")
    g = torch.Generator().manual_seed(0)
    w = torch.randn(3, 256, 384, generator=g) * 0.02
    w[1, :128, :128] *= 1e3          # one hot tile
    q, s = f8.quantize_fp8_blocks(w, fmt)
    assert q.dtype == torch.uint8 and q.shape == w.shape
    assert s.shape == (3, 2, 3) and (s.dtype == torch.uint8) == (fmt == "e8m0")
    assert not torch.isnan(q.view(torch.float8_e4m3fn).float()).any()
    back = torch.stack([M.fp8_block_dequant(q[e], s[e], dtype=torch.float32) for e in range(3)])
    # e4m3 keeps 3 mantissa bits: relative error <= 2^-4 of each tile's scale range
    tiles = lambda t: t.view(3, 2, 128, 3, 128)  # noqa: E731
    err = tiles(back - w).abs().amax(dim=(2, 4))
    amax = tiles(w).abs().amax(dim=(2, 4))
    assert (err <= amax * 2 ** -3).all()


def test_module_loop_matches_oracle_loop(e4b):
    g = torch.Generator().manual_seed(1)
    E, H, I, T, k = 4, 256, 128, 12, 2
    gu = torch.randn(E, 2 * I, H, generator=g) * 0.05
    dn = torch.randn(E, H, I, generator=g) * 0.05
    mod = e4b.ExpertsFp8Blocks.from_float(gu, dn)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, idx = M.route_on_host(torch.randn(T, E, generator=g), k)
    st = {"format": "fp8", "gate_up_w": mod.gate_up_proj.data, "gate_up_scale": mod.gate_up_scale,
          "down_w": mod.down_proj.data, "down_scale": mod.down_scale, "E": E, "H": H, "I": I, "has_gate": True}
    with torch.no_grad():
        got = mod(x, idx, w)
    ref = M.reference_forward(st, x, idx, w, torch.bfloat16)
    assert torch.equal(got, ref)
    mx, mean = M.rel_errors(got.float(), M.fp32_oracle(st, x, idx, w))
    assert mx <= 1e-2 and mean <= 5e-3
