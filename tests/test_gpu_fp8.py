"""GPU: block-scaled FP8 expert storage through the C ABI -- the dequant entry
point bit-exact against the reference's own ``dequantize_fp8_blocks`` outputs
(fixtures), and the fused layer (decode GEMV and tcgen05 regimes, enable_fast,
expert parallelism) against the fp32 oracle within the layer tolerance."""
from __future__ import annotations

import os

import numpy as np
import pytest
import torch

from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"
GOLD = os.path.join(os.path.dirname(__file__), "golden", "fp8_blocks.npz")
DT = {"bf16": torch.bfloat16, "f16": torch.float16, "f32": torch.float32}


def _names():
    return sorted({k.split("__")[0] for k in np.load(GOLD).files})


@pytest.mark.parametrize("name", _names())
def test_fp8_dequant_bit_exact_vs_reference_fixture(e4b, name):
    d = np.load(GOLD)
    dt = DT[name.rsplit("_", 1)[1]]
    w = torch.from_numpy(d[name + "__w"]).to(DEV)
    s = M.fp8_scale_values(torch.from_numpy(d[name + "__scale"])).to(DEV)
    y = e4b.ops.fp8_block_dequantize(w, s, dt).cpu()
    bits = y.view(torch.int32).numpy() if dt == torch.float32 else y.view(torch.int16).numpy()
    assert np.array_equal(bits, d[name + "__out"])


def _layer(e4b, E, H, I, fmt="e8m0", seed=0):
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    mod = e4b.ExpertsFp8Blocks.from_float(gu.to(DEV), dn.to(DEV), scale_format=fmt)
    st = {"format": "fp8", "gate_up_w": mod.gate_up_proj.data.cpu(), "gate_up_scale": mod.gate_up_scale.cpu(),
          "down_w": mod.down_proj.data.cpu(), "down_scale": mod.down_scale.cpu(), "E": E, "H": H, "I": I,
          "has_gate": True}
    return mod, st


def _inputs(E, H, T, k, seed=1, zipf=False):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    if zipf:  # skewed popularity: a few hot experts
        logits = logits + torch.log(1.0 / torch.arange(1, E + 1).float() ** 1.1)[torch.randperm(E, generator=g)]
    w, idx = M.route_on_host(logits, k)
    return x, idx, w


def _check(got, st, x, idx, w):
    ref32 = M.fp32_oracle(st, x, idx, w)
    mx, mean = M.rel_errors(got.float().cpu(), ref32)
    loop = M.reference_forward(st, x, idx, w, torch.bfloat16)
    lmx, lmean = M.rel_errors(loop.float(), ref32)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)
    assert mx <= max(2 * lmx, 5e-3), (mx, lmx)


@pytest.mark.parametrize("T,fmt", [(1, "e8m0"), (5, "fp32"), (16, "e8m0"), (40, "e8m0"), (300, "fp32")])
def test_fp8_layer_vs_oracle(e4b, T, fmt):
    E, H, I, k = 16, 512, 256, 4
    mod, st = _layer(e4b, E, H, I, fmt)
    x, idx, w = _inputs(E, H, T, k, zipf=True)
    gs, ds = mod.scale_values()
    got = e4b.ops.moe_forward(x.to(DEV), idx.to(DEV), w.to(DEV), mod.gate_up_proj, gs, mod.down_proj, ds, E, I,
                              check_errors=True, weight_format=e4b._native.FMT_FP8_BLOCK128)
    _check(got, st, x, idx, w)


def test_fp8_enable_fast_and_fallbacks(e4b):
    E, H, I, k, T = 8, 256, 128, 2, 24
    mod, st = _layer(e4b, E, H, I, seed=3)
    x, idx, w = _inputs(E, H, T, k, seed=4)
    xc, ic, wc = x.to(DEV), idx.to(DEV), w.to(DEV)
    with torch.no_grad():
        ref = mod(xc, ic, wc)
        assert e4b.enable_fast(mod) == 1
        got = mod(xc, ic, wc)
        assert e4b.disable_fast(mod) == 1
        again = mod(xc, ic, wc)
    assert torch.equal(ref, again)
    _check(got, st, x, idx, w)


def test_fp8_fp16_activations_and_adapter_refusal(e4b):
    E, H, I, k = 4, 256, 128, 2
    mod, st = _layer(e4b, E, H, I)
    x, idx, w = _inputs(E, H, 20, k)
    gs, ds = mod.scale_values()
    got = e4b.ops.moe_forward(x.to(DEV).half(), idx.to(DEV), w.to(DEV), mod.gate_up_proj, gs, mod.down_proj, ds, E,
                              I, check_errors=True, weight_format=e4b._native.FMT_FP8_BLOCK128)
    _check(got.to(torch.bfloat16), st, x.half().to(torch.bfloat16), idx, w)
    r = 8
    lora = tuple(torch.zeros(s_, device=DEV) for s_ in ((E, r, H), (E, 2 * I, r), (E, r, I), (E, H, r))) + (1.0,)
    with pytest.raises(e4b._native.E4BError):
        e4b.ops.moe_forward(x.to(DEV), idx.to(DEV), w.to(DEV), mod.gate_up_proj, gs, mod.down_proj, ds, E, I,
                            lora=lora, weight_format=e4b._native.FMT_FP8_BLOCK128)


@pytest.mark.parametrize("P", [2, 4])
def test_fp8_expert_parallel_bitexact(e4b, P):
    from test_gpu_ep import emulate_ep
    E, H, I, k, T = 8, 256, 256, 2, 256
    mod, st = _layer(e4b, E, H, I, seed=5)
    x, idx, w = _inputs(E, H, T, k, seed=6)
    xc, ic, wc = x.to(DEV), idx.to(DEV), w.to(DEV)
    gs, ds = mod.scale_values()
    single = e4b.ops.moe_forward(xc, ic, wc, mod.gate_up_proj, gs, mod.down_proj, ds, E, I,
                                 weight_format=e4b._native.FMT_FP8_BLOCK128)
    got = emulate_ep(e4b, mod, xc, ic, wc, P)
    torch.cuda.synchronize()
    assert torch.equal(got, single)
    _check(got, st, x, idx, w)
