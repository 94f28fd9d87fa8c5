"""GPU: the fused training path (``enable_fast_train``) against the reference loop.

The contract is the reference's (tests/test_fused_train_parity.py:46-170 there):
forward values, dL/dx and dL/d(every LoRA parameter) of the patched ``ExpertsLoRA``
must match the unpatched module's loop forward within the bf16 noise floor
(norm-relative 1.5e-2 forward, 1e-2 gradients), with a load-bearing adapter; and
the same assertions must REJECT a path whose LoRA scaling is off by 1%."""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu
DEV = "cuda"
FWD_TOL = 1.5e-2
GRAD_TOL = 1.0e-2


def _rel(got, want):
    want = want.float()
    return ((got.float() - want).norm() / want.norm().clamp_min(1e-12)).item()


def _build(e4b, E=8, H=128, I=192, r=8, seed=0, scaling_bug=1.0):
    torch.manual_seed(seed)
    gate_up = (torch.randn(E, 2 * I, H) * 0.1).to(DEV)
    down = (torch.randn(E, H, I) * 0.1).to(DEV)
    base = e4b.Experts4bit.from_float(gate_up, down, quant_type="nf4", compute_dtype=torch.bfloat16)
    mod = e4b.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.float32).to(DEV)
    with torch.no_grad():
        for p in (mod.gate_up_lora_B, mod.down_lora_B):
            p.normal_(0, 0.02)
    mod.scaling *= scaling_bug
    return mod.train()


def _inputs(E, H, k=2, n_tok=64, seed=1):
    torch.manual_seed(seed)
    hs = torch.randn(n_tok, H, dtype=torch.bfloat16, device=DEV)
    idx = torch.randint(0, E, (n_tok, k), device=DEV)
    wts = torch.rand(n_tok, k, dtype=torch.bfloat16, device=DEV)
    torch.manual_seed(seed + 100)
    loss_w = torch.randn(n_tok, H, device=DEV)
    return hs, idx, wts, loss_w


def _forward_backward(mod, hs, idx, wts, loss_w):
    hs = hs.clone().requires_grad_(True)
    wts = wts.clone().requires_grad_(True)
    for p in mod.parameters():
        p.grad = None
    out = mod(hs, idx, wts)
    assert out.requires_grad
    (out.float() * loss_w).sum().backward()
    grads = {n: p.grad.detach().clone() for n, p in mod.named_parameters() if p.grad is not None}
    assert grads
    return out.detach(), hs.grad.detach().clone(), wts.grad.detach().clone(), grads


def _parity(cand, ref, args):
    ref_out, ref_dx, ref_dw, ref_g = _forward_backward(ref, *args)
    out, dx, dw, g = _forward_backward(cand, *args)
    m = {"forward": _rel(out, ref_out), "dL/dx": _rel(dx, ref_dx), "dL/dw": _rel(dw, ref_dw)}
    assert set(g) == set(ref_g)
    for n in ref_g:
        m[f"dL/d{n}"] = _rel(g[n], ref_g[n])
    return m


def _ok(m):
    return m["forward"] < FWD_TOL and all(v < GRAD_TOL for k, v in m.items() if k != "forward")


@pytest.mark.parametrize("dgrad", [False, True], ids=["decode_once", "dgrad_kernel"])
@pytest.mark.parametrize("geom", [(8, 128, 192, 64), (8, 256, 256, 512), (8, 512, 768, 384)],
                         ids=["reference_fixture", "tensor_core", "qwen3_widths"])
def test_fused_train_matches_reference_forward_and_gradients(e4b, geom, dgrad):
    """With dgrad=True the tensor-core geometries take both input gradients through
    e4b_grouped_nf4_dgrad (the reference fixture's widths are not multiples of 256 and keep
    the decode-once path)."""
    E, H, I, T = geom
    ref = _build(e4b, E, H, I)
    cand = _build(e4b, E, H, I)
    for (n, p), (_, q) in zip(cand.named_parameters(), ref.named_parameters()):
        assert torch.equal(p, q), n
    assert e4b.enable_fast_train(cand, dgrad=dgrad) == 1
    m = _parity(cand, ref, _inputs(E, H, n_tok=T))
    print("\nfused train vs loop: " + "  ".join(f"{k}={v:.2e}" for k, v in m.items()))
    assert _ok(m), m
    assert e4b.disable_fast_train(cand) == 1
    assert not hasattr(cand, "_e4b_train_ref")


def test_contract_rejects_a_one_percent_scaling_error(e4b):
    ref = _build(e4b)
    mutant = _build(e4b, scaling_bug=1.01)
    assert e4b.enable_fast_train(mutant) == 1
    m = _parity(mutant, ref, _inputs(8, 128))
    assert not _ok(m), m


def test_enable_fast_train_skips_ineligible_and_repatch(e4b):
    mod = _build(e4b)
    assert e4b.enable_fast_train(mod) == 1
    with pytest.warns(RuntimeWarning):
        assert e4b.enable_fast_train(mod, dgrad=True) == 0
    assert e4b.disable_fast_train(mod) == 1
    assert e4b.disable_fast_train(mod) == 0
