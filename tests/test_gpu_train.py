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


@pytest.mark.parametrize("has_gate", [True, False])
def test_swiglu_kernels_match_torch(e4b, has_gate):
    """e4b_swiglu_forward equals the reference's act(gate) * up in bf16 (SiLU rounded, then the
    product rounded) bit for bit; e4b_swiglu_backward matches the fp32 derivative to 1 bf16 ulp."""
    R, I = 300, 256
    g = torch.Generator(device=DEV).manual_seed(5)
    n1 = 2 * I if has_gate else I
    proj = (torch.randn(R, n1, generator=g, device=DEV) * 3).to(torch.bfloat16)
    h = e4b.ops.swiglu_forward(proj, has_gate)
    if has_gate:
        gt, up = proj.chunk(2, dim=-1)
        ref = torch.nn.functional.silu(gt) * up
    else:
        ref = torch.nn.functional.silu(proj)
    assert torch.equal(h, ref)
    dh = torch.randn(R, I, generator=g, device=DEV)
    dp = e4b.ops.swiglu_backward(proj, dh, has_gate).float()
    pf = proj.float()
    if has_gate:
        gt, up = pf.chunk(2, dim=-1)
        s = torch.sigmoid(gt)
        want = torch.cat([dh * up * (s * (1 + gt * (1 - s))), dh * (gt * s)], dim=-1)
    else:
        s = torch.sigmoid(pf)
        want = dh * (s * (1 + pf * (1 - s)))
    assert torch.allclose(dp, want, rtol=8e-3, atol=1e-6)


def test_combine_row_grads_and_unit_weight_combine(e4b):
    T, k, H = 97, 4, 512
    g = torch.Generator(device=DEV).manual_seed(6)
    R = T * k
    grad = torch.randn(T, H, generator=g, device=DEV)
    order = torch.randperm(R, generator=torch.Generator().manual_seed(1)).to(DEV)
    rows = order // k
    w = torch.rand(R, generator=g, device=DEV)
    down = torch.randn(R, H, generator=g, device=DEV).to(torch.bfloat16)
    dd, dw = e4b.ops.combine_row_grads(grad, rows, w, down)
    assert torch.equal(dd, (grad[rows] * w.view(-1, 1)).to(torch.bfloat16))
    assert torch.allclose(dw, (grad[rows] * down.float()).sum(-1), rtol=1e-5, atol=1e-4)
    inv = torch.empty(R, dtype=torch.int32, device=DEV)
    inv[order] = torch.arange(R, dtype=torch.int32, device=DEV)
    x = torch.randn(R, H, generator=g, device=DEV)
    s = e4b.ops.combine(x, inv, None, T, k, torch.float32)
    assert torch.allclose(s, x[inv.long()].view(T, k, H).sum(1), rtol=1e-6, atol=1e-5)


def test_adapter_segment_kernels_match_per_expert_fp32(e4b):
    """e4b_lora_rank_down / _rank_up / _outer against per-expert fp32 matmuls over ragged segments
    (an empty expert, a one-row expert, segments across several 32-row tiles)."""
    E, r, H, Nn = 5, 16, 512, 384
    counts = [70, 0, 1, 33, 96]
    g = torch.Generator(device=DEV).manual_seed(9)
    offs = [0]
    for c in counts:
        offs.append(offs[-1] + c)
    R = offs[-1]
    tiles = e4b.ops.RowTiles(offs, torch.device(DEV))
    X = torch.randn(R, H, generator=g, device=DEV).to(torch.bfloat16)
    A = torch.randn(E, r, H, generator=g, device=DEV) * 0.05
    B = torch.randn(E, Nn, r, generator=g, device=DEV) * 0.05
    Y = e4b.ops.lora_rank_down(X, A, (r * H, H, 1), r, tiles)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        want = torch.zeros(R, r, device=DEV)
        for e in range(E):
            want[offs[e]:offs[e + 1]] = X[offs[e]:offs[e + 1]].float() @ A[e].t()
        assert torch.allclose(Y, want, rtol=1e-4, atol=1e-4)
        out = torch.zeros(R, Nn, device=DEV)
        e4b.ops.lora_rank_up(Y, B, (Nn * r, 1, r), Nn, tiles, out, 0.5)
        want_up = torch.zeros(R, Nn, device=DEV)
        for e in range(E):
            want_up[offs[e]:offs[e + 1]] = 0.5 * (Y[offs[e]:offs[e + 1]] @ B[e].t())
        assert torch.allclose(out, want_up, rtol=1e-4, atol=1e-5)
        P = torch.randn(R, Nn, generator=g, device=DEV).to(torch.bfloat16)
        G = torch.zeros(E, Nn, r, device=DEV)
        e4b.ops.lora_outer(P, Y, tiles, G, (Nn * r, r, 1), 2.0)
        for e in range(E):
            we = 2.0 * (P[offs[e]:offs[e + 1]].float().t() @ Y[offs[e]:offs[e + 1]])
            assert torch.allclose(G[e], we, rtol=1e-4, atol=1e-4), e
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
