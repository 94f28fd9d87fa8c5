"""CPU: the training path's autograd math (train.py) with its device calls -- permutation,
grouped NF4 GEMM, stack dequantization, the SwiGLU and combine steps -- replaced by CPU
stand-ins built on the oracle, the host codec and the same formulas in torch. Forward and every gradient of the fused autograd function
must match autograd through the ``ExpertsLoRA`` loop on the same NF4 bytes (the GPU test,
test_gpu_train.py, checks the real kernels under the same contract)."""
import importlib
import types

import pytest
import torch

from oracle import moe as M


def _rel(got, want):
    return float((got.float() - want.float()).norm() / want.float().norm().clamp_min(1e-12))


def _cpu_ops(e4b):
    real = e4b.ops

    def permute(idx, E):
        order, _, _, _, offsets = M.permute(idx.cpu(), E)
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.numel())
        return order.to(torch.int32), inv.to(torch.int32), offsets.to(torch.int32)

    def grouped_nf4_gemm(a, packed, absmax, offsets, a_rows=None, epilogue=0):
        E, Nn, Kh = packed.shape
        W = real.nf4_dequantize(packed, absmax, (E, Nn, Kh * 2), a.dtype)   # host codec
        x = a[a_rows.long()] if a_rows is not None else a
        out = torch.empty(x.shape[0], Nn, dtype=a.dtype)
        for e in range(E):
            lo, hi = int(offsets[e]), int(offsets[e + 1])
            out[lo:hi] = (x[lo:hi].float() @ W[e].float().t()).to(a.dtype)
        return out

    def swiglu_forward(proj, has_gate=True):
        if has_gate:
            g, u = proj.chunk(2, dim=-1)
            return torch.nn.functional.silu(g) * u
        return torch.nn.functional.silu(proj)

    def swiglu_backward(proj, dh, has_gate=True):
        pf = proj.float()
        if has_gate:
            g, u = pf.chunk(2, dim=-1)
            s = torch.sigmoid(g)
            return torch.cat([dh * u * (s * (1 + g * (1 - s))), dh * (g * s)], dim=-1).to(proj.dtype)
        s = torch.sigmoid(pf)
        return (dh * (s * (1 + pf * (1 - s)))).to(proj.dtype)

    def combine(rows, inv, w, T, k, out_dtype=torch.bfloat16):
        r = rows.float()[inv.long()].view(T, k, -1)
        if w is not None:
            r = r * w.float().view(T, k, 1)
        return r.sum(1).to(out_dtype)

    def combine_row_grads(grad, token_rows, w_rows, down):
        g = grad.float()[token_rows.long()]
        return (g * w_rows.float().view(-1, 1)).to(down.dtype), (g * down.float()).sum(-1)

    class RowTiles:
        def __init__(self, offs, device):
            self.offs = list(offs)

        def rows(self):
            for e in range(len(self.offs) - 1):
                if self.offs[e + 1] > self.offs[e]:
                    yield e, self.offs[e], self.offs[e + 1]

    def _m(M, strides, e, d0, d1):  # M_e(j, k) as a [d0, d1] fp32 matrix
        sE, sj, sk = strides
        flat = M.float().reshape(-1)
        j = torch.arange(d0).view(-1, 1)
        kk = torch.arange(d1).view(1, -1)
        return flat[e * sE + j * sj + kk * sk]

    def lora_rank_down(X, M, strides, rk, tiles, scale=1.0):
        Y = torch.zeros(X.shape[0], rk)
        for e, a, b in tiles.rows():
            Y[a:b] = scale * (X[a:b].float() @ _m(M, strides, e, rk, X.shape[1]).t())
        return Y

    def lora_rank_up(Y, M, strides, n, tiles, out, scale=1.0):
        out = out.clone()
        for e, a, b in tiles.rows():
            d = scale * (Y[a:b] @ _m(M, strides, e, Y.shape[1], n))
            if out.dtype == torch.float32:
                out[a:b] += d
            else:
                out[a:b] = out[a:b] + d.to(out.dtype)
        return out

    def lora_outer(P, Y, tiles, G, strides, scale=1.0):
        gE, ga, gj = strides
        flat = G.view(-1)
        A = P.shape[1]
        for e, a0, b0 in tiles.rows():
            g = scale * (P[a0:b0].float().t() @ Y[a0:b0])           # [A, rk]
            idx = e * gE + torch.arange(A).view(-1, 1) * ga + torch.arange(Y.shape[1]).view(1, -1) * gj
            flat[idx.reshape(-1)] = g.reshape(-1)
        return G

    return types.SimpleNamespace(RowTiles=RowTiles, lora_rank_down=lora_rank_down, lora_rank_up=lora_rank_up,
                                 lora_outer=lora_outer, permute=permute, grouped_nf4_gemm=grouped_nf4_gemm,
                                 nf4_dequantize=real.nf4_dequantize, swiglu_forward=swiglu_forward,
                                 swiglu_backward=swiglu_backward, combine=combine,
                                 combine_row_grads=combine_row_grads, dgrad_eligible=lambda n, k: False)


@pytest.mark.parametrize("has_gate", [True, False])
def test_fused_train_autograd_matches_loop_on_cpu(e4b, monkeypatch, has_gate):
    train = importlib.import_module("experts4bit-qlora_b200.train")
    monkeypatch.setattr(train, "ops", _cpu_ops(e4b))
    E, H, I, k, T = 8, 128, 192, 2, 48
    torch.manual_seed(0)
    n1 = 2 * I if has_gate else I
    base = e4b.Experts4bit.from_float(torch.randn(E, n1, H) * 0.1, torch.randn(E, H, I) * 0.1,
                                      has_gate=has_gate, compute_dtype=torch.bfloat16)
    lm = e4b.ExpertsLoRA(base, r=8, alpha=16, dtype=torch.float32)
    with torch.no_grad():
        lm.gate_up_lora_B.normal_(0, 0.02)
        lm.down_lora_B.normal_(0, 0.02)
    lm.train()
    torch.manual_seed(1)
    hs = torch.randn(T, H, dtype=torch.bfloat16)
    idx = torch.randint(0, E, (T, k))
    idx[:, 1] = (idx[:, 0] + 1 + torch.randint(0, E - 1, (T,))) % E        # distinct picks per token
    idx[idx == 5] = 6                                                     # expert 5 never routed
    idx[:, 1] = torch.where(idx[:, 1] == idx[:, 0], (idx[:, 0] + 2) % E, idx[:, 1])
    wts = torch.rand(T, k, dtype=torch.bfloat16)
    loss_w = torch.randn(T, H)

    def run(fused):
        x = hs.clone().requires_grad_(True)
        w = wts.clone().requires_grad_(True)
        for p in lm.parameters():
            p.grad = None
        if fused:
            out = train._FusedExpertsLoRATrain.apply(x, w, lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A,
                                                     lm.down_lora_B, lm, idx).to(x.dtype)
        else:
            out = lm(x, idx, w)
        (out.float() * loss_w).sum().backward()
        grads = {n: p.grad.clone() for n, p in lm.named_parameters() if p.grad is not None}
        return out.detach(), x.grad.clone(), w.grad.clone(), grads

    ref = run(False)
    got = run(True)
    print("\nfwd %.2e dx %.2e dw %.2e " % (_rel(got[0], ref[0]), _rel(got[1], ref[1]), _rel(got[2], ref[2])) + " ".join("%s %.2e" % (n, _rel(got[3][n], ref[3][n])) for n in ref[3]))
    assert _rel(got[0], ref[0]) < 1e-2
    assert _rel(got[1], ref[1]) < 1e-2
    assert _rel(got[2], ref[2]) < 1e-2
    assert set(got[3]) == set(ref[3])
    for n in ref[3]:
        assert _rel(got[3][n], ref[3][n]) < 1e-2, n
        # the adapter rows of the expert nobody routed to get exactly zero gradient
        assert got[3][n][5].abs().sum() == 0, n


def _split3(v: torch.Tensor):
    """The adapter kernels' fp32 -> three bf16 parts: hi = bf16(v), mid = bf16(v - hi),
    lo = bf16(v - hi - mid) (csrc/lora_train.cu, the tensor-core rank-down and outer product)."""
    hi = v.to(torch.bfloat16)
    r1 = v - hi.float()
    mid = r1.to(torch.bfloat16)
    lo = (r1 - mid.float()).to(torch.bfloat16)
    return hi, mid, lo


def test_three_part_bf16_split_keeps_fp32_accuracy():
    """The split reconstructs fp32 values to within 2^-24 relative, and a product of bf16 rows with
    the split adapter (each part exact against bf16, summed smallest first) is as close to the
    float64 product as an fp32 matmul is."""
    g = torch.Generator().manual_seed(0)
    v = torch.randn(200000, generator=g) * torch.logspace(-8, 4, 200000)
    hi, mid, lo = _split3(v)
    rec = hi.double() + mid.double() + lo.double()
    assert ((rec - v.double()).abs() / v.double().abs()).max().item() <= 2.0 ** -24
    x = (torch.randn(256, 2048, generator=g)).to(torch.bfloat16)
    m = torch.randn(2048, 16, generator=g) * 0.01
    exact = x.double() @ m.double()
    parts = [p.double() for p in _split3(m)]
    split = x.double() @ parts[2] + x.double() @ parts[1] + x.double() @ parts[0]
    fp32 = (x.float() @ m).double()
    scale = exact.abs().max()
    err_split = ((split - exact).abs().max() / scale).item()
    err_fp32 = ((fp32 - exact).abs().max() / scale).item()
    assert err_split <= max(4 * err_fp32, 1e-7), (err_split, err_fp32)
