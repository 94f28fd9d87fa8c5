"""MXFP4 dequantization: the oracle restatement and the library against the reference's
own ``dequantize_mxfp4`` outputs (tests/golden/mxfp4.npz, made by
tests/golden/make_mxfp4_golden.py), bit for bit in bf16, fp16 and fp32."""
import importlib
import os

import numpy as np
import pytest
import torch

from oracle import mxfp4 as OM

HERE = os.path.dirname(os.path.abspath(__file__))
G = np.load(os.path.join(HERE, "golden", "mxfp4.npz"))
DTYPES = [(torch.bfloat16, "bf16", torch.int16), (torch.float16, "f16", torch.int16), (torch.float32, "f32", torch.int32)]


def _bits(t, view):
    return t.contiguous().view(view).cpu().numpy()


@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_oracle_matches_reference(case, dt, tag, view):
    v = OM.dequantize_mxfp4_f32(G[f"{case}_blocks"], G[f"{case}_scales"])
    got = torch.from_numpy(v).to(dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_host_library_matches_reference(e4b, case, dt, tag, view):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    got = mx.dequantize_mxfp4(torch.from_numpy(G[f"{case}_blocks"]), torch.from_numpy(G[f"{case}_scales"]), dtype=dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


def test_byte_reinterpretation_and_shape_errors(e4b):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    b, s = torch.from_numpy(G["single_blocks"]), torch.from_numpy(G["single_scales"])
    ref = mx.dequantize_mxfp4(b, s)
    assert torch.equal(mx.dequantize_mxfp4(b.view(torch.int8), s), ref)  # int8-labelled blocks: same bytes
    with pytest.raises(ValueError):
        mx.dequantize_mxfp4(b, s[:, :1])
    with pytest.raises(ValueError):
        mx.dequantize_mxfp4(b[0], s[0])


@pytest.mark.gpu
@pytest.mark.parametrize("case", ["stack", "single"])
@pytest.mark.parametrize("dt,tag,view", DTYPES)
def test_device_kernel_matches_reference(e4b, case, dt, tag, view):
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    got = mx.dequantize_mxfp4(torch.from_numpy(G[f"{case}_blocks"]).cuda(),
                              torch.from_numpy(G[f"{case}_scales"]).cuda(), dtype=dt)
    assert np.array_equal(_bits(got, view), G[f"{case}_{tag}"])


def test_scales_on_another_device_are_refused(e4b):
    """Scales on another device than the blocks are refused before any pointer reaches a kernel."""
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    b, s = torch.from_numpy(G["single_blocks"]), torch.from_numpy(G["single_scales"])
    with pytest.raises(ValueError, match="blocks on"):
        mx.dequantize_mxfp4(b, s.to("meta"))


def test_scale_255_follows_ldexp():
    """e8m0 255 is 2**128: 0.5 * 2**128 stays finite, codes >= 1 overflow, zero codes stay zeros."""
    blocks = np.array([[[0x10, 0x8A]]], dtype=np.uint8)   # codes (lo, hi): 0, 0.5 | -1.0, -0.0
    v = OM.dequantize_mxfp4_f32(blocks, np.array([[255]], dtype=np.uint8)).reshape(-1)
    assert v[0] == 0 and not np.signbit(v[0])
    assert v[1] == np.float32(2.0 ** 127)
    assert v[2] == -np.inf
    assert v[3] == 0 and np.signbit(v[3])


def test_quantizer_and_module_reference_loop(e4b):
    """The MXFP4 module's reference loop is the NF4 module's loop over MXFP4-dequantized weights."""
    from oracle import moe as M
    mx = importlib.import_module("experts4bit-qlora_b200.mxfp4")
    g = torch.Generator().manual_seed(3)
    E, H, I, k, T = 4, 128, 128, 2, 5
    gu = (torch.randn(E, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    m = mx.ExpertsMxfp4.from_float(gu, dn)
    assert m.gate_up_proj.shape == (E, 2 * I * H // 2) and m.gate_up_absmax.dtype == torch.uint8
    W = m._dequantize_expert(m.gate_up_proj, m.gate_up_absmax, m._gate_up_shape, 2, torch.float32)
    # every block's scale is the smallest power of two that keeps amax / scale <= 6
    blocks = gu[2].float().reshape(-1, 32)
    sc = torch.exp2(m.gate_up_absmax[2].float() - 127)
    assert torch.all(blocks.abs().amax(1) / sc <= 6) and torch.all(blocks.abs().amax(1) / sc > 3)
    assert torch.all((W.reshape(-1, 32) / sc[:, None]).abs() <= 6)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    got = m(x, idx, w).float()
    Wg = torch.stack([m._dequantize_expert(m.gate_up_proj, m.gate_up_absmax, m._gate_up_shape, e, torch.float32)
                      for e in range(E)])
    Wd = torch.stack([m._dequantize_expert(m.down_proj, m.down_absmax, m._down_shape, e, torch.float32)
                      for e in range(E)])
    ref = torch.zeros(T, H)
    for t in range(T):
        for s in range(k):
            e = int(idx[t, s])
            gg, u = (x[t].float() @ Wg[e].t()).chunk(2)
            ref[t] += w[t, s] * ((torch.nn.functional.silu(gg) * u) @ Wd[e].t())
    mxr, mean = M.rel_errors(got, ref)
    assert mxr <= 2e-2 and mean <= 5e-3, (mxr, mean)


@pytest.mark.gpu
@pytest.mark.parametrize("T", [1, 7, 64, 700])
def test_fused_mxfp4_layer_vs_fp32(e4b, T):
    """The fused MXFP4 layer (bf16 tcgen05 GEMMs over exactly decoded weights) against fp32 math
    on the same dequantized weights, through enable_fast."""
    from oracle import moe as M
    E, H, I, k = 16, 1024, 512, 4
    g = torch.Generator(device="cuda").manual_seed(T)
    gu = (torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16)
    m = e4b.ExpertsMxfp4.from_float(gu, dn).eval()
    x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
    w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device="cuda"), -1), k)
    with torch.no_grad():
        loop = m(x, idx, w)
        assert e4b.enable_fast(m) == 1
        got = m(x, idx, w)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    anchor = torch.zeros(T, H, device="cuda")
    for e in torch.unique(idx).tolist():
        tok, pos = torch.where(idx == e)
        wg = m._dequantize_expert(m.gate_up_proj, m.gate_up_absmax, m._gate_up_shape, e, torch.float32)
        wd = m._dequantize_expert(m.down_proj, m.down_absmax, m._down_shape, e, torch.float32)
        gg, u = (x[tok].float() @ wg.t()).chunk(2, -1)
        anchor.index_add_(0, tok, ((torch.nn.functional.silu(gg) * u) @ wd.t()) * w[tok, pos, None])
    torch.backends.cuda.matmul.allow_tf32 = prev
    mxr, mean = M.rel_errors(got.float(), anchor)
    lmx, lmean = M.rel_errors(loop.float(), anchor)
    # h is rounded to bf16 between the projections, as the reference's MXFP4 lane does
    # (engines/nvme_experts.py:856-862): the reference's bars against its own loop
    assert mxr <= 1e-2 and mean <= max(2 * lmean, 2e-3), (mxr, mean, lmean)
    assert mxr <= max(2 * lmx, 5e-3)
