"""GPU: the fused layer at the benchmarked shapes, against an fp32 anchor.

* Qwen3-30B-A3B geometry (E=128, H=2048, I=768, top-8) at T=4096 with LoRA r=16
  adapters (bf16, N(0, 0.01)): the tcgen05 kernels with ~256 rows per expert.
* Mixtral-8x7B geometry (E=8, H=4096, I=14336, top-2) at T=8192: the K=14336
  down-projection loop and 2048-row experts.
* DeepSeek-V3 geometry with FP8 e4m3 128x128 blocks (E=256, H=7168, I=2048,
  top-8, Zipf(1.1) expert popularity) at T=64 (decode GEMV) and T=2048 (tcgen05).

The anchor dequantizes each hit expert to fp32 on the device (bit-exact codecs)
and runs fp32 matmuls with TF32 off. Bars: max-rel <= 1e-2 and mean-rel <= 2e-3
(norm-relative), the layer tolerance of this path.
"""
from __future__ import annotations

import pytest
import torch

from _anchor import fp32_anchor_gpu
from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _routes(E, T, k, g, zipf=False):
    logits = torch.randn(T, E, generator=g, device=DEV)
    if zipf:
        perm = torch.randperm(E, generator=g, device=DEV)
        pop = torch.empty(E, device=DEV)
        pop[perm] = 1.0 / torch.arange(1, E + 1, device=DEV, dtype=torch.float32) ** 1.1
        logits = logits + torch.log(pop)
    return torch.topk(torch.softmax(logits, -1), k)


def test_qwen3_prefill_t4096_lora16(e4b):
    E, H, I, k, T, r = 128, 2048, 768, 8, 4096, 16
    g = torch.Generator(device=DEV).manual_seed(30)
    gu = (torch.randn(E, 2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    base = e4b.Experts4bit.from_float(gu, dn)
    del gu, dn
    lm = e4b.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.bfloat16).to(DEV).eval()
    with torch.no_grad():
        for p in (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B):
            p.copy_(torch.randn(p.shape, generator=g, device=DEV) * 0.01)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    w, idx = _routes(E, T, k, g)
    assert e4b.ops.moe_path(E, H, I, k, T, lora_rank=r) == e4b._native.PATH_TENSOR_CORE
    assert e4b.enable_fast(lm) == 1
    with torch.no_grad():
        got = lm(x, idx, w)
    lora = (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B, lm.scaling)
    anchor = fp32_anchor_gpu(base, x, idx, w, lora)
    mx, mean = M.rel_errors(got.float(), anchor)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)
    # the adapters are load-bearing at this scale
    plain = fp32_anchor_gpu(base, x, idx, w)
    assert M.rel_errors(plain, anchor)[1] > 5 * mean


def test_mixtral_t8192(e4b):
    E, H, I, k, T = 8, 4096, 14336, 2, 8192
    g = torch.Generator(device=DEV).manual_seed(31)
    mod = e4b.Experts4bit(E, H, I, device=DEV)
    with torch.no_grad():  # quantize expert by expert (the bf16 stack would be 2.8 GB)
        gp = mod.gate_up_proj.view(E, -1)
        ga = mod.gate_up_absmax.view(E, -1)
        dp = mod.down_proj.view(E, -1)
        da = mod.down_absmax.view(E, -1)
        for e in range(E):
            p, a = e4b.ops.nf4_quantize((torch.randn(2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16))
            gp[e].copy_(p)
            ga[e].copy_(a)
            p, a = e4b.ops.nf4_quantize((torch.randn(H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16))
            dp[e].copy_(p)
            da[e].copy_(a)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    w, idx = _routes(E, T, k, g)
    got = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, E, I,
                              check_errors=True)
    anchor = fp32_anchor_gpu(mod, x, idx, w)
    mx, mean = M.rel_errors(got.float(), anchor)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


def _fp8_anchor(mod, x, idx, w):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.zeros(x.shape[0], mod.hidden_dim, dtype=torch.float32, device=DEV)
        for e in torch.unique(idx).tolist():
            tok, pos = torch.where(idx == e)
            wgu = mod.dequantize_expert("gate_up", e, torch.float32)
            wdn = mod.dequantize_expert("down", e, torch.float32)
            gg, u = (x[tok].float() @ wgu.t()).chunk(2, -1)
            d = (torch.nn.functional.silu(gg) * u) @ wdn.t()
            out.index_add_(0, tok, d * w[tok, pos, None].float())
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.fixture(scope="module")
def deepseek_fp8(e4b):
    E, H, I = 256, 7168, 2048
    g = torch.Generator(device=DEV).manual_seed(32)
    mod = e4b.ExpertsFp8Blocks(E, H, I, device=DEV)
    f8 = e4b.fp8_experts
    with torch.no_grad():  # expert by expert: the bf16 stacks would take 22 GB
        for e in range(E):
            q, s = f8.quantize_fp8_blocks((torch.randn(2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16))
            mod.gate_up_proj[e].copy_(q)
            mod.gate_up_scale[e].copy_(s)
            q, s = f8.quantize_fp8_blocks((torch.randn(H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16))
            mod.down_proj[e].copy_(q)
            mod.down_scale[e].copy_(s)
    yield mod
    del mod
    torch.cuda.empty_cache()


@pytest.mark.parametrize("T", [64, 2048])
def test_deepseek_fp8_zipf(e4b, deepseek_fp8, T):
    mod = deepseek_fp8
    E, H, I, k = 256, 7168, 2048, 8
    g = torch.Generator(device=DEV).manual_seed(33 + T)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    w, idx = _routes(E, T, k, g, zipf=True)
    gs, ds = mod.scale_values()
    got = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, gs, mod.down_proj, ds, E, I, check_errors=True,
                              weight_format=e4b._native.FMT_FP8_BLOCK128)
    anchor = _fp8_anchor(mod, x, idx, w)
    mx, mean = M.rel_errors(got.float(), anchor)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)
