"""GPU: the dgrad kernel (``e4b_grouped_nf4_dgrad``, tcgen05 with the decoded weights as an
MN-major operand) against the fp32 product with the dequantized NF4 stack, per expert segment.

dx[r] = dy[r] . W_e is the input gradient of the frozen projection that the reference's
fused_grouped_lora backward computes with its dgrad kernel (engines/fast.py:519-550). Bars:
max relative error <= 1e-2 and mean <= 2e-3 against fp32 (dy enters as fp16 under a per-row
power-of-two scale, W's NF4 values are exact in fp16, accumulation is fp32)."""
from __future__ import annotations

import pytest
import torch

from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _case(e4b, E, N, K, counts, out_dtype=torch.float32, dy_dtype=torch.bfloat16, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w = (torch.randn(E, N, K, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    packed, absmax = e4b.ops.nf4_quantize(w.reshape(E * N, K))
    packed = packed.view(E, N, K // 2)
    absmax = absmax.view(E, N, K // 64)
    Wd = e4b.ops.nf4_dequantize(packed, absmax, (E, N, K), torch.float32)
    R = sum(counts)
    offsets = torch.tensor([0] + list(torch.tensor(counts).cumsum(0)), dtype=torch.int32, device=DEV)
    dy = (torch.randn(R, N, generator=g, device=DEV) * 0.5).to(dy_dtype)
    dx = e4b.ops.grouped_nf4_dgrad(dy, packed, absmax, offsets, out_dtype=out_dtype)
    torch.cuda.synchronize()
    ref = torch.zeros(R, K, device=DEV)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    for e in range(E):
        a, b = int(offsets[e]), int(offsets[e + 1])
        if b > a:
            ref[a:b] = dy[a:b].float() @ Wd[e]
    torch.backends.cuda.matmul.allow_tf32 = prev
    return dx, ref


@pytest.mark.parametrize("E,N,K,counts", [
    (4, 128, 256, [130, 0, 7, 300]),             # ragged segments, an empty expert, one partial tile
    (8, 1536, 2048, [256] * 8),                  # Qwen3 gate_up geometry (N = 2I): dL/dx
    (8, 2048, 768, [200, 57, 0, 512, 1, 128, 129, 64]),  # Qwen3 down geometry (N = H): dL/dh
])
def test_dgrad_matches_fp32_product(e4b, E, N, K, counts):
    dx, ref = _case(e4b, E, N, K, counts)
    assert dx.dtype == torch.float32
    mx, mean = M.rel_errors(dx.cpu(), ref.cpu())
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


def test_dgrad_bf16_out_and_fp16_in_deterministic(e4b):
    dx, ref = _case(e4b, 3, 192, 512, [100, 300, 20], out_dtype=torch.bfloat16, dy_dtype=torch.float16, seed=3)
    assert dx.dtype == torch.bfloat16
    mx, mean = M.rel_errors(dx.float().cpu(), ref.cpu())
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)
    again, _ = _case(e4b, 3, 192, 512, [100, 300, 20], out_dtype=torch.bfloat16, dy_dtype=torch.float16, seed=3)
    assert torch.equal(dx, again)


def test_dgrad_refuses_unsupported_shapes(e4b):
    packed = torch.zeros(2, 96, 128, dtype=torch.uint8, device=DEV)   # N = 96 is not a multiple of 64
    absmax = torch.ones(2, 96, 4, device=DEV)
    offsets = torch.tensor([0, 3, 5], dtype=torch.int32, device=DEV)
    with pytest.raises(e4b._native.E4BError):
        e4b.ops.grouped_nf4_dgrad(torch.zeros(5, 96, dtype=torch.bfloat16, device=DEV), packed, absmax, offsets)
