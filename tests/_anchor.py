"""fp32 anchor of a layer computed on the GPU, for shapes the CPU oracle is too slow for.

The module's own NF4 dequantization (bit-exact against oracle/nf4.py, see
test_gpu_kernels) gives fp32 expert weights, one hit expert at a time; the
products run as fp32 torch matmuls with TF32 off. The arithmetic is the
oracle's fp32 forward (oracle/moe.py ``fp32_oracle``)."""
from __future__ import annotations

import torch


def fp32_anchor_gpu(mod, x, idx, w, lora=None):
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.zeros(x.shape[0], mod.hidden_dim, dtype=torch.float32, device=x.device)
        xf = x.float()
        for e in torch.unique(idx).tolist():
            tok, pos = torch.where(idx == e)
            wgu = mod._dequantize_expert(mod.gate_up_proj, mod.gate_up_absmax, mod._gate_up_shape, e, torch.float32)
            wdn = mod._dequantize_expert(mod.down_proj, mod.down_absmax, mod._down_shape, e, torch.float32)
            h = xf[tok] @ wgu.t()
            if lora is not None:
                h = h + lora[4] * ((xf[tok] @ lora[0][e].float().t()) @ lora[1][e].float().t())
            if mod.has_gate:
                gg, u = h.chunk(2, -1)
                h = torch.nn.functional.silu(gg) * u
            else:
                h = torch.nn.functional.silu(h)
            d = h @ wdn.t()
            if lora is not None:
                d = d + lora[4] * ((h @ lora[2][e].float().t()) @ lora[3][e].float().t())
            out.index_add_(0, tok, d * w[tok, pos, None].float())
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
