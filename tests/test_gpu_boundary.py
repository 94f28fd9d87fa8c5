"""GPU: the drop-in boundary around the fused layer.

* A device error (fp16 saturation of h) recorded by one patched call surfaces
  through a later patched call with ``E4B_CHECK_ERRORS`` unset, although a clean
  layer ran in between (the error word is sticky, the read is asynchronous).
* A base with its own activation hook (``_apply_gate``: a clamped SwiGLU, as
  DeepSeek-V4's experts) is patched, bare and inside ``ExpertsLoRA``, and runs
  the epilogue route: grouped GEMM, the base's epilogue, grouped GEMM, combine
  (reference engines/fast.py:137-156, :214-257, :320-347).
* A CUDA graph captured before the workspace cache grows replays unchanged.
* Mis-shaped or misplaced tensors are refused before any kernel sees them.
"""
from __future__ import annotations

import pytest
import torch
import torch.nn.functional as F

from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _stack(E, H, I, seed, scale=0.02):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gu = (torch.randn(E, 2 * I, H, generator=g, device=DEV) * scale).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g, device=DEV) * scale).to(torch.bfloat16)
    return gu, dn


def _route(E, T, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device=DEV), -1), k)
    return w, idx


def test_sticky_device_error_surfaces_on_a_later_patched_call(e4b):
    E, H, I, k, T = 16, 512, 256, 2, 4
    gu, dn = _stack(E, H, I, seed=1)
    mod = e4b.Experts4bit.from_float(gu, dn, compute_dtype=torch.bfloat16).eval()
    assert e4b.enable_fast(mod) == 1
    w, idx = _route(E, T, k, seed=2)
    g = torch.Generator(device=DEV).manual_seed(3)
    clean = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    huge = (clean.float() * 4000).to(torch.bfloat16)  # h = silu(gate) * up far beyond +-65504
    raised = None
    with torch.no_grad():
        mod(clean, idx, w)
        torch.cuda.synchronize()
        try:
            mod(huge, idx, w)      # records E4B_ERR_RANGE; no host sync, so nothing raises here
            mod(clean, idx, w)     # a clean layer after it
            torch.cuda.synchronize()
            mod(clean, idx, w)     # by now the asynchronous read has landed
        except e4b._native.E4BError as e:
            raised = e
    assert raised is not None and raised.status == e4b._native.E4B_ERR_RANGE
    with torch.no_grad():          # reported once: the read cleared the word
        mod(clean, idx, w)
        torch.cuda.synchronize()
        mod(clean, idx, w)
    e4b.check_errors()


def test_error_word_is_sticky_across_clean_calls(e4b, monkeypatch):
    """The kernels only ever set the word (first error wins); a clean call leaves it as it is."""
    E, H, I, k, T = 16, 512, 256, 2, 4
    gu, dn = _stack(E, H, I, seed=21)
    mod = e4b.Experts4bit.from_float(gu, dn)
    w, idx = _route(E, T, k, seed=22)
    clean = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    huge = (clean.float() * 4000).to(torch.bfloat16)
    monkeypatch.setattr(e4b._native.error_watch, "before", lambda ws, what: None)
    monkeypatch.setattr(e4b._native.error_watch, "after", lambda ws, what="": None)
    ws = torch.zeros(1 << 24, dtype=torch.uint8, device=DEV)
    args = (mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, E, I)
    for T_ in (4, 1):  # the flow kernel (T=1) and the multi-kernel path's shapes alike
        e4b.ops.moe_forward(huge[:T_], idx[:T_], w[:T_], *args, workspace=ws)
        e4b.ops.moe_forward(clean[:T_], idx[:T_], w[:T_], *args, workspace=ws)
        assert e4b._native.read_device_error(ws) == e4b._native.E4B_ERR_RANGE
        e4b.ops.moe_forward(clean[:T_], idx[:T_], w[:T_], *args, workspace=ws)
        assert e4b._native.read_device_error(ws) == 0


def test_check_errors_raises_at_once(e4b):
    E, H, I, k, T = 16, 512, 256, 2, 4
    gu, dn = _stack(E, H, I, seed=4)
    mod = e4b.Experts4bit.from_float(gu, dn).eval()
    e4b.enable_fast(mod)
    w, idx = _route(E, T, k, seed=5)
    x = (torch.randn(T, H, device=DEV) * 4000).to(torch.bfloat16)
    with torch.no_grad():
        mod(x, idx, w)
    with pytest.raises(e4b._native.E4BError):
        e4b.check_errors()
    e4b.check_errors()  # cleared


def _clamped_class(e4b, limit=0.3):
    class ClampedExperts(e4b.Experts4bit):
        """A base whose activation is a clamped SwiGLU and whose forward is its own loop."""

        def _apply_gate(self, proj):
            g, u = proj.chunk(2, -1)
            return F.silu(g.clamp(max=limit)) * u.clamp(-limit, limit)

        def forward(self, x, idx, w):
            out = torch.zeros(x.shape, dtype=torch.float32, device=x.device)
            for e in torch.unique(idx).tolist():
                tok, pos = torch.where(idx == e)
                proj = self._project(self.gate_up_proj, self.gate_up_absmax, self._gate_up_shape, e, x[tok], x.dtype)
                h = self._apply_gate(proj)
                d = self._project(self.down_proj, self.down_absmax, self._down_shape, e, h, x.dtype)
                out.index_add_(0, tok, (d * w[tok, pos, None]).float())
            return out.to(x.dtype)

    return ClampedExperts


def _clamped_anchor(mod, x, idx, w, limit=0.3, lora=None):
    out = torch.zeros(x.shape[0], mod.hidden_dim, dtype=torch.float32, device=DEV)
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        for e in torch.unique(idx).tolist():
            tok, pos = torch.where(idx == e)
            wgu = mod._dequantize_expert(mod.gate_up_proj, mod.gate_up_absmax, mod._gate_up_shape, e, torch.float32)
            wdn = mod._dequantize_expert(mod.down_proj, mod.down_absmax, mod._down_shape, e, torch.float32)
            xf = x[tok].float()
            p = xf @ wgu.t()
            if lora is not None:
                p = p + lora[4] * ((xf @ lora[0][e].float().t()) @ lora[1][e].float().t())
            g, u = p.chunk(2, -1)
            h = F.silu(g.clamp(max=limit)) * u.clamp(-limit, limit)
            d = h @ wdn.t()
            if lora is not None:
                d = d + lora[4] * ((h @ lora[2][e].float().t()) @ lora[3][e].float().t())
            out.index_add_(0, tok, d * w[tok, pos, None].float())
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev
    return out


@pytest.mark.parametrize("T", [1, 5, 300])
def test_apply_gate_base_is_patched_and_fused(e4b, T):
    E, H, I, k = 16, 1024, 512, 4
    gu, dn = _stack(E, H, I, seed=6)
    cls = _clamped_class(e4b)
    mod = cls.from_float(gu, dn).eval()
    w, idx = _route(E, T, k, seed=7)
    x = torch.randn(T, H, generator=torch.Generator(device=DEV).manual_seed(8), device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        loop = mod(x, idx, w)
    assert e4b.enable_fast(mod) == 1
    with torch.no_grad():
        got = mod(x, idx, w)
    anchor = _clamped_anchor(mod, x, idx, w)
    mx, mean = M.rel_errors(got.float(), anchor)
    mx_ref, mean_ref = M.rel_errors(loop.float(), anchor)
    # the epilogue route keeps the reference's bf16 intermediate (as engines/fast.py:137-156), so
    # it is held to the reference's own bars against the loop's error, not the fused layer's
    assert mx <= 1e-2 and mean <= max(2 * mean_ref, 2e-3), (mx, mean, mean_ref)
    assert mx <= max(2 * mx_ref, 5e-3)
    # the clamp is load-bearing: a plain SwiGLU is far off
    plain = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax,
                                E, I)
    assert M.rel_errors(plain.float(), anchor)[1] > 10 * max(mean, 1e-4)
    assert e4b.disable_fast(mod) == 1


def test_apply_gate_base_inside_lora_wrapper(e4b):
    E, H, I, k, T, r = 16, 1024, 512, 4, 40, 8
    gu, dn = _stack(E, H, I, seed=9)
    base = _clamped_class(e4b).from_float(gu, dn)
    lm = e4b.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.bfloat16).to(DEV).eval()
    g = torch.Generator(device=DEV).manual_seed(10)
    with torch.no_grad():
        for p in (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B):
            p.copy_(torch.randn(p.shape, generator=g, device=DEV) * 0.05)
    w, idx = _route(E, T, k, seed=11)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    assert e4b.enable_fast(lm) == 1
    with torch.no_grad():
        got = lm(x, idx, w)
    lora = (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B, lm.scaling)
    anchor = _clamped_anchor(base, x, idx, w, lora=lora)
    with torch.no_grad():
        e4b.disable_fast(lm)
        loop = lm(x, idx, w)
    mx, mean = M.rel_errors(got.float(), anchor)
    mx_ref, mean_ref = M.rel_errors(loop.float(), anchor)
    assert mx <= 1e-2 and mean <= max(2 * mean_ref, 2e-3), (mx, mean, mean_ref)


def test_graph_survives_workspace_growth(e4b):
    E, H, I, k, T = 16, 1024, 512, 4, 3
    gu, dn = _stack(E, H, I, seed=12)
    mod = e4b.Experts4bit.from_float(gu, dn).eval()
    e4b.enable_fast(mod)
    w, idx = _route(E, T, k, seed=13)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        ref = mod(x, idx, w).clone()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            mod(x, idx, w)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = mod(x, idx, w)
        # a much larger call grows the cached workspace; the old buffer must stay alive
        big_T = 4096
        wb, ib = _route(E, big_T, k, seed=14)
        mod(torch.randn(big_T, H, device=DEV).to(torch.bfloat16), ib, wb)
        junk = [torch.full((1 << 20,), 7, dtype=torch.int32, device=DEV) for _ in range(8)]  # reuse freed memory
        for _ in range(5):
            out.zero_()
            graph.replay()
            torch.cuda.synchronize()
            assert torch.equal(out, ref)
        del junk


def test_misshaped_tensors_are_refused(e4b):
    E, H, I, k, T = 8, 512, 256, 2, 3
    gu, dn = _stack(E, H, I, seed=15)
    mod = e4b.Experts4bit.from_float(gu, dn)
    w, idx = _route(E, T, k, seed=16)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    args = [mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax]
    f = e4b.ops.moe_forward
    with pytest.raises(ValueError):
        f(x, idx, w, args[0][:-1], *args[1:], E, I)                      # short packed stack
    with pytest.raises(ValueError):
        f(x, idx, w, args[0], args[1].cpu(), *args[2:], E, I)             # absmax on the host
    with pytest.raises(ValueError):
        f(x, idx[:-1], w, *args, E, I)                                    # index rows != tokens
    with pytest.raises(ValueError):
        f(x, idx, w[:, :1], *args, E, I)                                  # weights [T, 1]
    with pytest.raises(ValueError):
        f(x, idx, w, *args, E, I, out=torch.empty(T, H + 8, dtype=torch.bfloat16, device=DEV))
    lora = (torch.zeros(E, 4, H, device=DEV), torch.zeros(E, 2 * I, 4, device=DEV, dtype=torch.bfloat16),
            torch.zeros(E, 4, I, device=DEV), torch.zeros(E, H, 4, device=DEV), 1.0)
    with pytest.raises(ValueError):
        f(x, idx, w, *args, E, I, lora=lora)                              # mixed adapter dtypes
