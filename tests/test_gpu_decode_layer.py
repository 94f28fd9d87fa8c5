"""GPU: the one-launch decode-layer kernels.

Three kernels take the decode regime in one launch: the flow kernel
(decode_flow.cu: per-expert completion counters, k-split warps; up to 8 tokens
and 64 picks), the phase kernel (decode_layer.cu: grid-synchronised phases;
up to 16 tokens and 128 picks) and the slice kernel (decode_layer.cu: units of
one expert x 64 intermediate columns, gate_up then the down strip in the same
CTA; up to 8 tokens), selected with ``set_decode_kernel`` mode 1 / 2 / 3
(mode 0 = the multi-kernel path). The phase kernel runs the streaming GEMV's
arithmetic and must equal the multi-kernel path bit for bit; the flow and slice
kernels sum in another order and must meet the layer tolerance against the
fp32 oracle and agree with the multi-kernel path to 1e-2 / 1e-3 (max / mean
relative). All must be deterministic, capture into a CUDA graph and report
device errors."""
from __future__ import annotations

import pytest
import torch

from oracle import moe as M
from _anchor import fp32_anchor_gpu

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _layer(e4b, E, H, I, has_gate=True, seed=0):
    n1 = 2 * I if has_gate else I
    if E * n1 * H > (1 << 26):  # large stacks: drawn on the device, anchored on the GPU
        g = torch.Generator(device=DEV).manual_seed(seed)
        gu = (torch.randn(E, n1, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
        dn = (torch.randn(E, H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
        return e4b.Experts4bit.from_float(gu, dn, has_gate=has_gate), None
    g = torch.Generator().manual_seed(seed)
    gu = (torch.randn(E, n1, H, generator=g) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g) * 0.02).to(torch.bfloat16)
    mod = e4b.Experts4bit.from_float(gu.to(DEV), dn.to(DEV), has_gate=has_gate)
    st = {"gate_up_packed": mod.gate_up_proj.data.cpu(), "gate_up_absmax": mod.gate_up_absmax.cpu(),
          "down_packed": mod.down_proj.data.cpu(), "down_absmax": mod.down_absmax.cpu(), "E": E, "H": H, "I": I,
          "has_gate": has_gate}
    return mod, st


def _inputs(E, H, T, k, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, idx = M.route_on_host(torch.randn(T, E, generator=g), k)
    return x, idx, w


def _fwd(e4b, mod, x, idx, w, E, I, has_gate=True, out_dtype=None, check=True):
    return e4b.ops.moe_forward(x.to(DEV), idx.to(DEV), w.to(DEV), mod.gate_up_proj, mod.gate_up_absmax,
                               mod.down_proj, mod.down_absmax, E, I, has_gate=has_gate, out_dtype=out_dtype,
                               check_errors=check)


class _Mode:
    def __init__(self, e4b, mode):
        self.e4b, self.mode = e4b, mode

    def __enter__(self):
        self.old = self.e4b._native.lib().e4b_set_decode_kernel(self.mode)

    def __exit__(self, *a):
        self.e4b._native.lib().e4b_set_decode_kernel(self.old)


SHAPES = [(64, 2048, 1024, 8, 1), (64, 2048, 1024, 8, 2), (64, 2048, 1024, 8, 3), (64, 2048, 1024, 8, 4),
          (32, 512, 256, 8, 12), (128, 1024, 512, 4, 8), (64, 2048, 1024, 8, 8), (8, 4096, 14336, 2, 1),
          (128, 2048, 768, 8, 2)]


PHASE_BITEXACT = {(64, 2048, 1024, 8, 1), (64, 2048, 1024, 8, 2), (64, 2048, 1024, 8, 3), (128, 1024, 512, 4, 8)}


@pytest.mark.parametrize("E,H,I,k,T", SHAPES)
def test_decode_layer_vs_multikernel_and_oracle(e4b, E, H, I, k, T):
    mod, st = _layer(e4b, E, H, I)
    x, idx, w = _inputs(E, H, T, k, seed=T)
    with _Mode(e4b, 0):
        assert e4b.ops.moe_path(E, H, I, k, T) == e4b._native.PATH_STREAMING
        multi = _fwd(e4b, mod, x, idx, w, E, I)
    ref = M.fp32_oracle(st, x, idx, w) if st is not None else fp32_anchor_gpu(mod, x.to(DEV), idx.to(DEV), w.to(DEV)).cpu()
    for mode in (1, 2, 3):
        with _Mode(e4b, mode):
            if e4b.ops.moe_path(E, H, I, k, T) != e4b._native.PATH_DECODE_LAYER:
                continue
            fused = _fwd(e4b, mod, x, idx, w, E, I)
            again = _fwd(e4b, mod, x, idx, w, E, I)
        assert torch.equal(fused, again)  # deterministic
        if mode == 2 and (E, H, I, k, T) in PHASE_BITEXACT:
            # the streaming kernel runs the phase kernel's arithmetic on these shapes (its token and
            # h rows fit its 64 KB of shared memory and it takes the same K split); elsewhere it
            # takes the general GEMV, which sums in another order
            assert torch.equal(fused, multi)
        else:
            mx, mean = M.rel_errors(fused.float(), multi.float())
            assert mx <= 1e-2 and mean <= 1e-3, (mode, mx, mean)
        mx, mean = M.rel_errors(fused.float().cpu(), ref)
        assert mx <= 1e-2 and mean <= 2e-3, (mode, mx, mean)


def test_flow_kernel_takes_the_decode_shapes(e4b):
    """Mode 1 takes one token up to a few (its staged token and h rows must fit shared memory);
    the phase kernel takes up to 16 tokens with its 20 KB of token rows."""
    assert e4b.ops.moe_path(64, 2048, 1024, 8, 1) == e4b._native.PATH_DECODE_LAYER
    assert e4b.ops.moe_path(64, 2048, 1024, 8, 4) == e4b._native.PATH_DECODE_LAYER
    assert e4b.ops.moe_path(32, 512, 256, 8, 12) == e4b._native.PATH_DECODE_LAYER
    with _Mode(e4b, 2):
        assert e4b.ops.moe_path(64, 2048, 1024, 8, 4) == e4b._native.PATH_DECODE_LAYER
    with _Mode(e4b, 0):
        assert e4b.ops.moe_path(64, 2048, 1024, 8, 1) == e4b._native.PATH_STREAMING


def test_flow_duplicate_expert_in_one_token(e4b):
    """A token that lists one expert twice gets that expert's output twice (as the reference loop)."""
    E, H, I, k, T = 16, 1024, 512, 4, 3
    mod, st = _layer(e4b, E, H, I, seed=11)
    x, idx, w = _inputs(E, H, T, k, seed=12)
    idx[1, 2] = idx[1, 0]
    got = _fwd(e4b, mod, x, idx, w, E, I)
    mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(st, x, idx, w))
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


def test_decode_layer_silu_only_and_fp32_out(e4b):
    E, H, I, k, T = 16, 512, 256, 4, 3
    mod, st = _layer(e4b, E, H, I, has_gate=False, seed=2)
    x, idx, w = _inputs(E, H, T, k, seed=3)
    assert e4b.ops.moe_path(E, H, I, k, T, has_gate=False) == e4b._native.PATH_DECODE_LAYER
    got = _fwd(e4b, mod, x, idx, w, E, I, has_gate=False, out_dtype=torch.float32)
    assert got.dtype == torch.float32
    mx, mean = M.rel_errors(got.cpu(), M.fp32_oracle(st, x, idx, w))
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


@pytest.mark.parametrize("mode", [2, 3])
def test_decode_layer_graph_capture_and_repeat(e4b, mode):
    with _Mode(e4b, mode):
        _graph_case(e4b)


def _graph_case(e4b):
    E, H, I, k, T = 64, 2048, 1024, 8, 1
    mod, _ = _layer(e4b, E, H, I, seed=4)
    x, idx, w = _inputs(E, H, T, k, seed=5)
    xc, ic, wc = x.to(DEV), idx.to(DEV), w.to(DEV)
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    call = lambda: e4b.ops.moe_forward(xc, ic, wc, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj,  # noqa
                                       mod.down_absmax, E, I, out=out)
    call()
    ref = out.clone()
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        call()
    torch.cuda.current_stream().wait_stream(s)
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph):
        call()
    for _ in range(20):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out, ref)


@pytest.mark.parametrize("mode", [2, 3])
def test_decode_layer_reports_errors_per_call(e4b, mode):
    with _Mode(e4b, mode):
        _errors_case(e4b)


def _errors_case(e4b):
    E, H, I, k, T = 16, 512, 256, 2, 2
    mod, _ = _layer(e4b, E, H, I, seed=6)
    x, idx, w = _inputs(E, H, T, k, seed=7)
    bad = idx.clone()
    bad[0, 0] = E + 3
    with pytest.raises(e4b._native.E4BError) as ei:
        _fwd(e4b, mod, x, bad, w, E, I)
    assert ei.value.status == e4b._native.E4B_ERR_EXPERT_INDEX
    _fwd(e4b, mod, x, idx, w, E, I)  # a valid call afterwards reports nothing


@pytest.mark.parametrize("mode", [1, 2, 3])
@pytest.mark.parametrize("E,H,I,k,T,kind,norm", [(64, 2048, 1024, 8, 1, 0, False), (64, 2048, 1024, 8, 3, 0, True),
                                                 (128, 1024, 512, 4, 8, 1, False), (64, 2048, 1024, 8, 24, 0, False),
                                                 (256, 2048, 512, 8, 4, 0, True)])
def test_decode_step_router_fused_equals_two_calls(e4b, E, H, I, k, T, kind, norm, mode):
    """Router + layer in one launch equals e4b_router_topk followed by e4b_moe_forward bit for bit
    (T=24 is past the one-launch regime: the call falls back to those two)."""
    with _Mode(e4b, mode):
        _router_fused_case(e4b, E, H, I, k, T, kind, norm)


def _router_fused_case(e4b, E, H, I, k, T, kind, norm):
    mod, st = _layer(e4b, E, H, I, seed=T)
    if st is None:
        st = {"gate_up_packed": mod.gate_up_proj.data.cpu(), "gate_up_absmax": mod.gate_up_absmax.cpu(),
              "down_packed": mod.down_proj.data.cpu(), "down_absmax": mod.down_absmax.cpu(), "E": E, "H": H,
              "I": I, "has_gate": True}
    g = torch.Generator().manual_seed(100 + T)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16).to(DEV)
    wr = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16).to(DEV)
    out, w, idx = e4b.ops.moe_decode_step(x, wr, k, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj,
                                          mod.down_absmax, E, I, kind=kind, norm_topk_prob=norm, check_errors=True)
    w2, idx2 = e4b.ops.router_topk(x, wr, k, kind, norm)
    assert torch.equal(idx, idx2) and torch.equal(w, w2)
    ref = e4b.ops.moe_forward(x, idx2, w2, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, E, I,
                              check_errors=True)
    assert torch.equal(out, ref)
    mx, mean = M.rel_errors(out.float().cpu(), M.fp32_oracle(st, x.cpu(), idx.cpu(), w.cpu()))
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


_PW_SCRIPT = r"""
import importlib, sys, torch
sys.path.insert(0, sys.argv[1])
e4b = importlib.import_module("experts4bit-qlora_b200")
E, H, I, k, T = 64, 2048, 1024, 8, 3
g = torch.Generator(device="cuda").manual_seed(7)
mod = e4b.Experts4bit.from_float((torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16),
                                 (torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device="cuda"), -1), k)
out = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, E, I,
                          check_errors=True)
torch.save(out.cpu(), sys.argv[2])
"""


def test_slice_register_decode_is_bit_identical(tmp_path):
    """The slice kernel decodes 0, 1 or 2 words of each block with byte permutes in registers
    (E4B_SLICE_PW) and the rest through the shared pair table: the same fp16 values either way,
    so the layer output is identical bit for bit."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "pw.py"
    script.write_text(_PW_SCRIPT)
    outs = []
    for pw in ("0", "1", "2"):
        path = tmp_path / f"out{pw}.pt"
        env = dict(os.environ, E4B_SLICE_PW=pw, E4B_DECODE_KERNEL="3")
        r = subprocess.run([sys.executable, str(script), root, str(path)], env=env, capture_output=True, text=True,
                           timeout=600)
        assert r.returncode == 0, r.stderr[-2000:]
        outs.append(torch.load(path))
    assert torch.equal(outs[0], outs[1]) and torch.equal(outs[0], outs[2])
