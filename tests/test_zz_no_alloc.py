"""GPU: e4b_moe_forward_static, the layer entry point for callers that cannot allocate.

Callers such as a serving runtime that owns every device allocation, or a plugin
host that forbids cudaMalloc once started, cannot hand the library a workspace.
e4b_moe_forward_static runs the same fused expert layer on a fixed device array
inside the library. Here it is called through the C ABI, twice on the same
inputs with a call on another layer shape in between (the array keeps whatever
that call left behind), and each result must equal the workspace entry point
e4b_moe_forward bit for bit: the same kernels run on the same bytes. This file
is collected last on purpose.
"""
import ctypes

import pytest
import torch

from oracle import moe as M
from oracle.nf4 import quantize_stack

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
MAX_REL, MEAN_REL = 1e-2, 2e-3


def _layer(E, H, I, k, T, seed):
    g = torch.Generator().manual_seed(seed)
    gp, ga = quantize_stack(torch.randn(E, 2 * I, H, generator=g) * 0.02)
    dp, da = quantize_stack(torch.randn(E, H, I, generator=g) * 0.02)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    idx = torch.stack([torch.randperm(E, generator=g)[:k] for _ in range(T)])
    w = torch.rand(T, k, generator=g)
    return [t.to(DEV) for t in (x, idx, w, gp, ga, dp, da)]


def _static_call(e4b, x, idx, w, gp, ga, dp, da, E, I):
    N = e4b._native
    T, H = x.shape
    k = idx.shape[1]
    out = torch.empty(T, H, dtype=torch.bfloat16, device=DEV)
    d = e4b.ops.MoeDesc_from(E, H, I, k, T, True, x.dtype, w.dtype, out.dtype, None)
    t = N.MoeTensors()
    t.hidden, t.topk_idx, t.topk_w = x.data_ptr(), idx.data_ptr(), w.data_ptr()
    t.gate_up_packed, t.gate_up_absmax = gp.data_ptr(), ga.data_ptr()
    t.down_packed, t.down_absmax = dp.data_ptr(), da.data_ptr()
    t.out = out.data_ptr()
    st = N.lib().e4b_moe_forward_static(ctypes.byref(d), ctypes.byref(t), N.stream_handle(DEV))
    return st, out


SHAPES = [(64, 2048, 1024, 8, 1), (16, 256, 128, 4, 33), (32, 1024, 512, 4, 300)]


@pytest.mark.parametrize("case", range(len(SHAPES)))
def test_static_scratch_matches_workspace_entry_point_twice(e4b, case):
    E, H, I, k, T = SHAPES[case]
    x, idx, w, gp, ga, dp, da = _layer(E, H, I, k, T, seed=E + T)
    ref = e4b.ops.moe_forward(x, idx, w, gp, ga, dp, da, E, I)
    oE, oH, oI, ok, oT = SHAPES[(case + 1) % len(SHAPES)]
    other = _layer(oE, oH, oI, ok, oT, seed=7)
    other_ref = e4b.ops.moe_forward(*other, oE, oI)
    for _ in range(2):
        st, out = _static_call(e4b, x, idx, w, gp, ga, dp, da, E, I)
        assert st == 0, e4b._native.status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out, ref)
        mx, mean = M.rel_errors(out, ref)
        assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)
        st, out2 = _static_call(e4b, *other, oE, oI)  # another shape leaves its scratch behind
        assert st == 0, e4b._native.status_string(st)
        torch.cuda.synchronize()
        assert torch.equal(out2, other_ref)


def test_static_scratch_refuses_layers_beyond_its_size(e4b):
    E, H, I, k, T = 8, 4096, 2048, 2, 2048      # needs tens of MiB of scratch
    N = e4b._native
    d = e4b.ops.MoeDesc_from(E, H, I, k, T, True, torch.bfloat16, torch.float32, torch.bfloat16, None)
    assert N.lib().e4b_moe_workspace_bytes(ctypes.byref(d)) > (16 << 20)
    t = N.MoeTensors()
    st = N.lib().e4b_moe_forward_static(ctypes.byref(d), ctypes.byref(t), N.stream_handle(DEV))
    assert st == 9 and "static" in N.status_string(st)
