"""GPU: expert residency engines over the fused layer.

Hot experts stay in a resident device sub-stack; the others are read from a pinned
host arena through the address table (``e4b_gather_expert_rows``). The layer runs
the same fused kernels over the same NF4 bytes, so it must equal the fused layer
on the full stack bit for bit in the decode regime (the flow kernel's arithmetic
does not depend on where an expert's rows sit in the stack), and meet the layer
tolerance against the fp32 anchor in prefill (with an expert map over the
resident / staged rows). Reference: engines/hot_residency.py, engines/pipelined.py.
"""
from __future__ import annotations

import pytest
import torch

from _anchor import fp32_anchor_gpu
from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _module(e4b, E=64, H=2048, I=1024, seed=0):
    g = torch.Generator(device=DEV).manual_seed(seed)
    gu = (torch.randn(E, 2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    return e4b.Experts4bit.from_float(gu, dn).eval()


def _route(E, T, k, seed):
    g = torch.Generator(device=DEV).manual_seed(seed)
    w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device=DEV), -1), k)
    return w, idx


@pytest.mark.parametrize("hot", [[], [1, 5, 9, 33], list(range(64))])
def test_pipelined_decode_equals_full_stack(e4b, hot):
    E, H, I, k = 64, 2048, 1024, 8
    mod = _module(e4b)
    assert e4b.enable_pipelined_residency(mod, [torch.tensor(hot)], k_slots=k) == 1
    outs = []
    for step in range(6):  # slot caching: repeated and changing expert sets
        w, idx = _route(E, 1, k, seed=step // 2)
        x = torch.randn(1, H, device=DEV).to(torch.bfloat16)
        with torch.no_grad():
            got = mod(x, idx, w)
        full = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj,
                                   mod.down_absmax, E, I, check_errors=True)
        assert torch.equal(got, full), step
        outs.append(got)
    assert e4b.disable_pipelined_residency(mod) == 1


def test_pipelined_decode_captures_in_a_graph(e4b):
    E, H, I, k = 64, 2048, 1024, 8
    mod = _module(e4b, seed=1)
    e4b.enable_pipelined_residency(mod, [torch.tensor([3, 4])], k_slots=k)
    x = torch.zeros(1, H, dtype=torch.bfloat16, device=DEV)
    w = torch.zeros(1, k, device=DEV)
    idx = torch.zeros(1, k, dtype=torch.int64, device=DEV)
    with torch.no_grad():
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            mod(x, idx, w)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = mod(x, idx, w)
        for step in range(5):
            wv, iv = _route(E, 1, k, seed=100 + step)
            xv = torch.randn(1, H, device=DEV).to(torch.bfloat16)
            x.copy_(xv)
            w.copy_(wv)
            idx.copy_(iv)
            graph.replay()
            full = e4b.ops.moe_forward(xv, iv, wv, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj,
                                       mod.down_absmax, E, I)
            torch.cuda.synchronize()
            assert torch.equal(out, full), step


@pytest.mark.parametrize("T", [4, 64, 600])
def test_hot_residency_prefill_and_decode(e4b, T):
    E, H, I, k = 64, 2048, 1024, 8
    mod = _module(e4b, seed=2)
    hot = torch.tensor([0, 7, 12, 40, 41, 63])
    assert e4b.enable_hot_residency(mod, [hot]) == 1
    w, idx = _route(E, T, k, seed=3)
    x = torch.randn(T, H, device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        got = mod(x, idx, w)
        one = mod(x[:1], idx[:1], w[:1])  # a decode step after a prefill reuses the stacks
    anchor = fp32_anchor_gpu(mod, x, idx, w)
    mx, mean = M.rel_errors(got.float(), anchor)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)
    full1 = e4b.ops.moe_forward(x[:1], idx[:1], w[:1], mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj,
                                mod.down_absmax, E, I)
    assert torch.equal(one, full1)
    assert e4b.disable_hot_residency(mod) == 1


def test_gather_reports_bad_ids_and_skips_held_slots(e4b):
    import ctypes
    N = e4b._native
    E, rows, slots = 6, 48, 3
    seg_bytes = [32, 16, 64, 16]
    seg_off = [0, 32, 48, 112]
    row_bytes = 128
    arena = torch.arange(E * row_bytes, dtype=torch.int64).remainder(251).to(torch.uint8).view(E, row_bytes)
    arena = arena.pin_memory()
    table = (torch.arange(E, dtype=torch.int64) * row_bytes + arena.data_ptr()).to(DEV)
    stacks = [torch.zeros(slots, b, dtype=torch.uint8, device=DEV) for b in seg_bytes]
    ids = torch.tensor([2, 5, 1], device=DEV)
    have = torch.tensor([-1, 5, -1], device=DEV)
    local = torch.empty(slots, dtype=torch.int64, device=DEV)
    ws = torch.zeros(4096, dtype=torch.uint8, device=DEV)
    arr = lambda t, v: ctypes.cast((t * 4)(*v), ctypes.c_void_p)  # noqa: E731
    N.check(N.lib().e4b_gather_expert_rows(table.data_ptr(), E, ids.data_ptr(), have.data_ptr(), slots, None, 0,
                                           local.data_ptr(), arr(ctypes.c_uint64, seg_off),
                                           arr(ctypes.c_uint64, seg_bytes),
                                           arr(ctypes.c_void_p, [s.data_ptr() for s in stacks]), ws.data_ptr(),
                                           ws.numel(), N.stream_handle(torch.device(DEV))), "gather")
    torch.cuda.synchronize()
    assert local.tolist() == [0, 1, 2] and have.tolist() == [2, 5, 1]
    for s, (o, b) in enumerate(zip(seg_off, seg_bytes)):
        assert torch.equal(stacks[s][0].cpu(), arena[2, o:o + b])
        assert torch.equal(stacks[s][2].cpu(), arena[1, o:o + b])
        assert not stacks[s][1].any()  # slot 1 already held expert 5: not copied
    bad = torch.tensor([0, E + 1, 3], device=DEV)
    N.lib().e4b_gather_expert_rows(table.data_ptr(), E, bad.data_ptr(), have.data_ptr(), slots, None, 0,
                                   local.data_ptr(), arr(ctypes.c_uint64, seg_off), arr(ctypes.c_uint64, seg_bytes),
                                   arr(ctypes.c_void_p, [s.data_ptr() for s in stacks]), ws.data_ptr(), ws.numel(),
                                   N.stream_handle(torch.device(DEV)))
    assert N.read_device_error(ws) == N.E4B_ERR_EXPERT_INDEX
    del rows


def test_residency_rules(e4b):
    mod = _module(e4b, E=8, H=512, I=256, seed=4)
    with pytest.raises(ValueError):
        e4b.enable_pipelined_residency(mod, [torch.tensor([1])])          # k_slots required
    with pytest.raises(ValueError):
        e4b.enable_pipelined_residency(mod, [], k_slots=2)                # one hot set per module
    with pytest.raises(ValueError):
        e4b.enable_hot_residency(mod, [torch.tensor([8])])                # id out of range
    e4b.enable_fast(mod)
    assert e4b.enable_pipelined_residency(mod, [torch.tensor([1])], k_slots=2) == 0  # another patch active
    e4b.disable_fast(mod)
    lm = e4b.ExpertsLoRA(mod, r=4).to(DEV).eval()
    assert e4b.enable_hot_residency(lm, [torch.tensor([1])]) == 0        # a wrapped base: v0 skips it
    assert e4b.enable_pipelined_residency(lm, [torch.tensor([1])], k_slots=2) == 1  # reached through the wrapper
    w, idx = _route(8, 1, 2, seed=5)
    x = torch.randn(1, 512, device=DEV).to(torch.bfloat16)
    with torch.no_grad():
        got = lm(x, idx, w)
    full = e4b.ops.moe_forward(x, idx, w, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, 8, 256)
    assert torch.equal(got, full)
