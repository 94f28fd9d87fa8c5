"""Expert-parallel kernels on one GPU: P ranks emulated in one process.

Each emulated rank runs ``e4b_ep_dispatch`` on its token shard and
``e4b_ep_experts`` on its expert slice; the all-to-alls are done with device
index copies that follow the exchange contract of include/e4b.h. The combined
output must equal the single-GPU fused layer bit for bit when both run the same
GEMM regime (every row sees the same kernels), and the fp32 oracle within the
layer tolerance. With two or more GPUs the same layer also runs over NCCL
(tests/ep_worker.py under torchrun)."""
from __future__ import annotations

import os
import socket
import subprocess
import sys

import pytest
import torch

from oracle import moe as M
from oracle.nf4 import quantize_stack

pytestmark = pytest.mark.gpu

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _layer(e4b, E, H, I, seed=0, lora_rank=0):
    g = torch.Generator().manual_seed(seed)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.05).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.05).to(torch.bfloat16)
    mod = e4b.Experts4bit.from_float(gate_up.cuda(), down.cuda())
    if lora_rank:
        mod = e4b.ExpertsLoRA(mod, r=lora_rank, alpha=16, dtype=torch.bfloat16).cuda().eval()
        with torch.no_grad():
            for p in (mod.gate_up_lora_A, mod.gate_up_lora_B, mod.down_lora_A, mod.down_lora_B):
                p.copy_(torch.randn(p.shape, generator=g).to(p.dtype) * 0.05)
    return mod


def _st(mod):
    b = mod.base if hasattr(mod, "base") else mod
    return {"gate_up_packed": b.gate_up_proj.data.cpu(), "gate_up_absmax": b.gate_up_absmax.cpu(),
            "down_packed": b.down_proj.data.cpu(), "down_absmax": b.down_absmax.cpu(), "E": b.num_experts,
            "H": b.hidden_dim, "I": b.intermediate_dim, "has_gate": True}


def _lora_dict(mod):
    if not hasattr(mod, "base"):
        return None
    return {"gate_up_A": mod.gate_up_lora_A.data.cpu(), "gate_up_B": mod.gate_up_lora_B.data.cpu(),
            "down_A": mod.down_lora_A.data.cpu(), "down_B": mod.down_lora_B.data.cpu(), "scaling": mod.scaling}


def emulate_ep(e4b, mod, x, idx, w, P, shard_sizes=None):
    """The expert-parallel layer over P emulated ranks; returns the [T,H] output."""
    from importlib import import_module
    ep = import_module("experts4bit-qlora_b200.ep")
    b = mod.base if hasattr(mod, "base") else mod
    E, H, I = b.num_experts, b.hidden_dim, b.intermediate_dim
    El = E // P
    T = x.shape[0]
    if shard_sizes is None:
        shard_sizes = [T // P + (1 if r < T % P else 0) for r in range(P)]
    bounds = [sum(shard_sizes[:r]) for r in range(P + 1)]
    stages = [ep.NativeStages(ep.shard_experts(mod, r, P), E, H, I, True, P) for r in range(P)]
    sent = []
    for r in range(P):
        t0, t1 = bounds[r], bounds[r + 1]
        send, counts, inv = stages[r].dispatch(x[t0:t1].contiguous(), idx[t0:t1].contiguous())
        sent.append((send, counts.cpu(), inv))
    backs = []
    for q in range(P):
        parts, rc = [], []
        for p in range(P):
            send, counts, _ = sent[p]
            offs = torch.cat([torch.zeros(1, dtype=torch.long), torch.cumsum(counts.long(), 0)])
            parts.append(send[offs[q * El]:offs[(q + 1) * El]])
            rc.append(counts[q * El:(q + 1) * El])
        rows = torch.cat(parts).contiguous()
        recv_counts = torch.stack(rc).cuda()
        backs.append((stages[q].experts(rows, recv_counts), torch.stack(rc)))
    outs = []
    for p in range(P):
        pieces = []
        for q in range(P):
            back, rc = backs[q]
            start = int(rc[:p].sum())
            pieces.append(back[start:start + int(rc[p].sum())])
        ret = torch.cat(pieces).contiguous()
        t0, t1 = bounds[p], bounds[p + 1]
        outs.append(stages[p].combine(ret, sent[p][2], w[t0:t1].contiguous(), t1 - t0, idx.shape[1], x.dtype))
    return torch.cat(outs)


def _inputs(E, H, T, k, seed=1):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    w, idx = M.route_on_host(torch.randn(T, E, generator=g), k, M.SOFTMAX_THEN_TOPK, False)
    return x, idx, w


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_ep_prefill_bitexact_vs_single_gpu(e4b, P):
    E, H, I, k, T = 8, 256, 256, 2, 384
    mod = _layer(e4b, E, H, I)
    x, idx, w = _inputs(E, H, T, k)
    xc, ic, wc = x.cuda(), idx.cuda(), w.cuda()
    single = e4b.ops.moe_forward(xc, ic, wc, *[t for t in (mod.gate_up_proj.data, mod.gate_up_absmax,
                                                            mod.down_proj.data, mod.down_absmax)], E, I,
                                 check_errors=True)
    got = emulate_ep(e4b, mod, xc, ic, wc, P)
    torch.cuda.synchronize()
    assert torch.equal(got, single)
    mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(_st(mod), x, idx, w))
    assert mx <= 1e-2 and mean <= 2e-3


def test_ep_lora_and_ragged_shards(e4b):
    E, H, I, k, T = 8, 256, 128, 2, 200
    mod = _layer(e4b, E, H, I, seed=3, lora_rank=16)
    x, idx, w = _inputs(E, H, T, k, seed=4)
    got = emulate_ep(e4b, mod, x.cuda(), idx.cuda(), w.cuda(), 4, shard_sizes=[0, 17, 150, 33])
    torch.cuda.synchronize()
    ref = M.fp32_oracle(_st(mod), x, idx, w, lora=_lora_dict(mod))
    mx, mean = M.rel_errors(got.float().cpu(), ref)
    assert mx <= 1e-2 and mean <= 2e-3


def test_ep_decode_rows(e4b):
    """A few tokens per rank: the experts take the streaming GEMV on the received rows."""
    E, H, I, k, T = 16, 512, 256, 4, 6
    mod = _layer(e4b, E, H, I, seed=5)
    x, idx, w = _inputs(E, H, T, k, seed=6)
    for P in (2, 4):
        got = emulate_ep(e4b, mod, x.cuda(), idx.cuda(), w.cuda(), P)
        torch.cuda.synchronize()
        mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(_st(mod), x, idx, w))
        assert mx <= 1e-2 and mean <= 2e-3, (P, mx, mean)


def test_ep_skewed_routing_empty_ranks(e4b):
    """Every pick lands on one rank's experts; the other experts receive no rows."""
    E, H, I, k, T = 8, 256, 128, 2, 64
    mod = _layer(e4b, E, H, I, seed=7)
    x, _, w = _inputs(E, H, T, k, seed=8)
    idx = torch.stack([torch.full((T,), 6), torch.full((T,), 7)], 1)
    got = emulate_ep(e4b, mod, x.cuda(), idx.cuda(), w.cuda(), 4)
    torch.cuda.synchronize()
    mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(_st(mod), x, idx, w))
    assert mx <= 1e-2 and mean <= 2e-3


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs for the NCCL exchange")
def test_ep_nccl_two_ranks():
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", os.path.join(ROOT, "tests", "ep_worker.py")]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    r = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert "EP_OK" in r.stdout


def emulate_ep_peer(e4b, mod, x, idx, w, P, shard_sizes=None, layers=1, exchanges=None):
    """The peer-memory layer over P emulated ranks whose exchange regions all live on this GPU.

    Launch order is rank by rank for each step (every dispatch, then every expert side, then every
    combine), so each flag a kernel waits for was set by a kernel that already finished."""
    import ctypes
    from importlib import import_module
    ep = import_module("experts4bit-qlora_b200.ep")
    N = e4b._native
    b = mod.base if hasattr(mod, "base") else mod
    E, H, I = b.num_experts, b.hidden_dim, b.intermediate_dim
    El, k, T = E // P, idx.shape[1], x.shape[0]
    if shard_sizes is None:
        shard_sizes = [T // P + (1 if r < T % P else 0) for r in range(P)]
    bounds = [sum(shard_sizes[:r]) for r in range(P + 1)]
    cap = max(max(shard_sizes), 1) * k
    exs = exchanges or ep.PeerExchange.emulated(P, El, cap, H, x.dtype, x.device)
    stages = [ep.NativeStages(ep.shard_experts(mod, r, P), E, H, I, True, P) for r in range(P)]
    L = N.lib()
    stream = N.stream_handle(x.device)
    outs_all = []
    for _ in range(layers):
        descs = [ex.desc for ex in exs]
        invs, dws = [], []
        for r in range(P):
            t0, t1 = bounds[r], bounds[r + 1]
            inv = torch.empty((t1 - t0) * k, dtype=torch.int32, device=x.device)
            ws = torch.empty(L.e4b_ep_dispatch_peer_workspace_bytes(t1 - t0, k, E), dtype=torch.uint8,
                             device=x.device)
            N.check(L.e4b_ep_dispatch_peer(ctypes.byref(descs[r]), x[t0:t1].data_ptr(), idx[t0:t1].data_ptr(),
                                           t1 - t0, k, inv.data_ptr(), ws.data_ptr(), ws.numel(), stream),
                    "dispatch_peer")
            invs.append(inv)
            dws.append(ws)
        for r in range(P):
            stages[r].experts_peer(exs[r], (bounds[r + 1] - bounds[r]) * k)
        outs = []
        for r in range(P):
            t0, t1 = bounds[r], bounds[r + 1]
            out = torch.empty(t1 - t0, H, dtype=x.dtype, device=x.device)
            wr = w[t0:t1].contiguous()
            N.check(L.e4b_ep_combine_peer(ctypes.byref(descs[r]), invs[r].data_ptr(), wr.data_ptr(),
                                          N.dtype_code(wr.dtype), t1 - t0, k, out.data_ptr(),
                                          N.dtype_code(x.dtype), stream), "combine_peer")
            outs.append(out)
        outs_all.append(torch.cat(outs))
    torch.cuda.synchronize()
    for ex in exs:
        err = ctypes.c_int(-1)
        N.check(L.e4b_read_device_error(ex.region.data_ptr(), stream, ctypes.byref(err)), "read_device_error")
        assert err.value == 0, N.status_string(err.value)
    return outs_all if layers > 1 else outs_all[0]


@pytest.mark.parametrize("P", [1, 2, 4, 8])
def test_ep_peer_prefill_bitexact_vs_single_gpu(e4b, P):
    E, H, I, k, T = 8, 256, 256, 2, 384
    mod = _layer(e4b, E, H, I)
    x, idx, w = _inputs(E, H, T, k)
    xc, ic, wc = x.cuda(), idx.cuda(), w.cuda()
    single = e4b.ops.moe_forward(xc, ic, wc, mod.gate_up_proj.data, mod.gate_up_absmax, mod.down_proj.data,
                                 mod.down_absmax, E, I, check_errors=True)
    got = emulate_ep_peer(e4b, mod, xc, ic, wc, P)
    assert torch.equal(got, single)


def test_ep_peer_lora_ragged_and_repeated_layers(e4b):
    """Ragged shards (one empty), LoRA, three layer calls on the same regions (call numbers 1..3)."""
    E, H, I, k, T = 8, 256, 128, 2, 200
    mod = _layer(e4b, E, H, I, seed=3, lora_rank=16)
    x, idx, w = _inputs(E, H, T, k, seed=4)
    outs = emulate_ep_peer(e4b, mod, x.cuda(), idx.cuda(), w.cuda(), 4, shard_sizes=[0, 17, 150, 33], layers=3)
    ref = M.fp32_oracle(_st(mod), x, idx, w, lora=_lora_dict(mod))
    for got in outs:
        assert torch.equal(got, outs[0])
        mx, mean = M.rel_errors(got.float().cpu(), ref)
        assert mx <= 1e-2 and mean <= 2e-3


def test_ep_peer_matches_nccl_layout_path(e4b):
    """Decode-sized shards and all picks on one rank's experts: same result as the all-to-all path's
    kernels within the layer tolerance, and the fp32 oracle."""
    E, H, I, k, T = 16, 512, 256, 4, 6
    mod = _layer(e4b, E, H, I, seed=5)
    x, idx, w = _inputs(E, H, T, k, seed=6)
    for P in (2, 4):
        got = emulate_ep_peer(e4b, mod, x.cuda(), idx.cuda(), w.cuda(), P)
        mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(_st(mod), x, idx, w))
        assert mx <= 1e-2 and mean <= 2e-3, (P, mx, mean)
    idx2 = torch.stack([torch.full((T,), 14), torch.full((T,), 15), torch.full((T,), 13), torch.full((T,), 12)], 1)
    got = emulate_ep_peer(e4b, mod, x.cuda(), idx2.cuda(), w.cuda(), 4)
    mx, mean = M.rel_errors(got.float().cpu(), M.fp32_oracle(_st(mod), x, idx2, w))
    assert mx <= 1e-2 and mean <= 2e-3


def test_ep_peer_wait_times_out_and_context_survives(e4b):
    """A source that never dispatches: the expert side's bounded wait gives up (a few seconds),
    reports E4B_ERR_TIMEOUT in the region's error word, treats that source as empty, and the
    context keeps working. Nothing else waits on this kernel."""
    import ctypes
    import time
    from importlib import import_module
    ep = import_module("experts4bit-qlora_b200.ep")
    N = e4b._native
    E, H, I = 8, 256, 128
    mod = _layer(e4b, E, H, I, seed=9)
    exs = ep.PeerExchange.emulated(2, E // 2, 32, H, torch.bfloat16, torch.device("cuda"))
    stage = ep.NativeStages(ep.shard_experts(mod, 0, 2), E, H, I, True, 2)
    t0 = time.time()
    stage.experts_peer(exs[0], 32)        # rank 0's expert side; no rank ever dispatched
    torch.cuda.synchronize()
    waited = time.time() - t0
    err = ctypes.c_int(-1)
    N.check(N.lib().e4b_read_device_error(exs[0].region.data_ptr(), N.stream_handle(torch.device("cuda")),
                                          ctypes.byref(err)), "read_device_error")
    assert err.value == N.E4B_ERR_TIMEOUT, N.status_string(err.value)
    assert waited > 0.5
    x = torch.ones(4, device="cuda")
    assert float((x * 2).sum()) == 8.0    # the context is usable
