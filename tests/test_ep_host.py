"""Expert-parallel host logic on CPU: world_size-2 gloo ranks run
``ExpertParallelMoE`` (splits, count exchange, row all-to-alls, return order)
with its three device stages swapped for oracle restatements of the C-ABI
contract (include/e4b.h, expert-parallel section). The GPU kernels behind the
same contract are checked in test_gpu_ep.py."""
from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from oracle import moe as M
from oracle.nf4 import quantize_stack


class OracleStages:
    """The stage contract restated on CPU: dispatch in the single-GPU layer's stable
    order, experts on source-major received rows (regrouped expert-major, fp16 down
    rows returned in received order), fixed-order weighted combine."""

    def __init__(self, st_local, num_experts, world):
        self.st, self.E, self.P = st_local, num_experts, world
        self.El = st_local["E"]
        H, I = st_local["H"], st_local["I"]
        n1 = 2 * I if st_local["has_gate"] else I
        self.W_gu = M.dequant_stack_f32(st_local["gate_up_packed"], st_local["gate_up_absmax"], (n1, H))
        self.W_dn = M.dequant_stack_f32(st_local["down_packed"], st_local["down_absmax"], (H, I))

    def dispatch(self, hidden, idx):
        order, token_rows, _, counts, _ = M.permute(idx, self.E)
        inv = torch.empty_like(order)
        inv[order] = torch.arange(order.numel())
        return hidden[token_rows], counts.to(torch.int32), inv.to(torch.int32)

    def experts(self, rows, recv_counts):
        P, El = recv_counts.shape
        out = torch.empty(rows.shape[0], rows.shape[1], dtype=torch.float16)
        start = 0
        blocks = {}
        for p in range(P):
            for e in range(El):
                c = int(recv_counts[p, e])
                blocks[(p, e)] = (start, c)
                start += c
        assert start == rows.shape[0]
        x = rows.float()
        for e in range(El):  # expert-major, source-major within the expert
            idx = torch.cat([torch.arange(s, s + c) for p in range(P) for (s, c) in [blocks[(p, e)]]])
            if not idx.numel():
                continue
            h = M._epilogue(x[idx] @ self.W_gu[e].t(), self.st["has_gate"])
            out[idx] = (h @ self.W_dn[e].t()).to(torch.float16)
        return out

    def combine(self, rows, inv, w, T, k, out_dtype):
        buf = rows.float()[inv.long()].view(T, k, rows.shape[1]) * w.float().view(T, k, 1)
        return buf.sum(1).to(out_dtype)


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _case(E=8, H=128, I=64, k=2, T=24, seed=0):
    g = torch.Generator().manual_seed(seed)
    gate_up = (torch.randn(E, 2 * I, H, generator=g) * 0.1).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g) * 0.1).to(torch.bfloat16)
    gp, ga = quantize_stack(gate_up)
    dp, da = quantize_stack(down)
    st = {"gate_up_packed": gp, "gate_up_absmax": ga, "down_packed": dp, "down_absmax": da, "E": E, "H": H,
          "I": I, "has_gate": True}
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g)
    w, idx = M.route_on_host(logits, k, M.SOFTMAX_THEN_TOPK, False)
    return st, x, idx, w


def _worker(rank, world, port, shard_sizes, skew, q, micro_batches=None):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        import importlib
        ep = importlib.import_module("experts4bit-qlora_b200.ep")
        st, x, idx, w = _case()
        if skew:  # every pick on the last rank's experts: other ranks receive nothing
            idx = torch.stack([torch.full((x.shape[0],), 7), torch.full((x.shape[0],), 6)], 1)
        E = st["E"]
        El = E // world
        lo, hi = rank * El, (rank + 1) * El
        st_local = dict(st, E=El, gate_up_packed=st["gate_up_packed"][lo:hi], gate_up_absmax=st["gate_up_absmax"][lo:hi],
                        down_packed=st["down_packed"][lo:hi], down_absmax=st["down_absmax"][lo:hi])
        shard = ep.ExpertShard(st_local["gate_up_packed"], st_local["gate_up_absmax"], st_local["down_packed"],
                               st_local["down_absmax"], lo, El)
        layer = ep.ExpertParallelMoE(shard, E, st["H"], st["I"], True, stages=OracleStages(st_local, E, world))
        t0 = sum(shard_sizes[:rank])
        t1 = t0 + shard_sizes[rank]
        out = layer(x[t0:t1], idx[t0:t1], w[t0:t1], micro_batches=micro_batches)
        ref = M.fp32_oracle(st, x[t0:t1], idx[t0:t1], w[t0:t1])
        if t1 > t0:
            mx, mean = M.rel_errors(out.float(), ref)
        else:
            mx = mean = 0.0
        q.put((rank, tuple(out.shape), mx, mean))
    finally:
        dist.destroy_process_group()


def _run(shard_sizes, skew=False, micro_batches=None):
    world = len(shard_sizes)
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, shard_sizes, skew, q, micro_batches))
             for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=180)
    assert all(p.exitcode == 0 for p in procs), [p.exitcode for p in procs]
    res = sorted(q.get(timeout=5) for _ in range(world))
    return res


@pytest.mark.parametrize("shard_sizes", [(12, 12), (5, 19), (0, 24)], ids=["even", "ragged", "empty_rank"])
def test_ep_world2_matches_oracle(shard_sizes):
    for rank, shape, mx, mean in _run(shard_sizes):
        assert shape == (shard_sizes[rank], 128)
        assert mx <= 1e-2 and mean <= 2e-3, (rank, mx, mean)


def test_ep_world2_all_picks_on_one_rank():
    for rank, shape, mx, mean in _run((12, 12), skew=True):
        assert mx <= 1e-2 and mean <= 2e-3, (rank, mx, mean)


def test_ep_world2_micro_batches():
    """Three micro-batches per shard (one count exchange, per-micro-batch row exchanges)."""
    for rank, shape, mx, mean in _run((9, 15), micro_batches=3):
        assert shape == ((9, 15)[rank], 128)
        assert mx <= 1e-2 and mean <= 2e-3, (rank, mx, mean)


def test_ep_world4_ragged_with_an_empty_rank():
    """Four ranks (two experts each), shards of 0, 3, 14 and 7 tokens."""
    for rank, shape, mx, mean in _run((0, 3, 14, 7)):
        assert shape == ((0, 3, 14, 7)[rank], 128)
        assert mx <= 1e-2 and mean <= 2e-3, (rank, mx, mean)
