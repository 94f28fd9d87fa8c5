"""Expert parallelism: one expert layer with its experts sharded over a process group.

The reference has no distributed code (its loop is per expert,
experts4bit_qlora/_vendor/experts.py:486-513, so experts are independent).
Rank p of P owns experts ``[p*E/P, (p+1)*E/P)`` -- contiguous slices of the
packed ``[E, ...]`` stacks, absmax and LoRA factors -- and a shard of the
tokens; the router runs on each rank's own tokens. One layer:

1. ``e4b_ep_dispatch``: the shard's picks in the single-GPU layer's stable
   order (by global expert), their rows gathered, per-expert counts.
2. all-to-all of the counts (one host sync: the row splits), then of the rows.
3. ``e4b_ep_experts``: received rows regrouped by local expert, the fused
   gate_up -> SwiGLU -> down stages (with LoRA), unweighted fp16 down rows in
   the received order.
4. reverse all-to-all: the rows land in the shard's sorted order.
5. ``e4b_combine``: weighted fixed-order k-sum. Every row sees the same kernels
   as on one GPU, so the output does not depend on P.

The exchanges use ``torch.distributed`` (NCCL over NVLink on GPUs; gloo for the
CPU tests, which swap the kernel stages for the oracle through ``stages``).
"""
from __future__ import annotations

import ctypes
from dataclasses import dataclass

import torch
import torch.distributed as dist

from . import _native as N
from .ops import MoeDesc_from


@dataclass
class ExpertShard:
    """The rank's slice of an expert stack: experts ``[first, first + count)``."""
    gate_up_packed: torch.Tensor   # [El, n1*H/2] u8
    gate_up_absmax: torch.Tensor   # [El, n1*H/64] f32
    down_packed: torch.Tensor      # [El, H*I/2] u8
    down_absmax: torch.Tensor      # [El, H*I/64] f32
    first: int
    count: int
    lora: tuple | None = None      # (A_gu, B_gu, A_dn, B_dn, scaling), expert-sliced
    weight_format: int = N.FMT_NF4  # FMT_FP8_BLOCK128: *_packed = e4m3 bytes, *_absmax = fp32 tile scales


def shard_experts(mod, rank: int, world: int) -> ExpertShard:
    """Slice an ``ExpertsNbit`` / ``ExpertsLoRA`` / ``ExpertsFp8Blocks`` module's experts for ``rank``."""
    base = mod.base if hasattr(mod, "base") else mod
    E = base.num_experts
    if getattr(base, "quant_type", None) == "fp8_block128":
        if E % world:
            raise ValueError(f"{E} experts do not split evenly over {world} ranks")
        El = E // world
        lo, hi = rank * El, (rank + 1) * El
        gs, ds = base.scale_values()
        return ExpertShard(base.gate_up_proj.data[lo:hi].contiguous(), gs[lo:hi].contiguous(),
                           base.down_proj.data[lo:hi].contiguous(), ds[lo:hi].contiguous(), lo, El, None,
                           N.FMT_FP8_BLOCK128)
    if E % world:
        raise ValueError(f"{E} experts do not split evenly over {world} ranks")
    El = E // world
    lo, hi = rank * El, (rank + 1) * El
    lora = None
    if base is not mod:
        lora = (mod.gate_up_lora_A.data[lo:hi].contiguous(), mod.gate_up_lora_B.data[lo:hi].contiguous(),
                mod.down_lora_A.data[lo:hi].contiguous(), mod.down_lora_B.data[lo:hi].contiguous(), mod.scaling)
    return ExpertShard(base.gate_up_proj.data[lo:hi].contiguous(), base.gate_up_absmax[lo:hi].contiguous(),
                       base.down_proj.data[lo:hi].contiguous(), base.down_absmax[lo:hi].contiguous(), lo, El, lora)


class NativeStages:
    """The three device stages through libe4b.so (include/e4b.h, expert-parallel section)."""

    def __init__(self, shard: ExpertShard, num_experts: int, hidden: int, intermediate: int, has_gate: bool,
                 world: int):
        self.shard, self.E, self.H, self.I, self.has_gate, self.P = shard, num_experts, hidden, intermediate, \
            bool(has_gate), world

    def dispatch(self, hidden: torch.Tensor, idx: torch.Tensor):
        T, k = idx.shape
        dev = hidden.device
        R = T * k
        send = torch.empty(R, self.H, dtype=hidden.dtype, device=dev)
        counts = torch.empty(self.E, dtype=torch.int32, device=dev)
        inv = torch.empty(R, dtype=torch.int32, device=dev)
        L = N.lib()
        ws = N.workspaces.get(dev, L.e4b_ep_dispatch_workspace_bytes(T, k, self.E), "ep_dispatch")
        N.check(L.e4b_ep_dispatch(hidden.data_ptr(), N.dtype_code(hidden.dtype), idx.data_ptr(), T, k, self.E,
                                  self.H, send.data_ptr(), counts.data_ptr(), inv.data_ptr(), ws.data_ptr(),
                                  ws.numel(), N.stream_handle(dev)), "e4b_ep_dispatch")
        return send, counts, inv

    def experts(self, rows: torch.Tensor, recv_counts: torch.Tensor, events=None):
        sh = self.shard
        Rr = rows.shape[0]
        dev = rows.device
        out = torch.empty(Rr, self.H, dtype=torch.float16, device=dev)
        d = MoeDesc_from(sh.count, self.H, self.I, 1, Rr, self.has_gate, rows.dtype, torch.float32, torch.float16,
                         sh.lora, sh.weight_format)
        t = N.MoeTensors()
        t.hidden = rows.data_ptr() if Rr else None
        t.gate_up_packed, t.gate_up_absmax = sh.gate_up_packed.data_ptr(), sh.gate_up_absmax.data_ptr()
        t.down_packed, t.down_absmax = sh.down_packed.data_ptr(), sh.down_absmax.data_ptr()
        if sh.lora is not None:
            t.gate_up_lora_A, t.gate_up_lora_B, t.down_lora_A, t.down_lora_B = (m.data_ptr() for m in sh.lora[:4])
        t.out = out.data_ptr() if Rr else None
        keep = None
        if events is not None:
            keep = (ctypes.c_void_p * N.MOE_STAGE_EVENTS)(*events)
            t.stage_events = ctypes.cast(keep, ctypes.c_void_p)
        L = N.lib()
        nbytes = L.e4b_ep_experts_workspace_bytes(ctypes.byref(d), self.P)
        if nbytes == 0:
            raise ValueError("invalid expert-parallel geometry")
        ws = N.workspaces.get(dev, nbytes, "ep_experts")
        rc = recv_counts.to(torch.int32).contiguous()
        N.check(L.e4b_ep_experts(ctypes.byref(d), self.P, rc.data_ptr(), ctypes.byref(t), ws.data_ptr(), ws.numel(),
                                 N.stream_handle(dev)), "e4b_ep_experts")
        del keep
        return out

    def combine(self, rows: torch.Tensor, inv: torch.Tensor, w: torch.Tensor, T: int, k: int, out_dtype):
        out = torch.empty(T, self.H, dtype=out_dtype, device=rows.device)
        N.check(N.lib().e4b_combine(rows.data_ptr(), N.F16, inv.data_ptr(), w.data_ptr(), N.dtype_code(w.dtype), T, k,
                                    self.H, out.data_ptr(), N.dtype_code(out_dtype), N.stream_handle(rows.device)),
                "e4b_combine")
        return out


class ExpertParallelMoE:
    """One expert layer whose experts are sharded over ``group`` (default: WORLD).

    ``forward(hidden [T,H], top_k_index [T,k], top_k_weights [T,k])`` takes the
    rank's own token shard (global expert ids) and returns its ``[T,H]`` output,
    equal to the single-GPU layer on those tokens."""

    def __init__(self, shard: ExpertShard, num_experts: int, hidden: int, intermediate: int, has_gate: bool = True,
                 group=None, stages=None):
        self.group = group
        single = not (dist.is_available() and dist.is_initialized())
        self.world = 1 if single else dist.get_world_size(group)
        self.rank = 0 if single else dist.get_rank(group)
        if num_experts % self.world or shard.count != num_experts // self.world:
            raise ValueError("the shard must hold num_experts / world experts")
        if shard.first != self.rank * shard.count:
            raise ValueError("rank p must hold experts [p*E/P, (p+1)*E/P)")
        self.E, self.H, self.I = num_experts, hidden, intermediate
        self.shard = shard
        self.stages = stages or NativeStages(shard, num_experts, hidden, intermediate, has_gate, self.world)

    @classmethod
    def from_module(cls, mod, group=None, stages=None):
        single = not (dist.is_available() and dist.is_initialized())
        world = 1 if single else dist.get_world_size(group)
        rank = 0 if single else dist.get_rank(group)
        base = mod.base if hasattr(mod, "base") else mod
        return cls(shard_experts(mod, rank, world), base.num_experts, base.hidden_dim, base.intermediate_dim,
                   base.has_gate, group, stages)

    def exchange_counts(self, counts: torch.Tensor):
        """Counts all-to-all; returns (recv_counts [P, El] on the device, send splits, recv splits)."""
        recv, splits = self._exchange_counts_mb([counts])
        return recv[0], splits[0][0], splits[0][1]

    def _exchange_counts_mb(self, counts_list):
        """One all-to-all of the per-expert counts of every micro-batch and one host sync for all of
        their row splits. Returns per micro-batch recv_counts [P, El] and (send, recv) splits."""
        P, El, M = self.world, self.E // self.world, len(counts_list)
        # [P, M, El]: the block for peer q holds each micro-batch's counts of q's experts
        send = torch.stack([c.view(P, El) for c in counts_list], 1).contiguous()
        if P == 1:
            recv = send
        else:
            recv = torch.empty_like(send)
            dist.all_to_all_single(recv, send, group=self.group)
        host = torch.cat([send.view(-1), recv.view(-1)]).cpu()  # the one host sync: NCCL needs the row splits
        hs, hr = host[:P * M * El].view(P, M, El), host[P * M * El:].view(P, M, El)
        out_counts = [recv[:, m] for m in range(M)]
        splits = [(hs[:, m].sum(1).tolist(), hr[:, m].sum(1).tolist()) for m in range(M)]
        return out_counts, splits

    def forward(self, hidden: torch.Tensor, top_k_index: torch.Tensor, top_k_weights: torch.Tensor,
                out_dtype=None, micro_batches: int | None = None) -> torch.Tensor:
        """The rank's [T, H] output. With P > 1 the shard runs as micro-batches (two when it has at
        least 256 tokens): the row exchanges of one run on a communication stream while the experts
        of the other compute, and all micro-batches share one count exchange and host sync."""
        T, k = top_k_index.shape
        idx = top_k_index.contiguous().long()
        w = top_k_weights.contiguous()
        if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            w = w.float()
        hidden = hidden.contiguous()
        od = out_dtype or hidden.dtype
        M = micro_batches if micro_batches is not None else (2 if self.world > 1 and T >= 256 else 1)
        M = max(1, min(M, T)) if T > 0 else 1
        bounds = [T * m // M for m in range(M + 1)]
        parts = [self.stages.dispatch(hidden[bounds[m]:bounds[m + 1]], idx[bounds[m]:bounds[m + 1]])
                 for m in range(M)]
        recv_counts, splits = self._exchange_counts_mb([p[1] for p in parts])
        if self.world == 1:  # one rank: the exchanges are identities
            outs = [self.stages.combine(self.stages.experts(p[0], rc), p[2], w[bounds[m]:bounds[m + 1]],
                                        bounds[m + 1] - bounds[m], k, od)
                    for m, (p, rc) in enumerate(zip(parts, recv_counts))]
            return outs[0] if M == 1 else torch.cat(outs)
        cuda = hidden.is_cuda
        main = torch.cuda.current_stream(hidden.device) if cuda else None
        comm = self._comm_stream(hidden.device) if cuda else None

        def on_comm(fn, *wait):
            if not cuda:
                return fn(), None
            for ev in wait:
                comm.wait_event(ev)
            with torch.cuda.stream(comm):
                r = fn()
            done = torch.cuda.Event()
            done.record(comm)
            return r, done

        def event_main():
            if not cuda:
                return None
            ev = torch.cuda.Event()
            ev.record(main)
            return ev

        ready = event_main()
        rows, rows_done = [], []
        for m, (send, _, _) in enumerate(parts):  # every micro-batch's rows go out at once
            ss, rs = splits[m]
            buf = torch.empty(sum(rs), self.H, dtype=send.dtype, device=send.device)
            _, ev = on_comm(lambda buf=buf, send=send, ss=ss, rs=rs: dist.all_to_all_single(
                buf, send, rs, ss, group=self.group), *([ready] if ready is not None else []))
            if cuda:
                send.record_stream(comm)
                buf.record_stream(comm)
            rows.append(buf)
            rows_done.append(ev)
        rets, rets_done = [], []
        for m in range(M):
            if cuda:
                main.wait_event(rows_done[m])
            back = self.stages.experts(rows[m], recv_counts[m])
            ss, rs = splits[m]
            n = bounds[m + 1] - bounds[m]
            ret = torch.empty(n * k, self.H, dtype=back.dtype, device=back.device)
            computed = event_main()
            _, ev = on_comm(lambda ret=ret, back=back, ss=ss, rs=rs: dist.all_to_all_single(
                ret, back, ss, rs, group=self.group), *([computed] if computed is not None else []))
            if cuda:
                back.record_stream(comm)
                ret.record_stream(comm)
            rets.append(ret)
            rets_done.append(ev)
        outs = []
        for m in range(M):
            if cuda:
                main.wait_event(rets_done[m])
            outs.append(self.stages.combine(rets[m], parts[m][2], w[bounds[m]:bounds[m + 1]],
                                            bounds[m + 1] - bounds[m], k, od))
        return outs[0] if M == 1 else torch.cat(outs)

    def _comm_stream(self, device):
        st = getattr(self, "_comm", None)
        if st is None or st.device != device:
            st = torch.cuda.Stream(device=device)
            self._comm = st
        return st

    __call__ = forward
