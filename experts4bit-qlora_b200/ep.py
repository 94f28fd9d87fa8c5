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

On GPUs of one node the exchanges are the library's own peer-memory stores
(``exchange="peer"``, the default there): every rank maps every other rank's
exchange region (``PeerExchange``, CUDA IPC) once, dispatch stores rows and
counts straight into the owners' regions, the expert side stores its down rows
straight into the sources' regions, and flags order the steps -- no host sync,
no all-to-all. Otherwise (``exchange="nccl"``, or gloo for the CPU tests, which
swap the kernel stages for the oracle through ``stages``) the exchanges are
``torch.distributed`` all-to-alls.
"""
from __future__ import annotations

import ctypes
import socket
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

    def experts_peer(self, ex: "PeerExchange", expected_rows: int, events=None):
        """The expert side over peer memory: waits for every source, runs the stages, returns the
        down rows into the sources' regions (``e4b_ep_experts_peer``)."""
        sh = self.shard
        dev = ex.region.device
        d = MoeDesc_from(sh.count, self.H, self.I, 1, expected_rows, self.has_gate, ex.act_dtype, torch.float32,
                         torch.float16, sh.lora, sh.weight_format)
        t = N.MoeTensors()
        t.gate_up_packed, t.gate_up_absmax = sh.gate_up_packed.data_ptr(), sh.gate_up_absmax.data_ptr()
        t.down_packed, t.down_absmax = sh.down_packed.data_ptr(), sh.down_absmax.data_ptr()
        if sh.lora is not None:
            t.gate_up_lora_A, t.gate_up_lora_B, t.down_lora_A, t.down_lora_B = (m.data_ptr() for m in sh.lora[:4])
        keep = None
        if events is not None:
            keep = (ctypes.c_void_p * N.MOE_STAGE_EVENTS)(*events)
            t.stage_events = ctypes.cast(keep, ctypes.c_void_p)
        L = N.lib()
        nbytes = L.e4b_ep_experts_peer_workspace_bytes(ctypes.byref(ex.desc), ctypes.byref(d))
        if nbytes == 0:
            raise ValueError("invalid expert-parallel geometry")
        ws = N.workspaces.get(dev, nbytes, "ep_experts_peer")
        N.check(L.e4b_ep_experts_peer(ctypes.byref(ex.desc), ctypes.byref(d), ctypes.byref(t), ws.data_ptr(),
                                      ws.numel(), N.stream_handle(dev)), "e4b_ep_experts_peer")
        del keep

    def combine(self, rows: torch.Tensor, inv: torch.Tensor, w: torch.Tensor, T: int, k: int, out_dtype):
        out = torch.empty(T, self.H, dtype=out_dtype, device=rows.device)
        N.check(N.lib().e4b_combine(rows.data_ptr(), N.F16, inv.data_ptr(), w.data_ptr(), N.dtype_code(w.dtype), T, k,
                                    self.H, out.data_ptr(), N.dtype_code(out_dtype), N.stream_handle(rows.device)),
                "e4b_combine")
        return out


class PeerExchange:
    """This rank's exchange region and every peer's, mapped here (include/e4b.h, peer section).

    Built collectively once per (group, geometry): each rank allocates its region (zeroed),
    exports a CUDA IPC handle, gathers everyone's, and opens the others. One exchange serves
    every layer that all ranks call in the same order; the region counts the calls on the
    device, so a layer call can be captured in a CUDA graph and replayed."""

    def __init__(self, world: int, rank: int, local_experts: int, rows_per_rank: int, hidden: int,
                 act_dtype: torch.dtype, device: torch.device, group=None, _regions=None):
        L = N.lib()
        nbytes = L.e4b_ep_comm_bytes(world, local_experts, rows_per_rank, hidden)
        if nbytes == 0:
            raise ValueError("invalid peer-exchange geometry (world <= %d, E <= 1024)" % N.EP_MAX_PEERS)
        self.world, self.rank, self.act_dtype = world, rank, act_dtype
        self.rows_per_rank = rows_per_rank
        self._opened = []
        if _regions is not None:  # one process holding every rank's region (single-GPU emulation)
            self.region = _regions[rank]
            ptrs = [r.data_ptr() for r in _regions]
        else:
            self.region = torch.zeros(nbytes, dtype=torch.uint8, device=device)
            torch.cuda.synchronize(device)
            handle = (ctypes.c_char * N.IPC_HANDLE_BYTES)()
            off = ctypes.c_size_t()
            N.check(L.e4b_ipc_export(self.region.data_ptr(), handle, ctypes.byref(off)), "e4b_ipc_export")
            info = [None] * world
            dist.all_gather_object(info, (handle.raw, off.value), group=group)
            ptrs = []
            for q, (h, o) in enumerate(info):
                if q == rank:
                    ptrs.append(self.region.data_ptr())
                    continue
                p = ctypes.c_void_p()
                N.check(L.e4b_ipc_open(h, o, ctypes.byref(p)), "e4b_ipc_open")
                self._opened.append((p.value, o))
                ptrs.append(p.value)
            dist.barrier(group=group)  # every region mapped everywhere before the first store
        self._ptrs = (ctypes.c_void_p * world)(*ptrs)
        self.desc = N.EpPeerDesc(world, rank, local_experts, rows_per_rank, hidden, N.dtype_code(act_dtype),
                                 ctypes.cast(self._ptrs, ctypes.c_void_p))

    @classmethod
    def emulated(cls, world, local_experts, rows_per_rank, hidden, act_dtype, device):
        """``world`` exchanges whose regions all live on one device (tests; launches in rank order)."""
        nbytes = N.lib().e4b_ep_comm_bytes(world, local_experts, rows_per_rank, hidden)
        regions = [torch.zeros(nbytes, dtype=torch.uint8, device=device) for _ in range(world)]
        return [cls(world, r, local_experts, rows_per_rank, hidden, act_dtype, device, _regions=regions)
                for r in range(world)]

    def close(self):
        L = N.lib()
        for p, o in self._opened:
            L.e4b_ipc_close(p, o)
        self._opened = []


_exchanges = {}
_one_host = {}


def _peer_exchange(group, world, rank, El, cap, H, dtype, device):
    key = (id(group), world, rank, El, cap, H, dtype, device.index)
    ex = _exchanges.get(key)
    if ex is None:
        ex = _exchanges[key] = PeerExchange(world, rank, El, cap, H, dtype, device, group)
    return ex


class ExpertParallelMoE:
    """One expert layer whose experts are sharded over ``group`` (default: WORLD).

    ``forward(hidden [T,H], top_k_index [T,k], top_k_weights [T,k])`` takes the
    rank's own token shard (global expert ids) and returns its ``[T,H]`` output,
    equal to the single-GPU layer on those tokens.

    ``exchange``: "peer" (library stores into the other ranks' memory; GPUs of one node),
    "nccl" (torch.distributed all-to-alls), or "auto" (peer when every rank is a GPU process on
    this host, else nccl). ``max_tokens``: the most tokens any rank passes in one call, which
    sizes the peer regions; by default the largest shard of the first call (a collective)."""

    def __init__(self, shard: ExpertShard, num_experts: int, hidden: int, intermediate: int, has_gate: bool = True,
                 group=None, stages=None, exchange: str = "auto", max_tokens: int | None = None):
        if exchange not in ("auto", "peer", "nccl"):
            raise ValueError("exchange must be 'auto', 'peer' or 'nccl'")
        self.exchange = exchange
        self.max_tokens = max_tokens
        self._peer_ok = None
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
    def from_module(cls, mod, group=None, stages=None, **kw):
        single = not (dist.is_available() and dist.is_initialized())
        world = 1 if single else dist.get_world_size(group)
        rank = 0 if single else dist.get_rank(group)
        base = mod.base if hasattr(mod, "base") else mod
        return cls(shard_experts(mod, rank, world), base.num_experts, base.hidden_dim, base.intermediate_dim,
                   base.has_gate, group, stages, **kw)

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
        """The rank's [T, H] output. Over NCCL, ``micro_batches`` > 1 splits the shard: the row
        exchanges of one micro-batch run on a communication stream while the experts of the other
        compute, and all share one count exchange and host sync (default 1: on B200 the NCCL kernels
        beside the persistent GEMM cost more than the overlap gains)."""
        T, k = top_k_index.shape
        idx = top_k_index.contiguous().long()
        w = top_k_weights.contiguous()
        if w.dtype not in (torch.bfloat16, torch.float16, torch.float32):
            w = w.float()
        hidden = hidden.contiguous()
        od = out_dtype or hidden.dtype
        if self.world == 1 and hidden.is_cuda and isinstance(self.stages, NativeStages):
            # one rank holds every expert: the single-GPU fused layer (the same kernels on the
            # same rows, so the same result), with no exchange and no host sync
            sh = self.shard
            from .ops import moe_forward
            return moe_forward(hidden, idx, w, sh.gate_up_packed, sh.gate_up_absmax, sh.down_packed, sh.down_absmax,
                               self.E, self.I, self.stages.has_gate, od, sh.lora, weight_format=sh.weight_format)
        if self._use_peer(hidden):
            return self._forward_peer(hidden, idx, w, od)
        M = micro_batches if micro_batches is not None else 1
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

    def _use_peer(self, hidden):
        if self._peer_ok is None:
            ok = (self.world > 1 and hidden.is_cuda and isinstance(self.stages, NativeStages)
                  and self.exchange != "nccl")
            if ok and self.exchange == "auto":  # every rank on this host (a collective, once per group)
                key = id(self.group)
                if key not in _one_host:
                    names = [None] * self.world
                    dist.all_gather_object(names, socket.gethostname(), group=self.group)
                    _one_host[key] = len(set(names)) == 1
                ok = _one_host[key]
            if self.exchange == "peer" and not ok:
                raise ValueError("exchange='peer' needs CUDA tensors, native stages and world > 1 on one host")
            self._peer_ok = ok
        return self._peer_ok

    def _exchange_for(self, T, k, hidden):
        if self.max_tokens is None:  # the largest shard of the first call, agreed by all ranks
            t = torch.tensor([T], dtype=torch.int64, device=hidden.device)
            dist.all_reduce(t, op=dist.ReduceOp.MAX, group=self.group)
            self.max_tokens = max(1, int(t.item()))
        if T > self.max_tokens:
            raise ValueError(f"{T} tokens exceed max_tokens={self.max_tokens} of the peer exchange")
        return _peer_exchange(self.group, self.world, self.rank, self.E // self.world, self.max_tokens * k, self.H,
                              hidden.dtype, hidden.device)

    def _forward_peer(self, hidden, idx, w, od, ex=None, phase_events=None, stage_events=None):
        """Peer-memory layer. ``phase_events``: 4 CUDA events recorded before dispatch, after dispatch,
        after the expert side and after combine; ``stage_events``: passed to the expert side."""
        T, k = idx.shape
        rec = (lambda i: phase_events[i].record()) if phase_events else (lambda i: None)
        ex = ex or self._exchange_for(T, k, hidden)
        if hidden.dtype != ex.act_dtype:
            raise ValueError("the peer exchange carries %s rows" % ex.act_dtype)
        desc = ex.desc
        dev = hidden.device
        L = N.lib()
        stream = N.stream_handle(dev)
        inv = torch.empty(T * k, dtype=torch.int32, device=dev)
        ws = N.workspaces.get(dev, L.e4b_ep_dispatch_peer_workspace_bytes(T, k, self.E), "ep_dispatch")
        rec(0)
        N.check(L.e4b_ep_dispatch_peer(ctypes.byref(desc), hidden.data_ptr(), idx.data_ptr(), T, k, inv.data_ptr(),
                                       ws.data_ptr(), ws.numel(), stream), "e4b_ep_dispatch_peer")
        rec(1)
        self.stages.experts_peer(ex, T * k, events=stage_events)
        rec(2)
        out = torch.empty(T, self.H, dtype=od, device=dev)
        N.check(L.e4b_ep_combine_peer(ctypes.byref(desc), inv.data_ptr(), w.data_ptr(), N.dtype_code(w.dtype), T, k,
                                      out.data_ptr(), N.dtype_code(od), stream), "e4b_ep_combine_peer")
        rec(3)
        return out

    def _comm_stream(self, device):
        st = getattr(self, "_comm", None)
        if st is None or st.device != device:
            st = torch.cuda.Stream(device=device)
            self._comm = st
        return st

    __call__ = forward
