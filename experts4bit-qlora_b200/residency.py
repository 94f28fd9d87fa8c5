"""Expert residency: a resident sub-stack of hot experts on the GPU, the rest read from
pinned host memory on demand.

Drop-in for ``experts4bit_qlora.engines.hot_residency`` (``enable_hot_residency``,
``disable_hot_residency``, ``target_modules``, ``dispatched_modules``,
``hot_residency_available``; hot_residency.py:39-104, :222-300, :440-560) and
``experts4bit_qlora.engines.pipelined`` (``enable_pipelined_residency``,
``disable_pipelined_residency``, ``pipelined_available``; pipelined.py:117-150,
:155-540, :579-800).

Layout, per patched module:

* a pinned host arena ``[E, row_bytes]``: every expert's row-block of four segments
  (gate_up packed | gate_up absmax | down packed | down absmax, 16-byte aligned);
* four device stacks ``[n_hot + slots, segment]``, the layout ``e4b_moe_forward``
  reads: rows ``[0, n_hot)`` hold the hot experts for good, the rest are slots;
* an address table ``src[e]`` (the expert's arena row, a host address the GPU reads
  through unified addressing) and ``resident_row[e]`` (its hot row, or -1).

Decode (one token): ``e4b_gather_expert_rows`` fills slot ``j`` with the expert of
pick ``j`` unless that expert is hot (read in place) or the slot already holds it,
and writes the stack row of every pick; the fused layer then runs over the stacks
with those rows as its top-k ids. Nothing reaches the host, so the step is
capturable in a CUDA graph. Prefill (several tokens, hot residency only): the
routed cold experts are gathered into consecutive slots and an ``expert_map``
(``e4b_moe_desc.routed_experts``) sends every routed id to its stack row; the
number of routed cold experts is read on the host, as the reference's loop does.

The arithmetic is the fused layer's on the same NF4 bytes, so results equal
``enable_fast`` on the full stack (bit for bit where both take the same kernel).
"""
from __future__ import annotations

import ctypes
import warnings
from typing import Optional, Sequence

import torch

from . import _native as N
from . import ops

_SEGMENTS = ("gate_up_proj", "gate_up_absmax", "down_proj", "down_absmax")


def _align16(n: int) -> int:
    return (n + 15) // 16 * 16


def hot_residency_available() -> bool:
    return N.available() and torch.cuda.is_available()


def pipelined_available() -> bool:
    return N.available() and torch.cuda.is_available()


def wrapped_bases(model) -> set:
    """ids of every ``ExpertsNbit`` that is an ``ExpertsLoRA.base``."""
    from .lora import ExpertsLoRA
    return {id(m.base) for m in model.modules() if isinstance(m, ExpertsLoRA)}


def target_modules(model) -> list:
    """Every ``ExpertsNbit`` under ``model`` (wrapped bases included), in module order: the list
    ``hot_sets[i]`` is aligned with (hot_residency.py:343-383)."""
    from .experts import ExpertsNbit
    return [m for m in model.modules() if isinstance(m, ExpertsNbit)]


def dispatched_modules(model) -> list:
    """The modules actually called, aligned with :func:`target_modules`: the ``ExpertsLoRA``
    wrapper where one exists, else the bare module (hook these to observe routing)."""
    from .lora import ExpertsLoRA
    wrappers = {id(m.base): m for m in model.modules() if isinstance(m, ExpertsLoRA)}
    return [wrappers.get(id(m), m) for m in target_modules(model)]


def _eligible(mod) -> Optional[str]:
    if getattr(mod, "_e4b_mxfp4_arena", False):
        return "MXFP4 storage (the residency stacks hold NF4 row-blocks)"
    if getattr(mod, "bits", None) != 4 or getattr(mod, "quant_type", None) != "nf4":
        return "storage is not nf4-4bit"
    if getattr(mod, "blocksize", None) != 64:
        return f"blocksize {getattr(mod, 'blocksize', None)} != 64"
    n1, k1 = mod._gate_up_shape
    n2, k2 = mod._down_shape
    if k1 % 64 or k2 % 64:
        return "K not divisible by 64"
    if hasattr(mod, "_apply_gate") or getattr(mod, "act_fn", None) is not torch.nn.functional.silu:
        return "custom activation (the resident stacks run the fused SwiGLU / SiLU layer)"
    if not mod.gate_up_proj.is_cuda and not torch.cuda.is_available():
        return "no CUDA device"
    return None


class _Residency:
    """Per-module state: the pinned arena, the device stacks and the two id tables."""

    def __init__(self, mod, hot_ids, device, k_slots: int):
        if k_slots < 1:
            raise ValueError(f"k_slots must be >= 1, got {k_slots}")
        E = mod.num_experts
        hot = torch.as_tensor(hot_ids, dtype=torch.long).reshape(-1).unique()
        if hot.numel() and (int(hot.min()) < 0 or int(hot.max()) >= E):
            raise ValueError(f"hot ids must lie in [0, {E}); got range [{int(hot.min())}, {int(hot.max())}]")
        self.mod, self.device, self.k = mod, torch.device(device), int(k_slots)
        self.E, self.hot_ids, self.n_hot = E, hot, int(hot.numel())
        n1, H = mod._gate_up_shape
        n2, I = mod._down_shape
        self.H, self.I, self.has_gate = H, I, mod.has_gate
        self.seg_elems = [n1 * H // 2, n1 * H // 64, n2 * I // 2, n2 * I // 64]
        self.seg_dtypes = [torch.uint8, torch.float32, torch.uint8, torch.float32]
        self.seg_bytes = [n * (1 if d == torch.uint8 else 4) for n, d in zip(self.seg_elems, self.seg_dtypes)]
        if any(b % 16 for b in self.seg_bytes):
            raise ValueError("expert segments must be multiples of 16 bytes (hidden and intermediate % 256)")
        off = [0]
        for b in self.seg_bytes[:-1]:
            off.append(_align16(off[-1] + b))
        self.seg_off = off
        self.row_bytes = _align16(off[-1] + self.seg_bytes[-1])
        # pinned arena: every expert's row-block, filled from the module's current weights
        arena = torch.empty(E, self.row_bytes, dtype=torch.uint8).pin_memory()
        for name, o, b in zip(_SEGMENTS, off, self.seg_bytes):
            src = getattr(mod, name).detach().reshape(E, -1)
            arena[:, o:o + b].copy_(src.view(torch.uint8).reshape(E, b).cpu())
        self.arena = arena
        dev = self.device
        self.src_table = (torch.arange(E, dtype=torch.int64) * self.row_bytes + arena.data_ptr()).to(dev)
        rr = torch.full((E,), -1, dtype=torch.int32)
        rr[hot] = torch.arange(self.n_hot, dtype=torch.int32)
        self.resident_row = rr.to(dev)
        self.local = torch.empty(self.k, dtype=torch.int64, device=dev)
        self.ws = torch.zeros(4096, dtype=torch.uint8, device=dev)  # the gather's error word
        self._alloc(self.k)

    def _alloc(self, slots: int) -> None:
        """Device stacks with room for ``slots`` slots after the hot rows (hot rows re-filled)."""
        dev, rows = self.device, self.n_hot + slots
        self.slots = slots
        self.stacks = [torch.empty(rows, n, dtype=d, device=dev) for n, d in zip(self.seg_elems, self.seg_dtypes)]
        if self.n_hot:
            hi = self.hot_ids.to(dev)
            for st, name in zip(self.stacks, _SEGMENTS):
                st[:self.n_hot].copy_(getattr(self.mod, name).detach().reshape(self.E, -1).to(dev).index_select(0, hi))
        self.have = torch.full((slots,), -1, dtype=torch.int64, device=dev)
        self._seg_off = (ctypes.c_uint64 * 4)(*self.seg_off)
        self._seg_bytes = (ctypes.c_uint64 * 4)(*self.seg_bytes)
        self._seg_dst = (ctypes.c_void_p * 4)(*[s.data_ptr() for s in self.stacks])

    def _gather(self, ids: torch.Tensor, n: int, have, local) -> None:
        N.check(N.lib().e4b_gather_expert_rows(
            self.src_table.data_ptr(), self.E, ids.data_ptr(), None if have is None else have.data_ptr(), n,
            self.resident_row.data_ptr(), self.n_hot, local.data_ptr(), ctypes.cast(self._seg_off, ctypes.c_void_p),
            ctypes.cast(self._seg_bytes, ctypes.c_void_p), ctypes.cast(self._seg_dst, ctypes.c_void_p), self.ws.data_ptr(), self.ws.numel(), N.stream_handle(self.device)),
            "e4b_gather_expert_rows")

    def will_serve_decode(self, mod, hidden, idx) -> bool:
        cd = mod.compute_dtype if mod.compute_dtype is not None else hidden.dtype
        return (hidden.dim() == 2 and hidden.shape[0] == 1 and idx.shape[-1] == self.k and hidden.is_cuda
                and cd in (torch.bfloat16, torch.float16) and not _grad_needed(mod, hidden))

    def _layer(self, x, idx, w, out_dtype, E_local, expert_map=None):
        s = self.stacks
        return ops.moe_forward(x, idx, w, s[0], s[1], s[2], s[3], E_local, self.I, has_gate=self.has_gate,
                               out_dtype=out_dtype, expert_map=expert_map)

    def forward_decode(self, hidden, top_k_index, top_k_weights):
        """One token: slot gather (no host sync), then the fused layer over the stacks."""
        mod = self.mod
        cd = mod.compute_dtype if mod.compute_dtype is not None else hidden.dtype
        x = hidden.to(device=self.device, dtype=cd)
        k = top_k_index.shape[-1]
        if k != self.k:  # another top-k than the slots were laid out for
            self.k = k
            self.local = torch.empty(k, dtype=torch.int64, device=self.device)
        if self.slots != self.k:  # a prefill grew the slots, or k changed: the decode layout again
            self._alloc(self.k)
        ids = top_k_index.reshape(-1).to(device=self.device, dtype=torch.int64).contiguous()
        self._gather(ids, self.k, self.have, self.local)
        out = self._layer(x, self.local.view(1, self.k), top_k_weights.to(self.device), hidden.dtype,
                          self.n_hot + self.k)
        return out.to(hidden.device)

    def forward_prefill(self, hidden, top_k_index, top_k_weights):
        """Several tokens: the routed cold experts into consecutive slots, an expert map, one layer."""
        mod = self.mod
        cd = mod.compute_dtype if mod.compute_dtype is not None else hidden.dtype
        dev = self.device
        x = hidden.to(device=dev, dtype=cd)
        idx = top_k_index.to(device=dev, dtype=torch.int64).contiguous()
        routed = torch.unique(idx)
        cold = routed[self.resident_row[routed] < 0].contiguous()
        nc = int(cold.numel())  # host read of the routed cold count, as the reference's loop
        if nc > self.slots:
            self._alloc(nc)
        emap = self.resident_row.clone()
        if nc:
            local = torch.empty(nc, dtype=torch.int64, device=dev)
            self._gather(cold, nc, None, local)
            emap[cold] = local.to(torch.int32)
        self.have.fill_(-1)  # the slots no longer hold the decode picks
        return self._layer(x, idx, top_k_weights.to(dev), hidden.dtype, self.n_hot + self.slots,
                           expert_map=emap).to(hidden.device)


def _grad_needed(mod, hidden) -> bool:
    return torch.is_grad_enabled() and (hidden.requires_grad or any(p.requires_grad for p in mod.parameters()))


def _stock_forwards():
    from .experts import Experts4bit, ExpertsNbit
    return {ExpertsNbit.forward, Experts4bit.forward}


def enable_hot_residency(model, hot_sets: Sequence, device: str = "cuda", verbose: bool = False) -> int:
    """Partition every eligible ``ExpertsNbit`` under ``model`` into a resident hot sub-stack and
    the pinned host rest, in module order (hot_residency.py:440-560). ``hot_sets`` carries exactly
    one entry per :func:`target_modules` module (skipped modules consume theirs). ``ExpertsLoRA``
    bases, ``[fast]``-patched, pipelined or custom-forward modules are skipped. Any token count is
    served; grad-enabled forwards run the saved reference forward."""
    if not hot_residency_available():
        raise RuntimeError("hot residency runs on libe4b.so and a CUDA device")
    mods = target_modules(model) if hasattr(model, "modules") else [model]
    wrapped = wrapped_bases(model) if hasattr(model, "modules") else set()
    if len(hot_sets) != len(mods):
        raise ValueError(f"hot_sets has {len(hot_sets)} entries but the model has {len(mods)} ExpertsNbit "
                         "modules: exactly one entry per MoE layer in module order is required")
    stock = _stock_forwards()
    patched = 0
    for i, mod in enumerate(mods):
        why = None
        if id(mod) in wrapped:
            why = "ExpertsLoRA base (use enable_pipelined_residency, which the wrapper reaches)"
        elif type(mod).forward not in stock and not hasattr(mod, "_e4b_hot_ref"):
            why = "custom forward"
        elif any(hasattr(mod, a) for a in ("_e4b_fast_ref", "_e4b_pipe_ref")):
            why = "another engine is enabled; disable it first"
        else:
            why = _eligible(mod)
        if why is not None:
            if verbose:
                print(f"[hot_residency] skip {type(mod).__name__}: {why}")
            continue
        state = _Residency(mod, hot_sets[i], device, k_slots=8)  # re-laid out for the first decode's k
        mod._hot_residency = state  # rebuilt on every enable: never a stale partition
        if hasattr(mod, "_e4b_hot_ref"):
            patched += 1
            continue
        mod._e4b_hot_ref = mod.forward

        def _fwd(hidden, top_k_index, top_k_weights, _m=mod):
            st = _m._hot_residency
            cd = _m.compute_dtype if _m.compute_dtype is not None else hidden.dtype
            if _grad_needed(_m, hidden) or cd not in (torch.bfloat16, torch.float16) or hidden.shape[0] == 0:
                return _m._e4b_hot_ref(hidden, top_k_index, top_k_weights)
            if hidden.shape[0] == 1:
                return st.forward_decode(hidden, top_k_index, top_k_weights)
            return st.forward_prefill(hidden, top_k_index, top_k_weights)

        mod.forward = _fwd
        patched += 1
    return patched


def disable_hot_residency(model) -> int:
    """Undo :func:`enable_hot_residency`; returns the number of modules restored."""
    restored = 0
    for mod in (model.modules() if hasattr(model, "modules") else [model]):
        if hasattr(mod, "_e4b_hot_ref"):
            mod.forward = mod._e4b_hot_ref
            del mod._e4b_hot_ref
            if hasattr(mod, "_hot_residency"):
                del mod._hot_residency
            restored += 1
    return restored


def enable_pipelined_residency(model, hot_sets: Sequence, device: str = "cuda", k_slots: int | None = None,
                               verbose: bool = False) -> int:
    """The decode engine (pipelined.py:579-760): resident hot rows read in place, every other
    routed expert gathered into its pick's slot by one launch, then the fused layer over the
    stacks; no host sync, capturable. ``k_slots`` is the routed top-k (required). A 0-length hot
    set is pure streaming, all experts fully resident. ``ExpertsLoRA``-wrapped bases are patched
    too (the wrapper hands a zero adapter's forward to its base). Prefill (T > 1), grad-enabled
    forwards, another top-k and non-16-bit compute run the saved reference forward."""
    if k_slots is None:
        raise ValueError("k_slots (the model's routed top-k) is required")
    if not pipelined_available():
        raise RuntimeError("pipelined residency runs on libe4b.so and a CUDA device")
    mods = target_modules(model) if hasattr(model, "modules") else [model]
    if len(hot_sets) != len(mods):
        raise ValueError(f"hot_sets has {len(hot_sets)} entries but the model has {len(mods)} ExpertsNbit "
                         "modules: exactly one entry per MoE layer in module order")
    from .lora import ExpertsLoRA
    parents = {id(m.base): m for m in model.modules() if isinstance(m, ExpertsLoRA)} if hasattr(
        model, "modules") else {}
    stock = _stock_forwards()
    patched, unreachable, wrapped_patched = 0, [], 0
    for i, mod in enumerate(mods):
        why = None
        if any(hasattr(mod, a) for a in ("_e4b_fast_ref", "_e4b_hot_ref")):
            why = "another forward patch is active"
        elif type(mod).forward not in stock and not hasattr(mod, "_e4b_pipe_ref"):
            why = "custom forward"
        else:
            why = _eligible(mod)
        if why is not None:
            if verbose:
                print(f"[pipelined] skip {type(mod).__name__}: {why}")
            continue
        parent = parents.get(id(mod))
        if parent is not None:
            wrapped_patched += 1
            if not parent._adapter_is_zero():
                unreachable.append(type(mod).__name__)
        state = _Residency(mod, hot_sets[i], device, k_slots=int(k_slots))
        mod._pipelined = state
        if hasattr(mod, "_e4b_pipe_ref"):
            patched += 1
            continue
        mod._e4b_pipe_ref = mod.forward

        def _fwd(hidden, idx, wts, _m=mod):
            st = _m._pipelined
            if not st.will_serve_decode(_m, hidden, idx):
                return _m._e4b_pipe_ref(hidden, idx, wts)
            return st.forward_decode(hidden, idx, wts)

        mod.forward = _fwd
        patched += 1
    if wrapped_patched and getattr(model, "training", False):
        warnings.warn(f"[pipelined] model is in TRAINING mode: ExpertsLoRA only hands off to the patched base "
                      f"under eval + no_grad, so {wrapped_patched} patch(es) on wrapped bases will be bypassed. "
                      "Call model.eval() before inference.", RuntimeWarning, stacklevel=2)
    if unreachable:
        warnings.warn(f"[pipelined] {len(unreachable)} of {patched} patched module(s) are ExpertsLoRA bases with a "
                      "non-zero adapter: the wrapper injects its delta before the activation and never calls the "
                      "base, so these patches will not run.", RuntimeWarning, stacklevel=2)
    return patched


def disable_pipelined_residency(model) -> int:
    """Undo :func:`enable_pipelined_residency`; returns the number of modules restored."""
    restored = 0
    for mod in (model.modules() if hasattr(model, "modules") else [model]):
        if hasattr(mod, "_e4b_pipe_ref"):
            mod.forward = mod._e4b_pipe_ref
            del mod._e4b_pipe_ref
            if hasattr(mod, "_pipelined"):
                del mod._pipelined
            restored += 1
    return restored
