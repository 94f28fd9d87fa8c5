"""Kernel-level compatibility export: ``nf4_grouped.gemm_4bit_grouped``.

The reference's fused driver (experts4bit_qlora/engines/fast.py:115-156) calls
grouped-nf4-gemm as ``gemm_4bit_grouped(a, packed.view(E,N,K/2),
absmax.view(E,N,K/64), sizes, expert_ids)``. Putting this directory on
``sys.path`` lets that unmodified driver run on this library's grouped GEMM
(``e4b_grouped_nf4_gemm``). Rows of ``a`` are grouped contiguously in the order
of ``expert_ids``, which must be ascending (as ``fast.py`` produces them).
"""
from __future__ import annotations

import importlib

import torch

_ops = importlib.import_module("experts4bit-qlora_b200.ops")


def gemm_4bit_grouped(a, packed, absmax, sizes, expert_ids):
    E = packed.shape[0]
    sizes = [int(s) for s in sizes]
    expert_ids = [int(e) for e in expert_ids]
    if any(s <= 0 for s in sizes):
        raise ValueError("sizes must all be > 0")
    if any(b <= a_ for a_, b in zip(expert_ids, expert_ids[1:])):
        raise ValueError("expert_ids must be strictly ascending")
    counts = [0] * E
    for e, s in zip(expert_ids, sizes):
        counts[e] = s
    offsets = [0]
    for c in counts:
        offsets.append(offsets[-1] + c)
    offs = torch.tensor(offsets, dtype=torch.int32, device=a.device)
    return _ops.grouped_nf4_gemm(a, packed, absmax.float(), offs)
