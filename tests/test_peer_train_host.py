"""CPU: host-side pieces of the peer-memory expert exchange and of the training path.

The peer entry points validate their descriptor before any device work, so the refusals
are checked here without a GPU; the region size follows the layout every rank shares.
The training path's padded segment batching is pure host/torch logic."""
import ctypes
import importlib

import pytest
import torch


def _desc(N, world=2, rank=0, El=4, cap=64, H=128, peers=None):
    arr = (ctypes.c_void_p * max(world, 1))(*(peers if peers is not None else [256 * (q + 1) for q in range(world)]))
    d = N.EpPeerDesc(world, rank, El, cap, H, N.BF16, ctypes.cast(arr, ctypes.c_void_p))
    return d, arr


def test_comm_bytes_layout(e4b):
    L = e4b._native.lib()
    b = L.e4b_ep_comm_bytes(2, 4, 64, 128)
    rows = 2 * 64 * 128 * 2 + 64 * 128 * 2          # received rows + returned rows
    assert rows < b < rows + 8 * 4096                # plus error word, flags, counters, counts
    assert b % 256 == 0
    assert L.e4b_ep_comm_bytes(17, 4, 64, 128) == 0  # more than E4B_EP_MAX_PEERS
    assert L.e4b_ep_comm_bytes(2, 600, 64, 128) == 0  # more than 1024 experts
    assert L.e4b_ep_comm_bytes(2, 4, 0, 128) == 0


def test_peer_entry_points_refuse_bad_descriptors(e4b):
    N = e4b._native
    L = N.lib()
    ws = ctypes.create_string_buffer(1024)
    d, keep = _desc(N, world=2, rank=2)                           # rank out of range
    assert L.e4b_ep_dispatch_peer(ctypes.byref(d), None, None, 0, 2, None, ws, 1024, None) == 1
    d, keep = _desc(N, world=2, peers=[256, 0])                    # a missing peer region
    assert L.e4b_ep_dispatch_peer(ctypes.byref(d), None, None, 0, 2, None, ws, 1024, None) == 1
    d, keep = _desc(N, world=2, peers=[256, 300])                  # a region off 256-byte alignment
    assert L.e4b_ep_combine_peer(ctypes.byref(d), None, None, 2, 0, 2, None, 0, None) == 1
    d, keep = _desc(N, world=2, H=100)                             # H not a multiple of 64
    assert L.e4b_ep_combine_peer(ctypes.byref(d), None, None, 2, 0, 2, None, 0, None) == 1
    d, keep = _desc(N, world=2, cap=64)                            # T * k above rows_per_rank
    assert L.e4b_ep_dispatch_peer(ctypes.byref(d), None, None, 40, 2, None, ws, 1024, None) == 1
    md = e4b.ops.MoeDesc_from(8, 128, 128, 1, 64, True, torch.bfloat16, torch.float32, torch.float16, None)
    d, keep = _desc(N, world=2, El=4)
    assert L.e4b_ep_experts_peer_workspace_bytes(ctypes.byref(d), ctypes.byref(md)) == 0  # 8 != E/P
    md = e4b.ops.MoeDesc_from(4, 128, 128, 1, 64, True, torch.bfloat16, torch.float32, torch.float16, None)
    assert L.e4b_ep_experts_peer_workspace_bytes(ctypes.byref(d), ctypes.byref(md)) > 0


def test_ipc_helpers_refuse_null(e4b):
    L = e4b._native.lib()
    off = ctypes.c_size_t()
    h = (ctypes.c_char * 64)()
    assert L.e4b_ipc_export(None, h, ctypes.byref(off)) == 1
    p = ctypes.c_void_p()
    assert L.e4b_ipc_open(None, 0, ctypes.byref(p)) == 1
    assert L.e4b_ipc_close(None, 0) == 1


def test_segments_pad_unpad_round_trip():
    train = importlib.import_module("experts4bit-qlora_b200.train")
    offsets = [0, 3, 3, 7, 8, 8]                     # experts 1 and 4 empty
    seg = train._Segments(offsets, 8, "cpu")
    assert seg.experts == [0, 2, 3] and seg.L == 4
    x = torch.arange(16.).view(8, 2)
    p = seg.pad(x)
    assert p.shape == (3, 4, 2)
    assert torch.equal(p[0, :3], x[0:3]) and torch.equal(p[1], x[3:7]) and torch.equal(p[2, :1], x[7:8])
    assert p[0, 3].abs().sum() == 0 and p[2, 1:].abs().sum() == 0
    assert torch.equal(seg.unpad(p), x)


def test_enable_fast_train_skips_cpu_storage(e4b, capsys):
    g = torch.Generator().manual_seed(0)
    base = e4b.Experts4bit.from_float(torch.randn(4, 256, 128, generator=g) * 0.02,
                                      torch.randn(4, 128, 128, generator=g) * 0.02)
    lm = e4b.ExpertsLoRA(base, r=4)
    assert e4b.enable_fast_train(lm, verbose=True) == 0
    assert "storage not on CUDA" in capsys.readouterr().out
    assert e4b.disable_fast_train(lm) == 0
