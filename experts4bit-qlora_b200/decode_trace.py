"""Phase timeline of the one-launch decode kernel (``nf4_decode_layer_kernel``).

The kernel carries %globaltimer stamps at its phase boundaries when compiled with
``-DE4B_TRACE`` (read back with ``e4b_decode_trace_read``). This tool builds that
instrumented variant of the library into ``<out>/libe4b.so`` (the shipped library
is untouched), runs the fused decode step (router + layer) on a random layer of the
given geometry with the L2 flushed before every call, and prints, per phase, the
median over CTAs of the stamp relative to the launch's first stamp.

    python -m experts4bit-qlora_b200.decode_trace --out build_trace   # (run from the repo root)
"""
from __future__ import annotations

import argparse
import ctypes
import glob
import importlib
import os
import statistics
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)

# stamp index -> phase boundary (decode_layer.cu, DTRACE calls)
PHASES = [(0, "start"), (14, "router logits (+ grid sync)"), (15, "logits in shared memory"), (16, "top-k"),
          (17, "permutation count"), (18, "permutation place"), (1, "permutation done"),
          (10, "first weight copies issued"), (11, "pair table built"), (12, "token rows converted"),
          (13, "block barrier"), (2, "phase A start"), (3, "gate_up done, down copies issued"),
          (4, "grid barrier 1"), (5, "h staged"), (6, "down done"), (7, "grid barrier 2"), (8, "combine"),
          (9, "error fold")]


def build_traced(out: str) -> str:
    from .build import NVCC_FLAGS, _nvcc
    os.makedirs(out, exist_ok=True)
    lib = os.path.join(out, "libe4b.so")
    srcs = sorted(glob.glob(os.path.join(HERE, "csrc", "*.cu")) + glob.glob(os.path.join(HERE, "csrc", "*.cuh")))
    if os.path.exists(lib) and os.path.getmtime(lib) >= max(os.path.getmtime(f) for f in srcs):
        return lib  # up to date
    nvcc = _nvcc()
    objs = []
    for src in [f for f in srcs if f.endswith(".cu")]:
        obj = os.path.join(out, os.path.basename(src) + ".o")
        subprocess.run([nvcc, *NVCC_FLAGS, "-DE4B_TRACE", "-I", os.path.join(ROOT, "include"), "-c", src, "-o", obj],
                       check=True)
        objs.append(obj)
    subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-shared", "-o", lib, *objs, "-lcudart"],
                   check=True)
    return lib


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default="build_trace", help="directory for the instrumented library")
    ap.add_argument("--experts", type=int, default=64)
    ap.add_argument("--hidden", type=int, default=2048)
    ap.add_argument("--intermediate", type=int, default=1024)
    ap.add_argument("--top-k", type=int, default=8)
    ap.add_argument("--tokens", type=int, default=1)
    ap.add_argument("--reps", type=int, default=12)
    args = ap.parse_args()
    lib_path = build_traced(args.out)
    import torch
    pkg = importlib.import_module(__package__)
    pkg._native.LIB_PATH = lib_path
    L = pkg._native.lib()
    L.e4b_decode_trace_read.argtypes = [ctypes.c_void_p, ctypes.c_int]
    dev = torch.device("cuda")
    E, H, I, k, T = args.experts, args.hidden, args.intermediate, args.top_k, args.tokens
    g = torch.Generator(device=dev).manual_seed(0)
    mod = pkg.Experts4bit.from_float((torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16),
                                     (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    rw = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=dev).to(torch.bfloat16)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    res = {i: [] for i, _ in PHASES}
    for rep in range(args.reps):
        flush.zero_()
        pkg.ops.moe_decode_step(x, rw, k, mod.gate_up_proj, mod.gate_up_absmax, mod.down_proj, mod.down_absmax, E,
                                I)
        torch.cuda.synchronize()
        if rep < 4:
            continue
        buf = (ctypes.c_ulonglong * (sms * 24))()
        L.e4b_decode_trace_read(ctypes.addressof(buf), sms * 24)
        t0 = min(buf[c * 24] for c in range(sms))
        for i, _ in PHASES:
            res[i].append(statistics.median(buf[c * 24 + i] - t0 for c in range(sms)) / 1e3)
    prev = 0.0
    for i, name in PHASES:
        m = statistics.median(res[i])
        print(f"{name:34s} at {m:7.2f} us  (+{m - prev:5.2f})")
        prev = m


if __name__ == "__main__":
    main()
