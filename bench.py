"""MoE-layer throughput of the fused NF4 expert path on B200.

Default workload (one GPU): OLMoE-1B-7B geometry bs=1 decode --
16 MoE layers (E=64, H=2048, I=1024, top-8 softmax router), random-init NF4
experts (N(0, 0.02) bf16 weights quantized on the device). One step = one
decode token through all 16 MoE layers (router + fused expert layer each),
with a fresh synthetic token per layer and step. ``value`` is MoE-layer
tokens/s (layers x tokens / s: the throughput of one MoE layer, the unit of the
reference's own per-layer numbers) with inputs resident in HBM, timed over
CUDA-graph replays; ``e2e`` is the same metric through the public Python API
(eager calls) with pinned-host -> device copies of every step's inputs and a
device -> host read of its outputs inside the timed region.

Usage: python bench.py [--gpus N] [--steps K] [--warmup W] [--impl reference]
       [--workload olmoe-decode|qwen3-prefill]
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

PEAKS_FALLBACK = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

WORKLOADS = {
    # name: (E, H, I, k, tokens per layer, layers, router norm)
    "olmoe-decode": dict(E=64, H=2048, I=1024, k=8, T=1, layers=16, norm=False, lora=0,
                         desc="OLMoE-1B-7B geometry (config 2): 16 MoE layers, E=64, H=2048, I=1024, top-8, bs=1 decode"),
    "qwen3-prefill": dict(E=128, H=2048, I=768, k=8, T=4096, layers=4, norm=True, lora=16,
                          desc="Qwen3-30B-A3B geometry (config 3): E=128, H=2048, I=768, top-8, T=4096, LoRA r=16"),
    "qwen3-train": dict(E=128, H=2048, I=768, k=8, T=4096, layers=1, norm=True, lora=16, train=True,
                        desc="Qwen3-30B-A3B geometry, T=4096, LoRA r=16 (fp32 adapters, bf16 compute): one "
                             "forward + backward of the fused training path (enable_fast_train)"),
    "qwen3-prefill-base": dict(E=128, H=2048, I=768, k=8, T=4096, layers=4, norm=True, lora=0,
                               desc="Qwen3-30B-A3B geometry, T=4096, frozen NF4 experts without adapters"),
    # T is the GLOBAL token count per layer, split over the ranks (strong scaling)
    "mixtral-ep": dict(E=8, H=4096, I=14336, k=2, T=8192, layers=32, norm=True, lora=0, ep=True,
                       desc="Mixtral-8x7B geometry (config 4): 32 MoE layers, E=8, H=4096, I=14336, top-2, "
                            "T=8192 tokens per layer sharded over the ranks, experts sharded over the ranks"),
    # config 5: FP8 e4m3 experts with 128x128 e8m0 scales, Zipf(1.1) expert popularity; routes are
    # sampled from that popularity (DeepSeek's sigmoid group-limited router is not this path's)
    "deepseek-fp8-decode": dict(E=256, H=7168, I=2048, k=8, T=64, layers=4, norm=True, lora=0, ep=True, fmt="fp8",
                                routing="zipf", bound="hbm",
                                desc="DeepSeek-V3 geometry (config 5): E=256, H=7168, I=2048, top-8, FP8 e4m3 "
                                     "128x128 blocks, Zipf(1.1) routing, decode bs=64 (global)"),
    "deepseek-fp8-prefill": dict(E=256, H=7168, I=2048, k=8, T=16384, layers=4, norm=True, lora=0, ep=True,
                                 fmt="fp8", routing="zipf", bound="tensor",
                                 desc="DeepSeek-V3 geometry (config 5): E=256, H=7168, I=2048, top-8, FP8 e4m3 "
                                      "128x128 blocks, Zipf(1.1) routing, prefill T=16384 (global)"),
}


# DRAM bytes (read + write) per launch of the dominant kernel, from the ncu captures summarised
# under profiles/ (same kernels and shapes); workloads without a capture report null.
MEASURED_TRAFFIC = {
    "olmoe-decode": {"bytes": 28703744 + 768, "kernel": "nf4_decode_slice_kernel",
                     "source": "profiles/nf4_decode_slice__olmoe_decode.md"},
    "qwen3-prefill-base": {"bytes": 364481536 + 40394240, "kernel": "nf4_umma_kernel<__half, 2> (gate_up)",
                           "source": "profiles/nf4_umma__qwen3_prefill.md"},
}


def load_peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        with open(p) as f:
            d = json.load(f)
        return d, "measured"
    return PEAKS_FALLBACK, "fallback"


class ClockSampler:
    """nvidia-smi clocks/throttle reasons sampled every 50 ms while running."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.gpu}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self._t = threading.Thread(target=self._read, daemon=True)
            self._t.start()
            t0 = time.time()  # the timed region starts once the sampler reports (it takes a moment to start)
            while not self.lines and time.time() - t0 < 3.0 and self.proc.poll() is None:
                time.sleep(0.01)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def mark(self):
        """Index of the next sample: summary(since=mark()) keeps only samples taken after it."""
        return len(self.lines)

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self, since=0):
        sm, smax, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for line in self.lines[since:]:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                smax = float(parts[2])
            except ValueError:
                continue
            for n, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": smax,
                "reasons": sorted(reasons), "samples": len(sm)}


def config_of(args, wl, world):
    """The line's ``config``: the workload and its geometry only, so both arms print the same dict."""
    E, H, I, k = wl["E"], wl["H"], wl["I"], wl["k"]
    per_el = 1.0 if wl.get("fmt") == "fp8" else 0.5 + 4 / 64
    c = {"workload": args.workload, "desc": wl["desc"], "tokens_per_layer": wl["T"], "layers": wl["layers"],
         "experts": E, "hidden": H, "intermediate": I, "top_k": k, "lora_rank": wl["lora"],
         "weights": "fp8 e4m3 128x128" if wl.get("fmt") == "fp8" else "nf4 blocksize 64"}
    if wl.get("ep"):
        c["tokens_per_rank"] = wl["T"] // world
        c["parallelism"] = f"ep{world}" if world > 1 else "single-gpu"
        c["l2"] = ("inputs larger than L2: each step reads a %.0f MB layer slice per rank"
                   % (E * 3 * I * H * per_el / 1e6 / world))
        c["timing"] = "CUDA events around K steps, max over ranks"
    else:
        c["parallelism"] = "replicas" if world > 1 else "single-gpu"
        c["l2"] = ("inputs larger than L2: a step streams the weights of every expert its tokens pick, "
                   "at least %.0f MB" % (wl["layers"] * min(E, k * wl["T"]) * 3 * I * H * per_el / 1e6))
        c["timing"] = "CUDA-graph replay of the step, CUDA events, median of timed K-step blocks, max over ranks"
    return c


def dist_setup(n_gpus):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", device_id=torch.device("cuda", local))
    return world, rank, local


# --------------------------------------------------------------------------- #
# our arm
# --------------------------------------------------------------------------- #
def build_layers(pkg, wl, dev, seed=0):
    g = torch.Generator(device=dev).manual_seed(seed)
    layers = []
    for _ in range(wl["layers"]):
        gate_up = (torch.randn(wl["E"], 2 * wl["I"], wl["H"], generator=g, device=dev) * 0.02).to(torch.bfloat16)
        down = (torch.randn(wl["E"], wl["H"], wl["I"], generator=g, device=dev) * 0.02).to(torch.bfloat16)
        mod = pkg.Experts4bit.from_float(gate_up, down)
        del gate_up, down
        router = (torch.randn(wl["E"], wl["H"], generator=g, device=dev) * 0.02).to(torch.bfloat16)
        lora = None
        if wl["lora"]:
            r = wl["lora"]
            lm = pkg.ExpertsLoRA(mod, r=r, alpha=16, dtype=torch.bfloat16).to(dev)
            with torch.no_grad():
                for p in (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B):
                    p.copy_(torch.randn(p.shape, generator=g, device=dev) * 0.01)
            lora = (lm.gate_up_lora_A.data, lm.gate_up_lora_B.data, lm.down_lora_A.data, lm.down_lora_B.data,
                    lm.scaling)
            mod = lm.eval()
        layers.append((mod, router, lora))
    torch.cuda.synchronize()
    return layers


def run_ours(args, wl, world, rank, local):
    import importlib
    import ctypes
    pkg = importlib.import_module("experts4bit-qlora_b200")
    N = pkg._native
    ops = pkg.ops
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    layers = build_layers(pkg, wl, dev, seed=rank)
    Lc, T, H = wl["layers"], wl["T"], wl["H"]
    pool = 8
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    X = torch.randn(pool, Lc, T, H, generator=g, device=dev).to(torch.bfloat16)
    outs = torch.empty(Lc, T, H, dtype=torch.bfloat16, device=dev)
    base = lambda m: m.base if hasattr(m, "base") else m  # noqa: E731
    ws = N.workspaces.get(dev, max(ops.moe_workspace_bytes(wl["E"], H, wl["I"], wl["k"], T, lora_rank=wl["lora"]),
                                   ops.moe_decode_step_workspace_bytes(wl["E"], H, wl["I"], wl["k"], T), 1 << 20),
                          "bench")
    rws = N.workspaces.get(dev, N.lib().e4b_router_workspace_bytes(T, wl["E"]), "bench_router")
    topw = torch.empty(Lc, T, wl["k"], dtype=torch.float32, device=dev)
    topi = torch.empty(Lc, T, wl["k"], dtype=torch.int64, device=dev)
    L = N.lib()
    nstage = N.MOE_STAGE_EVENTS

    def layer_call(li, x, events=None):
        mod, router, lora = layers[li]
        b = base(mod)
        if lora is None:  # router + layer in one call (one launch in the decode regime)
            ev = [e.cuda_event for e in events] if events is not None else None
            ops.moe_decode_step(x, router, wl["k"], b.gate_up_proj, b.gate_up_absmax, b.down_proj, b.down_absmax,
                                wl["E"], wl["I"], norm_topk_prob=wl["norm"], out=outs[li], topk_idx=topi[li],
                                topk_w=topw[li], workspace=ws, stage_events=ev)
            return
        N.check(L.e4b_router_topk(x.data_ptr(), N.BF16, router.data_ptr(), N.BF16, T, H, wl["E"], wl["k"],
                                  N.SOFTMAX_THEN_TOPK, int(wl["norm"]), None, topi[li].data_ptr(), topw[li].data_ptr(),
                                  rws.data_ptr(), rws.numel(), torch.cuda.current_stream().cuda_stream), "router")
        d = ops.MoeDesc_from(wl["E"], H, wl["I"], wl["k"], T, True, torch.bfloat16, torch.float32, torch.bfloat16,
                             lora)
        t = N.MoeTensors()
        t.hidden, t.topk_idx, t.topk_w = x.data_ptr(), topi[li].data_ptr(), topw[li].data_ptr()
        t.gate_up_packed, t.gate_up_absmax = b.gate_up_proj.data_ptr(), b.gate_up_absmax.data_ptr()
        t.down_packed, t.down_absmax = b.down_proj.data_ptr(), b.down_absmax.data_ptr()
        if lora is not None:
            t.gate_up_lora_A, t.gate_up_lora_B, t.down_lora_A, t.down_lora_B = (m.data_ptr() for m in lora[:4])
        t.out = outs[li].data_ptr()
        if events is not None:
            arr = (ctypes.c_void_p * nstage)(*[e.cuda_event for e in events])
            t.stage_events = ctypes.cast(arr, ctypes.c_void_p)
            layer_call._keep = arr
        N.check(L.e4b_moe_forward(ctypes.byref(d), ctypes.byref(t), ws.data_ptr(), ws.numel(),
                                  torch.cuda.current_stream().cuda_stream), "moe")

    def step(s, events=None):
        xs = X[s % pool]
        for li in range(Lc):
            layer_call(li, xs[li], events[li] if events is not None else None)

    # --- capture one graph per pool slot (device-resident inputs) ----------------
    stream = torch.cuda.Stream(device=dev)
    stream.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(stream):
        for s in range(pool):
            step(s)
    torch.cuda.current_stream().wait_stream(stream)
    torch.cuda.synchronize()
    graphs = []
    for s in range(pool):
        gr = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gr):
            step(s)
        graphs.append(gr)
    for w in range(max(args.warmup, 3)):
        graphs[w % pool].replay()
    torch.cuda.synchronize()
    # The timed region: `blocks` repetitions of exactly K replayed steps, each bracketed by a barrier
    # and a synchronize; the reported time is the median block (min / max beside it), so the clock
    # sampler sees a long interval while every figure is still a K-step measurement.
    block_ms = []
    with ClockSampler(dev.index if world == 1 else local) as clocks:
        clock_mark = max(0, clocks.mark() - 1)  # the sample just before the region, and those during it
        blocks = args.blocks if args.blocks > 0 else 1
        b_ = 0
        while b_ < blocks:
            b_ += 1
            if world > 1:
                torch.distributed.barrier()
            torch.cuda.synchronize()
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record()
            for s_ in range(args.steps):
                graphs[s_ % pool].replay()
            end.record()
            torch.cuda.synchronize()
            ms_b = start.elapsed_time(end)
            if world > 1:
                t_ = torch.tensor([ms_b], device=dev)
                torch.distributed.all_reduce(t_, op=torch.distributed.ReduceOp.MAX)
                ms_b = float(t_.item())
            block_ms.append(ms_b)
            if args.blocks <= 0 and b_ == 1:  # auto: about one second of timed blocks, 5 to 200 of them
                blocks = int(min(200, max(5, math.ceil(1000.0 / max(ms_b, 1e-3)))))
    ms = statistics.median(block_ms)
    units = args.steps * T * Lc * world
    value = units / (ms / 1e3)

    # --- per-stage kernel times, live, from event nodes inside replayed graphs ----
    # (multi-kernel paths only: the stage boundaries of the one-launch kernels are inside one launch)
    cudart = _cudart()
    ev = [[_RawEvent(cudart) for _ in range(nstage)] for _ in range(Lc)]
    gt = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gt):
        step(0, ev)
    stage_ms = [[] for _ in range(nstage - 1)]
    for rep in range(max(5, min(args.steps, 20))):
        gt.replay()
        torch.cuda.synchronize()
        for li in range(Lc):
            for si in range(nstage - 1):
                stage_ms[si].append(ev[li][si].elapsed_ms(ev[li][si + 1]))
    stage_names = ["permute", "lora_a_x", "gate_up", "lora_a_h", "down", "combine"]
    stage_raw_us = {n: 1e3 * statistics.mean(v) for n, v in zip(stage_names, stage_ms)}
    # Each stage interval spans one event-record graph node besides its kernel(s). Without an
    # adapter the LoRA-A stages are empty, so their interval is exactly that node's cost; it is
    # subtracted from every stage (with an adapter the correction is not available and is 0).
    node_us = min(stage_raw_us["lora_a_x"], stage_raw_us["lora_a_h"]) if not wl["lora"] else 0.0
    stage_avg_us = {n: max(v - node_us, 1e-3) for n, v in stage_raw_us.items()}

    # algorithmic bytes of the dominant kernel (gate_up grouped GEMM), per launch
    E, I, k = wl["E"], wl["I"], wl["k"]
    n1 = 2 * I
    per_expert_gu = n1 * H // 2 + n1 * H // 64 * 4
    per_expert_dn = H * I // 2 + H * I // 64 * 4
    # unique experts touched per layer (measured from the routing of the timed inputs)
    uniq = []
    for s in range(min(pool, 8)):
        for li in range(Lc):
            uniq.append(int(torch.unique(_route_idx(pkg, layers[li][1], X[s][li], wl)).numel()))
    mean_uniq = statistics.mean(uniq)
    gu_bytes = mean_uniq * per_expert_gu + T * H * 2 + T * k * I * 2
    dn_bytes = mean_uniq * per_expert_dn + T * k * I * 2 + T * k * H * 2
    peaks, peak_kind = load_peaks()
    path = ops.moe_path(wl["E"], H, wl["I"], wl["k"], T, lora_rank=wl["lora"])
    one_launch = path == N.PATH_DECODE_LAYER
    if one_launch:
        # router + whole layer in one kernel, the only launch of the step: its time per launch is
        # the driver-timed step time over the layers (kernel time x launches <= ms_per_step)
        layer_us = 1e3 * ms / args.steps / Lc
        bound, unit = "hbm", "GB/s"
        gu_bytes += wl["E"] * H * 2  # the router weights the same launch reads
        achieved = (gu_bytes + dn_bytes) / (layer_us * 1e-6) / 1e9
        peak = peaks["hbm_gbs"]
        kernel_us = layer_us
        stage_report = {"decode_layer": round(layer_us, 3)}
    elif wl["T"] <= 16:
        bound, unit = "hbm", "GB/s"
        achieved = gu_bytes / (stage_avg_us["gate_up"] * 1e-6) / 1e9
        peak = peaks["hbm_gbs"]
        kernel_us = stage_avg_us["gate_up"]
        stage_report = {k_: round(v, 3) for k_, v in stage_avg_us.items()}
    else:
        bound, unit = "tensor", "TFLOP/s"
        flops = 2.0 * T * k * H * n1
        achieved = flops / (stage_avg_us["gate_up"] * 1e-6) / 1e12
        peak = peaks["bf16_tflops"]
        kernel_us = stage_avg_us["gate_up"]
        stage_report = {k_: round(v, 3) for k_, v in stage_avg_us.items()}
    decode_kernel = {"1": "nf4_decode_flow_kernel", "2": "nf4_decode_layer_kernel"}.get(
        os.environ.get("E4B_DECODE_KERNEL", "3"), "nf4_decode_slice_kernel")
    kname = decode_kernel if one_launch else "nf4 grouped gate_up (SwiGLU fused)"
    roofline = {"bound": bound,
                "kernel": ("%s: router + permute + gate_up GEMV (SwiGLU) + down GEMV + combine, one launch per "
                           "layer" % kname if one_launch else "nf4 grouped gate_up (SwiGLU fused)"),
                "achieved": round(achieved, 1),
                "peak": peak, "peak_source": peak_kind + (" (MEASURED_PEAKS.json)" if peak_kind == "measured" else ""),
                "unit": unit, "frac": round(achieved / peak, 4),
                "traffic": (MEASURED_TRAFFIC[args.workload]["bytes"] if args.workload in MEASURED_TRAFFIC else None),
                "traffic_source": (MEASURED_TRAFFIC[args.workload]["source"] if args.workload in MEASURED_TRAFFIC
                                   else None),
                "algorithmic_bytes_per_launch": int(gu_bytes + dn_bytes) if one_launch else int(gu_bytes),
                "kernel_us": round(kernel_us, 3),
                "kernel_us_source": ("ms_per_step / layers (the step is one launch per layer)" if one_launch
                                     else "event-record nodes around the kernel in a replayed graph"),
                "down_kernel_us": None if one_launch else round(stage_avg_us["down"], 3),
                "down_achieved": (round(dn_bytes / (stage_avg_us["down"] * 1e-6) / 1e9, 1)
                                  if bound == "hbm" and not one_launch else None),
                "layer_bytes": int(gu_bytes + dn_bytes + wl["E"] * H * 2),
                "stage_us": stage_report}
    if not one_launch:
        roofline["event_node_us_subtracted"] = round(node_us, 3)

    # --- e2e through the public API: pinned H2D in, eager calls, D2H out ----------
    e2e = run_e2e(pkg, layers, wl, dev, args, X) if not args.skip_e2e else {"ms": float("nan"), "h2d": 0, "d2h": 0}
    if world > 1:
        t_ = torch.tensor([e2e["ms"]], device=dev)
        torch.distributed.all_reduce(t_, op=torch.distributed.ReduceOp.MAX)
        e2e["ms"] = float(t_.item())
    e2e_value = args.steps * T * Lc * world / (e2e["ms"] / 1e3)

    # router 2; then one layer kernel, or permute, [lora x2], gate_up, down, combine
    launches_per_layer = 1 if one_launch else 2 + (5 if wl["lora"] else 3) + 1
    result = {
        "metric": "MoE-layer tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights quantized to NF4; N(0,1) tokens)",
        "config": config_of(args, wl, world),
        "model_tokens_per_s": round(value / Lc, 1),
        "roofline": roofline,
        "e2e": {"value": round(e2e_value, 1), "unit": "tokens/s", "h2d_bytes_per_step": e2e["h2d"],
                "d2h_bytes_per_step": e2e["d2h"], "path": "public API (route + enable_fast module call), eager"},
        "gpu_launches": launches_per_layer * Lc * args.steps,
        "clocks": clocks.summary(since=clock_mark),
        "timed_blocks": {"n": blocks, "steps_each": args.steps, "ms_min": round(min(block_ms), 4),
                         "ms_median": round(ms, 4), "ms_max": round(max(block_ms), 4)},
        "unique_experts_per_layer": round(mean_uniq, 2),
    }
    if rank == 0 and args.cpu_seconds > 0:
        result["cpu_baseline"] = cpu_baseline(wl, seconds=args.cpu_seconds)
    return result


def build_ep_layers(pkg, wl, dev, rank, world):
    """The rank's expert slice of every layer. Expert e of layer l is drawn from its own
    seed, so a slice holds the same weights whatever the world size."""
    ep = pkg.ep
    f8 = pkg.fp8_experts
    E, H, I = wl["E"], wl["H"], wl["I"]
    El = E // world
    fp8 = wl.get("fmt") == "fp8"
    shards, routers = [], []
    for li in range(wl["layers"]):
        parts = {"gu": [], "gua": [], "dn": [], "dna": []}
        for e in range(rank * El, (rank + 1) * El):
            g = torch.Generator(device=dev).manual_seed(1_000_003 * li + e)
            for key, shape in (("gu", (2 * I, H)), ("dn", (H, I))):
                w = (torch.randn(shape, generator=g, device=dev) * 0.02).to(torch.bfloat16)
                if fp8:
                    q, sc = f8.quantize_fp8_blocks(w, "e8m0")
                    packed, absmax = q, f8.scale_values(sc)
                else:
                    packed, absmax = pkg.ops.nf4_quantize(w)
                parts[key].append(packed)
                parts[key + "a"].append(absmax)
                del w
        shards.append(ep.ExpertShard(torch.stack(parts["gu"]), torch.stack(parts["gua"]), torch.stack(parts["dn"]),
                                     torch.stack(parts["dna"]), rank * El, El, None,
                                     pkg._native.FMT_FP8_BLOCK128 if fp8 else pkg._native.FMT_NF4))
        g = torch.Generator(device=dev).manual_seed(7_000_001 + li)
        routers.append((torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16))
    torch.cuda.synchronize()
    return shards, routers


def run_train(args, wl, world, rank, local):
    """One training step (forward + backward to dL/dx, dL/dw and the adapter gradients) of an
    ``ExpertsLoRA`` layer through ``enable_fast_train``, and the unpatched loop beside it."""
    import importlib
    pkg = importlib.import_module("experts4bit-qlora_b200")
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    E, H, I, k, T, r = wl["E"], wl["H"], wl["I"], wl["k"], wl["T"], wl["lora"]
    g = torch.Generator(device=dev).manual_seed(rank)
    gate_up = (torch.randn(E, 2 * I, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    base = pkg.Experts4bit.from_float(gate_up, down, compute_dtype=torch.bfloat16)
    del gate_up, down
    mod = pkg.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.float32).to(dev).train()
    with torch.no_grad():
        for p in (mod.gate_up_lora_B, mod.down_lora_B):
            p.normal_(0, 0.01, generator=g)
    router = (torch.randn(E, H, generator=g, device=dev) * 0.02).to(torch.bfloat16)
    pool = 4
    X = torch.randn(pool, T, H, generator=g, device=dev).to(torch.bfloat16)
    routes = [pkg.route(X[i], router, k, norm_topk_prob=True) for i in range(pool)]
    loss_w = torch.randn(T, H, generator=g, device=dev)

    def step(s):
        w, idx = routes[s % pool]
        x = X[s % pool].clone().requires_grad_(True)
        ww = w.clone().requires_grad_(True)
        out = mod(x, idx, ww)
        (out.float() * loss_w).sum().backward()
        return x.grad

    def timed(n, w):
        for s in range(w):
            step(s)
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for s in range(n):
            step(s)
        b.record()
        torch.cuda.synchronize()
        return a.elapsed_time(b) / n

    ref_ms = timed(3, 1)  # the unpatched per-expert loop (the reference's training forward)
    # the backward's input gradients decoded once per stack + batched GEMMs (dgrad=False), then
    # through the library's dgrad kernel (dgrad=True, the timed configuration)
    if pkg.enable_fast_train(mod, dgrad=False) != 1:
        raise SystemExit("enable_fast_train declined the layer")
    decode_once_ms = timed(max(args.steps // 2, 1), 2)
    pkg.disable_fast_train(mod)
    if pkg.enable_fast_train(mod, dgrad=True) != 1:
        raise SystemExit("enable_fast_train declined the layer")
    with ClockSampler(local) as clocks:
        ms = timed(args.steps, max(args.warmup, 3))
    R = T * k
    n1 = 2 * I
    flops = 2.0 * R * H * n1 + 2.0 * R * I * H  # one pass of both frozen projections
    flops_step = 2 * flops                      # forward + the two input-gradient products
    peaks, peak_kind = load_peaks()
    ach = flops_step / (ms * 1e-3) / 1e12
    return {
        "metric": "MoE-layer training tokens/s (forward + backward)", "value": round(T / (ms * 1e-3), 1),
        "unit": "tokens/s", "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights quantized to NF4; N(0,1) tokens; random router)",
        "config": {"workload": args.workload, "desc": wl["desc"], "tokens": T, "experts": E, "hidden": H,
                   "intermediate": I, "top_k": k, "lora_rank": r,
                   "l2": "inputs larger than L2: each step reads the 300 MB layer and its decoded stacks"},
        "roofline": {"bound": "tensor", "kernel": "whole step (frozen projections forward + input gradients)",
                     "achieved": round(ach, 1), "peak": peaks["bf16_tflops"], "peak_source": peak_kind,
                     "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4), "traffic": None},
        "reference_loop": {"value": round(T / (ref_ms * 1e-3), 1), "unit": "tokens/s",
                           "what": "the unpatched ExpertsLoRA per-expert loop, same GPU, same step"},
        "dgrad": "kernel (enable_fast_train(dgrad=True): e4b_grouped_nf4_dgrad for both input gradients)",
        "decode_once": {"value": round(T / (decode_once_ms * 1e-3), 1), "unit": "tokens/s",
                        "what": "enable_fast_train(dgrad=False): each frozen stack decoded once per backward, "
                                "batched GEMMs"},
        "clocks": clocks.summary(),
    }


def run_ep(args, wl, world, rank, local):
    """Expert-parallel layer over `world` ranks (config 4). One step = one MoE layer over
    the T global tokens (layers cycled), T/world tokens and E/world experts per rank;
    exchanges are NCCL all-to-alls over NVLink. Not graph-captured: the row splits need
    one host sync per layer."""
    import importlib
    pkg = importlib.import_module("experts4bit-qlora_b200")
    N = pkg._native
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    if wl["E"] % world:
        raise SystemExit(f"{wl['E']} experts do not split over {world} ranks")
    E, H, I, k, Lc = wl["E"], wl["H"], wl["I"], wl["k"], wl["layers"]
    T = wl["T"] // world
    shards, routers = build_ep_layers(pkg, wl, dev, rank, world)
    layers = [pkg.ExpertParallelMoE(sh, E, H, I, True, exchange=args.exchange, max_tokens=T) for sh in shards]
    pool = 4
    g = torch.Generator(device=dev).manual_seed(1000 + rank)
    X = torch.randn(pool, T, H, generator=g, device=dev).to(torch.bfloat16)
    zipf = wl.get("routing") == "zipf"
    routes = None
    if zipf:  # Zipf(1.1) popularity over a seeded permutation of the experts, the same on every rank
        gp = torch.Generator(device=dev).manual_seed(4242)
        perm = torch.randperm(E, generator=gp, device=dev)
        pop = torch.empty(E, device=dev)
        pop[perm] = 1.0 / torch.arange(1, E + 1, device=dev, dtype=torch.float32) ** 1.1
        routes = []
        for _ in range(pool):
            idx = torch.multinomial(pop.expand(T, E), k, replacement=False, generator=g)
            w = torch.softmax(torch.randn(T, k, generator=g, device=dev), -1)
            routes.append((w, idx))

    def route(s, x):
        if zipf:
            return routes[s % pool]
        return pkg.route(x, routers[s % Lc], k, norm_topk_prob=wl["norm"])

    def step(s, x=None):
        li = s % Lc
        x = X[s % pool] if x is None else x
        w, idx = route(s, x)
        return layers[li](x, idx, w, micro_batches=args.micro_batches)

    for s in range(max(args.warmup, 3)):
        step(s)
    torch.cuda.synchronize()
    # Peer exchange (or one rank): nothing waits on the host, so each layer's step (route + layer)
    # is captured once as a CUDA graph and replayed; the NCCL path needs a host sync per layer.
    peer = world > 1 and layers[0]._use_peer(X[0])
    graphs = None
    if (peer or world == 1) and not args.eager:
        for li in range(Lc):  # first calls (one-time set-up) outside the capture
            step(li)
        torch.cuda.synchronize()
        graphs, mempool = [], None
        for li in range(Lc):
            g_ = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g_, pool=mempool):
                step(li)
            mempool = g_.pool()
            graphs.append(g_)
        for li in range(Lc):
            graphs[li].replay()
        torch.cuda.synchronize()
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        if world > 1:  # after every rank's sampler is up, so all ranks enter the region together
            torch.distributed.barrier()
        torch.cuda.synchronize()
        clock_mark = max(0, clocks.mark() - 1)  # the sample just before the region, and those during it
        marks = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)] if args.trace else None
        host_t0 = time.perf_counter()
        start.record()
        for s in range(args.steps):
            if marks:
                marks[s].record()
            if graphs is not None:
                graphs[s % Lc].replay()
            else:
                step(s)
        if marks:
            marks[-1].record()
        end.record()
        host_ms = (time.perf_counter() - host_t0) * 1e3
        torch.cuda.synchronize()
    ms = start.elapsed_time(end)
    if world > 1:
        t_ = torch.tensor([ms], device=dev)
        torch.distributed.all_reduce(t_, op=torch.distributed.ReduceOp.MAX)
        ms = float(t_.item())
    value = args.steps * wl["T"] / (ms / 1e3)
    trace = None
    if marks:
        per = [marks[i].elapsed_time(marks[i + 1]) for i in range(args.steps)]
        by_layer = {}
        for i, v in enumerate(per):
            by_layer.setdefault(i % Lc, []).append(v)
        trace = {"host_enqueue_ms_per_step": round(host_ms / args.steps, 4),
                 "step_ms": {"min": round(min(per), 4), "median": round(statistics.median(per), 4),
                             "max": round(max(per), 4)},
                 "layer_ms": [round(statistics.mean(by_layer[li]), 3) for li in sorted(by_layer)]}

    # phase breakdown of one layer on every rank (events between phases; outside the timed region)
    def phases(s):
        li = s % Lc
        x = X[s % pool]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(8)]
        lay = layers[li]
        ev[0].record()
        w, idx = route(s, x)
        ev[1].record()
        send, counts, inv = lay.stages.dispatch(x, idx)
        ev[2].record()
        rc, ss, rs = lay.exchange_counts(counts)
        ev[3].record()
        rows = torch.empty(sum(rs), H, dtype=send.dtype, device=dev)
        if world > 1:
            torch.distributed.all_to_all_single(rows, send, rs, ss)
        else:
            rows.copy_(send)
        ev[4].record()
        back = lay.stages.experts(rows, rc)
        ev[5].record()
        ret = torch.empty(T * k, H, dtype=back.dtype, device=dev)
        if world > 1:
            torch.distributed.all_to_all_single(ret, back, ss, rs)
        else:
            ret.copy_(back)
        ev[6].record()
        lay.stages.combine(ret, inv, w, T, k, x.dtype)
        ev[7].record()
        torch.cuda.synchronize()
        return [ev[i].elapsed_time(ev[i + 1]) * 1e3 for i in range(7)]

    def phases_peer(s):
        li = s % Lc
        x = X[s % pool]
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(5)]
        ev[0].record()
        w, idx = route(s, x)
        layers[li]._forward_peer(x, idx.long(), w, x.dtype, phase_events=ev[1:])
        torch.cuda.synchronize()
        return [ev[i].elapsed_time(ev[i + 1]) * 1e3 for i in range(4)]

    if peer:
        ph = [phases_peer(s) for s in range(6)][2:]
        phase_names = ["router", "dispatch_peer", "experts_peer", "combine_peer"]
    else:
        ph = [phases(s) for s in range(6)][2:]
        phase_names = ["router", "dispatch", "count_exchange_sync", "rows_a2a", "experts", "return_a2a", "combine"]
    phase_us = {n: round(statistics.mean(v[i] for v in ph), 1) for i, n in enumerate(phase_names)}

    # per-stage device times of this rank's expert side, from the library's stage events
    cudart = _cudart()
    nst = N.MOE_STAGE_EVENTS
    stage_ms = [[] for _ in range(nst - 1)]
    recv_rows, uniq = [], []
    for rep in range(4):
        li = rep % Lc
        x = X[rep % pool]
        w, idx = route(rep, x)
        lay = layers[li]
        ev = [_RawEvent(cudart) for _ in range(nst)]
        if peer:
            lay._forward_peer(x, idx.long(), w, x.dtype, stage_events=[e.cuda_event for e in ev])
            torch.cuda.synchronize()
            for si in range(nst - 1):
                stage_ms[si].append(ev[si].elapsed_ms(ev[si + 1]))
            cnt = torch.bincount(idx.reshape(-1).long(), minlength=E)  # rows each expert gets, all ranks
            torch.distributed.all_reduce(cnt)
            mine = cnt[rank * (E // world):(rank + 1) * (E // world)]
            recv_rows.append(int(mine.sum().item()))
            uniq.append(int((mine > 0).sum().item()))
            continue
        send, counts, inv = lay.stages.dispatch(x, idx)
        rc, ss, rs = lay.exchange_counts(counts)
        rows = torch.empty(sum(rs), H, dtype=send.dtype, device=dev)
        if world > 1:
            torch.distributed.all_to_all_single(rows, send, rs, ss)
        else:
            rows.copy_(send)
        lay.stages.experts(rows, rc, events=[e.cuda_event for e in ev])
        torch.cuda.synchronize()
        for si in range(nst - 1):
            stage_ms[si].append(ev[si].elapsed_ms(ev[si + 1]))
        recv_rows.append(rows.shape[0])
        uniq.append(int((rc.sum(0) > 0).sum().item()))
    names = ["plan", "convert", "gate_up", "lora_a_h", "down", "scatter"]
    st_us = {n: 1e3 * statistics.mean(v) for n, v in zip(names, stage_ms)}
    Rr = statistics.mean(recv_rows)
    peaks, peak_kind = load_peaks()
    wfmt = "fp8 e4m3 128x128" if wl.get("fmt") == "fp8" else "nf4"
    if wl.get("bound", "tensor") == "hbm":
        per_el = 1.0 if wl.get("fmt") == "fp8" else 0.5 + 4 / 64
        gu_bytes = statistics.mean(uniq) * 2 * I * H * per_el
        dn_bytes = statistics.mean(uniq) * H * I * per_el
        achieved = gu_bytes / (st_us["gate_up"] * 1e-6) / 1e9
        peak, unit, bound = peaks["hbm_gbs"], "GB/s", "hbm"
        down_ach = dn_bytes / (st_us["down"] * 1e-6) / 1e9
    else:
        achieved = 2.0 * Rr * H * 2 * I / (st_us["gate_up"] * 1e-6) / 1e12
        peak, unit, bound = peaks["bf16_tflops"], "TFLOP/s", "tensor"
        down_ach = 2.0 * Rr * H * I / (st_us["down"] * 1e-6) / 1e12
    roofline = {"bound": bound, "kernel": f"{wfmt} grouped gate_up (SwiGLU fused), rank 0 expert side",
                "achieved": round(achieved, 1), "peak": peak, "peak_source": peak_kind, "unit": unit,
                "frac": round(achieved / peak, 4), "traffic": None, "kernel_us": round(st_us["gate_up"], 1),
                "down_kernel_us": round(st_us["down"], 1), "down_achieved": round(down_ach, 1),
                "unique_local_experts": round(statistics.mean(uniq), 2),
                "rows_received": int(Rr), "stage_us": {n: round(v, 1) for n, v in st_us.items()},
                "nvlink_bytes_per_layer_per_rank": int(2 * T * k * H * 2 * (world - 1) / world),
                "phase_us_rank%d" % rank: phase_us}
    if trace:
        roofline["trace_rank%d" % rank] = trace

    # e2e through the public API: pinned host tokens in, route + layer, output back to the host
    host_in = torch.empty(pool, T, H, dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(X.cpu())
    host_out = torch.empty(T, H, dtype=torch.bfloat16, pin_memory=True)
    e2e_steps = max(3, min(args.steps, 50))

    def one(s):
        x = host_in[s % pool].to(dev, non_blocking=True)
        with torch.no_grad():
            y = step(s, x)
        host_out.copy_(y, non_blocking=True)

    for s in range(3):
        one(s)
    torch.cuda.synchronize()
    if world > 1:
        torch.distributed.barrier()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(e2e_steps):
        one(s)
    b.record()
    torch.cuda.synchronize()
    e2e_ms = a.elapsed_time(b)
    if world > 1:
        t_ = torch.tensor([e2e_ms], device=dev)
        torch.distributed.all_reduce(t_, op=torch.distributed.ReduceOp.MAX)
        e2e_ms = float(t_.item())
    layer_gb = wl["E"] * (2 * I * H + H * I) * (1.0 if wl.get("fmt") == "fp8" else 0.5 + 4 / 64) / 1e9
    result = {
        "metric": "MoE-layer tokens/s", "value": round(value, 1), "unit": "tokens/s", "n_gpus": world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 4),
        "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
        "data": "synthetic (random-init N(0,0.02) weights quantized to %s; N(0,1) tokens; %s)" % (
            "FP8 e4m3 with e8m0 128x128 scales" if wl.get("fmt") == "fp8" else "NF4",
            "routes sampled from Zipf(1.1) expert popularity" if wl.get("routing") == "zipf" else "random router"),
        "config": config_of(args, wl, world),
        "run": {"micro_batches": args.micro_batches or "default",
                "launch": "one CUDA graph per layer step, replayed" if graphs is not None else "eager",
                "exchange": ("peer-memory stores (CUDA IPC over NVLink)" if peer else
                             "NCCL all-to-all" if world > 1 else "none (one rank)")},
        "roofline": roofline,
        "e2e": {"value": round(e2e_steps * wl["T"] / (e2e_ms / 1e3), 1), "unit": "tokens/s",
                "h2d_bytes_per_step": T * H * 2 * world, "d2h_bytes_per_step": T * H * 2 * world,
                "path": "public API (route + ExpertParallelMoE), pinned host tokens in, outputs out"},
        "gpu_launches": 10 * args.steps,
        "clocks": clocks.summary(since=clock_mark),
    }
    if rank == 0 and world == 1 and args.cpu_seconds > 0:
        result["cpu_baseline"] = cpu_baseline(wl, seconds=args.cpu_seconds)
    return result


def prefill_record(args, world, rank, local):
    """Config 3 (Qwen3 geometry, T=4096, LoRA r=16) timed in the same run: the prefill regime's
    tensor-core figures beside the decode headline. Bounded: a few layers, 10 steps."""
    import copy
    a2 = copy.copy(args)
    a2.workload, a2.steps, a2.warmup, a2.blocks = "qwen3-prefill", min(args.steps, 10), 3, 5
    a2.skip_e2e, a2.cpu_seconds = True, 0.0
    wl = dict(WORKLOADS["qwen3-prefill"])
    r = run_ours(a2, wl, world, rank, local)
    E, H, I, k, T, lr = wl["E"], wl["H"], wl["I"], wl["k"], wl["T"], wl["lora"]
    R = T * k
    layer_flops = 2.0 * R * H * 2 * I + 2.0 * R * I * H + 2.0 * R * lr * (H + 2 * I) + 2.0 * R * lr * (I + H)
    layer_ms = r["ms_per_step"] / wl["layers"]
    peaks, peak_kind = load_peaks()
    ach = layer_flops / (layer_ms * 1e-3) / 1e12
    torch.cuda.empty_cache()
    return {"workload": "qwen3-prefill", "desc": wl["desc"], "value": r["value"], "unit": "tokens/s",
            "ms_per_layer": round(layer_ms, 4), "roofline": r["roofline"],
            "layer_tensor": {"bound": "tensor", "achieved": round(ach, 1), "peak": peaks["bf16_tflops"],
                             "unit": "TFLOP/s", "frac": round(ach / peaks["bf16_tflops"], 4),
                             "flops_per_layer": layer_flops,
                             "what": "all of the layer (permute, LoRA-A, both grouped GEMMs, combine) over "
                                     "its dense FLOPs, base + adapters"},
            "clocks": r["clocks"], "timed_blocks": r["timed_blocks"]}


def _cudart():
    import ctypes
    for name in ("/usr/local/cuda/lib64/libcudart.so", "libcudart.so", "libcudart.so.12"):
        try:
            return ctypes.CDLL(name)
        except OSError:
            continue
    raise RuntimeError("libcudart not found")


class _RawEvent:
    """A timing cudaEvent_t owned here (torch's Event refuses elapsed_time on events
    recorded outside torch, e.g. by the library's graph event-record nodes)."""

    def __init__(self, cudart):
        import ctypes
        self._rt = cudart
        h = ctypes.c_void_p()
        if cudart.cudaEventCreate(ctypes.byref(h)) != 0:
            raise RuntimeError("cudaEventCreate failed")
        self.cuda_event = h.value

    def elapsed_ms(self, other):
        import ctypes
        out = ctypes.c_float()
        rc = self._rt.cudaEventElapsedTime(ctypes.byref(out), ctypes.c_void_p(self.cuda_event),
                                           ctypes.c_void_p(other.cuda_event))
        if rc != 0:
            raise RuntimeError(f"cudaEventElapsedTime failed ({rc})")
        return out.value


def _route_idx(pkg, router, x, wl):
    w, idx = pkg.route(x, router, wl["k"], norm_topk_prob=wl["norm"])
    return idx


def run_e2e(pkg, layers, wl, dev, args, X):
    Lc, T, H = wl["layers"], wl["T"], wl["H"]
    pool = X.shape[0]
    host_in = torch.empty(pool, Lc, T, H, dtype=torch.bfloat16, pin_memory=True)
    host_in.copy_(X.cpu())
    host_out = torch.empty(Lc, T, H, dtype=torch.bfloat16, pin_memory=True)
    for mod, _, _ in layers:
        pkg.enable_fast(mod)

    def one(s):
        xs = host_in[s % pool].to(dev, non_blocking=True)
        outs = []
        with torch.no_grad():
            for li in range(Lc):
                mod, router, _ = layers[li]
                w, idx = pkg.route(xs[li], router, wl["k"], norm_topk_prob=wl["norm"])
                outs.append(mod(xs[li], idx, w))
        host_out.copy_(torch.stack(outs), non_blocking=True)

    for s in range(max(args.warmup, 3)):
        one(s)
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record()
    for s in range(args.steps):
        one(s)
    b.record()
    torch.cuda.synchronize()
    return {"ms": a.elapsed_time(b), "h2d": Lc * T * H * 2, "d2h": Lc * T * H * 2}


# --------------------------------------------------------------------------- #
# CPU baseline: the reference's per-expert loop restated on CPU (oracle port)
# --------------------------------------------------------------------------- #
def cpu_baseline(wl, seconds=15.0, threads=None):
    """Times the reference loop (``ExpertsNbit.forward``, experts4bit_qlora/_vendor/experts.py:468-516,
    restated in oracle/moe.py) on the host cores, on a bounded sample of the same workload:
    one layer of the workload's geometry, its T tokens per call, repeated for ~``seconds``."""
    from oracle import moe as M
    from oracle.nf4 import quantize_stack

    ncores = len(os.sched_getaffinity(0))
    torch.set_num_threads(threads or ncores)
    g = torch.Generator().manual_seed(0)
    E, H, I, k = wl["E"], wl["H"], wl["I"], wl["k"]
    big = H * I > 16 * 2**20
    T = min(wl["T"], 16 if big else 128)
    if wl.get("fmt") == "fp8":
        T = min(T, 8)  # one call dequantizes every hit expert of a 256-expert layer
    # quantize a handful of distinct experts and reuse them (quantization is not timed)
    ne = 1 if big else min(E, 8)
    if wl.get("fmt") == "fp8":
        import importlib
        f8 = importlib.import_module("experts4bit-qlora_b200.fp8_experts")
        gq, gs = f8.quantize_fp8_blocks((torch.randn(1, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16))
        dq, ds = f8.quantize_fp8_blocks((torch.randn(1, H, I, generator=g) * 0.02).to(torch.bfloat16))
        st = {"format": "fp8", "gate_up_w": gq.expand(E, -1, -1), "gate_up_scale": gs.expand(E, -1, -1),
              "down_w": dq.expand(E, -1, -1), "down_scale": ds.expand(E, -1, -1), "E": E, "H": H, "I": I,
              "has_gate": True}
    else:
        gp, ga = quantize_stack((torch.randn(ne, 2 * I, H, generator=g) * 0.02).to(torch.bfloat16))
        dp, da = quantize_stack((torch.randn(ne, H, I, generator=g) * 0.02).to(torch.bfloat16))
        rep = (E + ne - 1) // ne
        st = {"gate_up_packed": gp.repeat(rep, 1)[:E], "gate_up_absmax": ga.repeat(rep, 1)[:E],
              "down_packed": dp.repeat(rep, 1)[:E], "down_absmax": da.repeat(rep, 1)[:E],
              "E": E, "H": H, "I": I, "has_gate": True}
    router = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    n_tok = 0
    t0 = time.perf_counter()
    while time.perf_counter() - t0 < seconds:
        x = torch.randn(T, H, generator=g).to(torch.bfloat16)
        w, idx = M.route_on_host(M.router_logits_f32(x, router), k, M.SOFTMAX_THEN_TOPK, wl["norm"])
        M.reference_forward(st, x, idx, w, torch.bfloat16)
        n_tok += T
    dt = time.perf_counter() - t0
    return {"value": round(n_tok / dt, 2), "unit": "tokens/s", "cores": torch.get_num_threads(), "kind": "port",
            "sample": f"reference per-expert loop (oracle port, torch CPU) on one {E}-expert layer, {T} token(s) "
                      f"per call, {n_tok} tokens in {dt:.1f} s"}


def run_reference(args, wl, rank):
    if rank != 0:
        return None
    cb = cpu_baseline(wl, seconds=max(5.0, min(60.0, 2.0 * args.steps)))
    return {"metric": "MoE-layer tokens/s", "value": cb["value"], "unit": "tokens/s", "impl": "reference",
            "n_gpus": int(os.environ.get("WORLD_SIZE", "1")), "steps": args.steps, "warmup": args.warmup,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic", "config": config_of(args, wl, int(os.environ.get("WORLD_SIZE", "1"))),
            "cpu_baseline": cb, "e2e": {"value": cb["value"], "unit": "tokens/s", "h2d_bytes_per_step": 0,
                                        "d2h_bytes_per_step": 0}}


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="auto", choices=["auto"] + sorted(WORKLOADS),
                    help="auto: olmoe-decode on one GPU, mixtral-ep (expert parallel) on several")
    ap.add_argument("--cpu-seconds", type=float, default=15.0, help="0 skips the CPU baseline")
    ap.add_argument("--layers", type=int, default=0, help="override the workload's layer count (profiling)")
    ap.add_argument("--micro-batches", type=int, default=None,
                    help="expert-parallel micro-batches per layer (default: the layer's own choice)")
    ap.add_argument("--trace", action="store_true", help="per-step device times inside the timed region")
    ap.add_argument("--eager", action="store_true", help="expert-parallel steps without CUDA graphs")
    ap.add_argument("--exchange", choices=["auto", "peer", "nccl"], default="auto",
                    help="expert-parallel exchange: peer-memory stores or NCCL all-to-alls")
    ap.add_argument("--skip-e2e", action="store_true", help="skip the public-API e2e leg (profiling)")
    ap.add_argument("--blocks", type=int, default=0,
                    help="timed blocks of K steps (median reported); 0 = enough blocks for about one second")
    ap.add_argument("--prefill-record", type=int, default=1,
                    help="with the default decode workload on one GPU, also time config 3 (Qwen3 prefill) "
                         "and add it as the line's `prefill` record")
    args = ap.parse_args()
    if args.workload == "auto":
        # Under torch.distributed.run (WORLD_SIZE set, the driver's scaling series) every N, N=1
        # included, runs the expert-parallel Mixtral layer, so the series compares one workload; a
        # plain one-GPU run is the OLMoE decode step (config 2), the headline line.
        launched = "WORLD_SIZE" in os.environ
        args.workload = "mixtral-ep" if (launched or args.gpus > 1) else "olmoe-decode"
    wl = dict(WORKLOADS[args.workload])
    if args.layers:
        wl["layers"] = args.layers
    if args.impl == "reference":
        rank = int(os.environ.get("RANK", "0"))
        res = run_reference(args, wl, rank)
        if res is not None:
            print(json.dumps(res), flush=True)
        return
    world, rank, local = dist_setup(args.gpus)
    res = (run_ep if wl.get("ep") else run_train if wl.get("train") else run_ours)(args, wl, world, rank, local)
    if args.workload == "olmoe-decode" and world == 1 and args.prefill_record:
        res["prefill"] = prefill_record(args, world, rank, local)
    if rank == 0:
        print(json.dumps(res), flush=True)
    if world > 1:
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
