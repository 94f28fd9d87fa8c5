"""GPU: the whole fused expert layer (e4b_moe_forward) and the drop-in module API.

Parity bars (the layer tolerance of this path, and the reference's tests/test_fast.py:71-91):
  * vs the fp32 anchor (fp32 dequantized NF4 values, fp32 math):
    max-rel <= 1e-2 and mean-rel <= 2e-3 (norm-relative: max|d|/max|ref|, mean|d|/mean|ref|);
  * vs the reference's bf16 loop: max-rel < 1.5e-2, and err_fast <= max(2 * err_ref, 5e-3).
"""
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")
GOLD = os.path.join(os.path.dirname(__file__), "golden")
MAX_REL, MEAN_REL = 1e-2, 2e-3


def _gold(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def _bf16(u16):
    return torch.from_numpy(u16.view(np.int16)).view(torch.bfloat16)


def _module_from_case(e4b, case, cls=None):
    st = case["st"]
    cls = cls or e4b.Experts4bit
    m = cls(st["E"], st["H"], st["I"], has_gate=st["has_gate"], compute_dtype=torch.bfloat16, device=DEV)
    with torch.no_grad():
        m.gate_up_proj.copy_(st["gate_up_packed"])
        m.down_proj.copy_(st["down_packed"])
        m.gate_up_absmax.copy_(st["gate_up_absmax"])
        m.down_absmax.copy_(st["down_absmax"])
    if case["lora"] is None:
        return m.eval()
    L = case["lora"]
    lm = e4b.ExpertsLoRA(m, r=L["r"], alpha=L["alpha"], dtype=L["gate_up_A"].dtype).to(DEV)
    with torch.no_grad():
        lm.gate_up_lora_A.copy_(L["gate_up_A"])
        lm.gate_up_lora_B.copy_(L["gate_up_B"])
        lm.down_lora_A.copy_(L["down_A"])
        lm.down_lora_B.copy_(L["down_B"])
    return lm.eval()


@pytest.mark.parametrize("name", C.CASES)
def test_golden_cases_fused_vs_reference(e4b, name):
    g = _gold(name)
    case = C.build(name)
    mod = _module_from_case(e4b, case)
    x, idx, w = case["x"].to(DEV), case["idx"].to(DEV), case["w"].to(DEV)
    assert e4b.enable_fast(mod) == 1
    with torch.no_grad():
        got = mod(x, idx, w).cpu()
    assert got.dtype == case["x"].dtype and got.shape == case["x"].shape
    anchor = torch.from_numpy(g["fp32_oracle"])
    ref = _bf16(g["ref_loop"])
    mx, mean = M.rel_errors(got, anchor)
    assert mx <= MAX_REL and mean <= MEAN_REL, (name, mx, mean)
    assert M.rel_errors(got, ref)[0] < 1.5e-2
    err_ref = M.rel_errors(ref, anchor)[0]
    assert mx <= max(2 * err_ref, 5e-3), (mx, err_ref)
    # disable restores the reference path bit-exactly against itself
    with torch.no_grad():
        e4b.disable_fast(mod)
        back1 = mod(x, idx, w)
        back2 = mod(x, idx, w)
    assert torch.equal(back1, back2)


@pytest.mark.parametrize("T", [1, 4, 16, 128])
def test_olmoe_layer_vs_fp32(e4b, T):
    """OLMoE layer geometry (E=64, H=2048, I=1024, top-8) at T tokens."""
    E, H, I, k = 64, 2048, 1024, 8
    g = torch.Generator(device=DEV).manual_seed(0)
    gate_up = (torch.randn(E, 2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    mod = e4b.Experts4bit.from_float(gate_up, down)
    del gate_up, down
    wr = (torch.randn(E, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    w, idx = e4b.route(x, wr, k)
    with torch.no_grad():
        ref_loop = mod(x, idx, w)
        e4b.enable_fast(mod)
        got = mod(x, idx, w)
    anchor = _fp32_anchor_gpu(mod, x, idx, w)
    mx, mean = M.rel_errors(got, anchor)
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)
    err_ref = M.rel_errors(ref_loop, anchor)[0]
    assert mx <= max(2 * err_ref, 5e-3), (mx, err_ref)


def _fp32_anchor_gpu(mod, x, idx, w, lora=None):
    """fp32 forward over the module's dequantized NF4 values (dequant is bit-exact
    against the oracle; see test_gpu_kernels), computed with fp32 torch matmuls."""
    prev = torch.backends.cuda.matmul.allow_tf32
    torch.backends.cuda.matmul.allow_tf32 = False
    try:
        out = torch.zeros(x.shape[0], mod.hidden_dim, dtype=torch.float32, device=x.device)
        xf = x.float()
        for e in torch.unique(idx).tolist():
            tok, pos = torch.where(idx == e)
            wgu = mod._dequantize_expert(mod.gate_up_proj, mod.gate_up_absmax, mod._gate_up_shape, e, torch.float32)
            wdn = mod._dequantize_expert(mod.down_proj, mod.down_absmax, mod._down_shape, e, torch.float32)
            h = xf[tok] @ wgu.t()
            if lora is not None:
                h = h + lora[4] * ((xf[tok] @ lora[0][e].float().t()) @ lora[1][e].float().t())
            gg, u = h.chunk(2, -1)
            h = torch.nn.functional.silu(gg) * u
            d = h @ wdn.t()
            if lora is not None:
                d = d + lora[4] * ((h @ lora[2][e].float().t()) @ lora[3][e].float().t())
            out.index_add_(0, tok, d * w[tok, pos, None].float())
        return out
    finally:
        torch.backends.cuda.matmul.allow_tf32 = prev


@pytest.mark.parametrize("T,E,H,I,k,r", [(1, 64, 2048, 1024, 8, 16), (24, 128, 2048, 768, 8, 16),
                                         (300, 128, 2048, 768, 8, 16)])
def test_lora_layer_vs_fp32(e4b, T, E, H, I, k, r):
    g = torch.Generator(device=DEV).manual_seed(3)
    gate_up = (torch.randn(E, 2 * I, H, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    down = (torch.randn(E, H, I, generator=g, device=DEV) * 0.02).to(torch.bfloat16)
    base = e4b.Experts4bit.from_float(gate_up, down)
    lm = e4b.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.bfloat16).to(DEV)
    with torch.no_grad():
        for p in (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B):
            p.copy_(torch.randn(p.shape, generator=g, device=DEV) * 0.01)
    lm.eval()
    x = torch.randn(T, H, generator=g, device=DEV).to(torch.bfloat16)
    logits = torch.randn(T, E, generator=g, device=DEV)
    w, idx = torch.topk(torch.softmax(logits, -1), k)
    with torch.no_grad():
        e4b.enable_fast(lm)
        got = lm(x, idx, w)
    lora = (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B, lm.scaling)
    anchor = _fp32_anchor_gpu(base, x, idx, w, lora)
    mx, mean = M.rel_errors(got, anchor)
    assert mx <= MAX_REL and mean <= MEAN_REL, (mx, mean)
    # the adapter is load-bearing: dropping it is far outside the bar
    no_lora = _fp32_anchor_gpu(base, x, idx, w)
    assert M.rel_errors(no_lora, anchor)[1] > 10 * mean


def test_repeat_forwards_are_bit_identical(e4b):
    case = C.build("olmoe_like")
    mod = _module_from_case(e4b, case)
    e4b.enable_fast(mod)
    x, idx, w = case["x"].to(DEV), case["idx"].to(DEV), case["w"].to(DEV)
    with torch.no_grad():
        first = mod(x, idx, w)
        for _ in range(25):
            assert torch.equal(first, mod(x, idx, w))


def test_training_falls_back_and_backprops(e4b):
    case = C.build("small")
    mod = _module_from_case(e4b, case)
    e4b.enable_fast(mod)
    x = case["x"].to(DEV).clone().requires_grad_(True)
    out = mod(x, case["idx"].to(DEV), case["w"].to(DEV))
    out.float().sum().backward()
    assert x.grad is not None and torch.isfinite(x.grad).all()


def test_lora_train_mode_falls_back_bit_exact(e4b):
    case = C.build("lora_multi")
    lm = _module_from_case(e4b, case)
    x, idx, w = case["x"].to(DEV), case["idx"].to(DEV), case["w"].to(DEV)
    lm.train()
    with torch.no_grad():
        ref = lm(x, idx, w)
    assert e4b.enable_fast(lm) == 1
    with torch.no_grad():
        got = lm(x, idx, w)
    assert torch.equal(got, ref)


def test_skips_ineligible_blocksize(e4b):
    mod = _module_from_case(e4b, C.build("small"))
    mod.blocksize = 128
    assert e4b.enable_fast(mod) == 0


def test_empty_tokens_and_cold_experts(e4b):
    case = C.build("uneven")
    mod = _module_from_case(e4b, case)
    e4b.enable_fast(mod)
    with torch.no_grad():
        out = mod(case["x"][:0].to(DEV), case["idx"][:0].to(DEV), case["w"][:0].to(DEV))
    assert out.shape == (0, case["st"]["H"])


def test_out_of_range_expert_is_reported_not_faulted(e4b):
    case = C.build("small")
    mod = _module_from_case(e4b, case)
    st = case["st"]
    idx = case["idx"].clone()
    idx[2, 1] = st["E"] + 5
    with pytest.raises(RuntimeError, match="expert index"):
        e4b.ops.moe_forward(case["x"].to(DEV), idx.to(DEV), case["w"].to(DEV), mod.gate_up_proj, mod.gate_up_absmax,
                            mod.down_proj, mod.down_absmax, st["E"], st["I"], check_errors=True)
    # the context is still usable
    e4b.ops.moe_forward(case["x"].to(DEV), case["idx"].to(DEV), case["w"].to(DEV), mod.gate_up_proj,
                        mod.gate_up_absmax, mod.down_proj, mod.down_absmax, st["E"], st["I"], check_errors=True)


def test_fp16_compute_and_fp32_io(e4b):
    case = C.build("small")
    st = case["st"]
    m = e4b.Experts4bit(st["E"], st["H"], st["I"], compute_dtype=torch.float16, device=DEV)
    with torch.no_grad():
        for n in ("gate_up_proj", "down_proj", "gate_up_absmax", "down_absmax"):
            getattr(m, n).copy_(st[n.replace("_proj", "_packed")] if n.endswith("proj") else st[n])
    e4b.enable_fast(m)
    x = case["x"].float().to(DEV)
    with torch.no_grad():
        got = m(x, case["idx"].to(DEV), case["w"].to(DEV))
    assert got.dtype == torch.float32
    anchor = torch.from_numpy(_gold("small")["fp32_oracle"])
    mx, mean = M.rel_errors(got.cpu(), anchor)
    assert mx <= MAX_REL and mean <= MEAN_REL


def test_cuda_graph_capture_of_fused_layer(e4b):
    case = C.build("olmoe_like")
    mod = _module_from_case(e4b, case)
    e4b.enable_fast(mod)
    x, idx, w = case["x"].to(DEV), case["idx"].to(DEV), case["w"].to(DEV)
    with torch.no_grad():
        eager = mod(x, idx, w)
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            mod(x, idx, w)
        torch.cuda.current_stream().wait_stream(s)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph):
            out = mod(x, idx, w)
        graph.replay()
        torch.cuda.synchronize()
    assert torch.equal(out, eager)


def test_compat_gemm_4bit_grouped_drives_reference_shape(e4b):
    import importlib
    import sys
    sys.path.insert(0, os.path.join(os.path.dirname(os.path.dirname(__file__)), "experts4bit-qlora_b200", "compat"))
    nf4_grouped = importlib.import_module("nf4_grouped")
    case = C.build("small")
    st = case["st"]
    E, H, I = st["E"], st["H"], st["I"]
    order, tok, pos, counts, off = M.permute(case["idx"], E)
    active = torch.nonzero(counts).view(-1)
    a = case["x"][tok].contiguous().to(DEV)
    up = nf4_grouped.gemm_4bit_grouped(a, st["gate_up_packed"].view(E, 2 * I, H // 2).to(DEV),
                                       st["gate_up_absmax"].view(E, 2 * I, H // 64).to(DEV),
                                       counts[active].tolist(), active.tolist())
    Wf = M.dequant_stack_f32(st["gate_up_packed"], st["gate_up_absmax"], (2 * I, H))
    ref = torch.cat([a[int(off[e]):int(off[e + 1])].cpu().float() @ Wf[e].t() for e in range(E)])
    mx, mean = M.rel_errors(up.cpu(), ref)
    assert mx <= MAX_REL and mean <= MEAN_REL


_PAIR_SCRIPT = r"""
import importlib, sys, torch
sys.path.insert(0, sys.argv[1])
e4b = importlib.import_module("experts4bit-qlora_b200")
E, H, I, k, T, r = 128, 2048, 768, 8, 700, 16
g = torch.Generator(device="cuda").manual_seed(11)
base = e4b.Experts4bit.from_float((torch.randn(E, 2 * I, H, generator=g, device="cuda") * 0.02).to(torch.bfloat16),
                                  (torch.randn(E, H, I, generator=g, device="cuda") * 0.02).to(torch.bfloat16))
lm = e4b.ExpertsLoRA(base, r=r, alpha=16, dtype=torch.bfloat16).to("cuda").eval()
with torch.no_grad():
    for p in (lm.gate_up_lora_A, lm.gate_up_lora_B, lm.down_lora_A, lm.down_lora_B):
        p.copy_(torch.randn(p.shape, generator=g, device="cuda") * 0.01)
x = torch.randn(T, H, generator=g, device="cuda").to(torch.bfloat16)
w, idx = torch.topk(torch.softmax(torch.randn(T, E, generator=g, device="cuda"), -1), k)
assert e4b.enable_fast(lm) == 1
with torch.no_grad():
    out = lm(x, idx, w)
torch.save(out.cpu(), sys.argv[2])
"""


def test_cta_pair_tensor_core_path_matches_single_cta(tmp_path):
    """E4B_UMMA_PAIR=1 runs the NF4 tensor-core GEMMs (gate_up with SwiGLU and the LoRA step,
    down with 256 features per tile) as clusters of two CTAs with tcgen05.mma.cta_group::2. Same
    decoded operands and K order as the one-CTA kernel; the layer outputs agree to the layer bar
    against each other (the one-CTA path is anchored to fp32 by the tests above)."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "pair.py"
    script.write_text(_PAIR_SCRIPT)
    outs = []
    for pair in ("0", "1"):
        path = tmp_path / f"out{pair}.pt"
        env = dict(os.environ, E4B_UMMA_PAIR=pair)
        res = subprocess.run([sys.executable, str(script), root, str(path)], env=env, capture_output=True, text=True,
                             timeout=600)
        assert res.returncode == 0, res.stderr[-2000:]
        outs.append(torch.load(path).float())
    mx, mean = M.rel_errors(outs[1], outs[0])
    assert mx <= 1e-3 and mean <= 1e-4, (mx, mean)


def test_pipelined_lora_a_prepass_is_bit_identical(tmp_path):
    """The LoRA-A pre-pass for ranks <= 16 double-buffers its K chunks (cp.async rows, vector
    adapter loads); the tensor-core fragments and their K order are those of the one-buffer
    kernel (E4B_LORA_A_PIPE=0), so the layer output is identical bit for bit."""
    import os
    import subprocess
    import sys
    root = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    script = tmp_path / "lora_a.py"
    script.write_text(_PAIR_SCRIPT)
    outs = []
    for pipe in ("0", "1"):
        path = tmp_path / f"out{pipe}.pt"
        env = dict(os.environ, E4B_LORA_A_PIPE=pipe)
        res = subprocess.run([sys.executable, str(script), root, str(path)], env=env, capture_output=True, text=True,
                             timeout=600)
        assert res.returncode == 0, res.stderr[-2000:]
        outs.append(torch.load(path))
    assert torch.equal(outs[0], outs[1])
