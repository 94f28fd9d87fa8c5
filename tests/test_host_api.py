"""CPU: the C-ABI library loads and exports every declared symbol, and the host
side mirrors the reference's module / patch semantics (no GPU compute here)."""
import ctypes
import os
import re

import numpy as np
import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_header_symbols_are_exported(e4b):
    with open(os.path.join(ROOT, "include", "e4b.h")) as f:
        header = f.read()
    declared = set(re.findall(r"E4B_API\s+[\w\s\*]+?\b(e4b_\w+)\s*\(", header))
    assert declared == set(e4b._native.EXPORTED_SYMBOLS)
    lib = ctypes.CDLL(e4b._native.LIB_PATH)
    for name in declared:
        assert hasattr(lib, name), name
    assert e4b._native.lib().e4b_abi_version() == e4b._native.ABI_VERSION == 4


def test_status_strings_and_argument_validation(e4b):
    L = e4b._native.lib()
    assert L.e4b_status_string(0) == b"ok"
    assert b"expert index" in L.e4b_status_string(6)
    # invalid sizes are refused before any device work
    assert L.e4b_nf4_quantize(None, 0, 63, None, None, None) == 1
    assert L.e4b_permute(None, 1, 0, 4, None, None, None, None, 0, None) == 1
    assert L.e4b_grouped_nf4_gemm(None, 0, None, None, None, None, 4, 1, 16, 100, 0, None, None, 0, None) == 2
    assert L.e4b_moe_workspace_bytes(None) == 0


def test_host_codec_matches_oracle(e4b):
    from oracle import nf4 as N
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(32, 256, generator=g) * 0.02).to(torch.bfloat16)
    p, a = e4b.ops.nf4_quantize(w)
    pr, ar = N.quantize_nf4(w)
    assert np.array_equal(p.numpy(), pr) and np.array_equal(a.numpy(), ar)
    d = e4b.ops.nf4_dequantize(p, a, (32, 256), torch.bfloat16)
    assert torch.equal(d, N.dequantize_nf4(pr, ar, (32, 256), torch.bfloat16))


def test_from_float_layout_and_extra_state(e4b):
    m = e4b.Experts4bit.from_float(torch.randn(4, 128, 64), torch.randn(4, 64, 64))
    assert m.gate_up_proj.shape == (4, 128 * 64 // 2) and m.gate_up_proj.dtype == torch.uint8
    assert m.down_absmax.shape == (4, 64 * 64 // 64)
    sd = m.state_dict()
    assert set(sd) == {"gate_up_proj", "down_proj", "gate_up_absmax", "down_absmax", "_extra_state"}
    assert sd["_extra_state"] == {"schema": 1, "quant_type": "nf4", "blocksize": 64, "has_gate": True,
                                  "num_experts": 4, "hidden_dim": 64, "intermediate_dim": 64}
    m2 = e4b.Experts4bit(4, 64, 64)
    m2.load_state_dict(sd)
    assert torch.equal(m2.gate_up_proj, m.gate_up_proj)
    bad = dict(sd)
    bad["_extra_state"] = dict(sd["_extra_state"], num_experts=8)
    with pytest.raises(ValueError, match="mismatch"):
        e4b.Experts4bit(4, 64, 64).load_state_dict(bad)
    legacy = {k: v for k, v in sd.items() if k != "_extra_state"}
    e4b.Experts4bit(4, 64, 64).load_state_dict(legacy)


def test_from_float_validation(e4b):
    with pytest.raises(ValueError, match="transposed"):
        e4b.Experts4bit.from_float(torch.randn(4, 128, 64), torch.randn(4, 64, 128))
    with pytest.raises(ValueError, match="divisible by blocksize"):
        e4b.Experts4bit(4, 100, 64)
    with pytest.raises(ValueError, match="quant_type must be one of"):
        e4b.Experts4bit(4, 64, 64, quant_type="int8")
    assert e4b.normalize_quant_type(" BFloat16 ") == "bf16"


def test_reference_loop_on_cpu_matches_oracle(e4b):
    import cases as C
    from oracle import moe as M
    case = C.build("small")
    st = case["st"]
    m = e4b.Experts4bit(st["E"], st["H"], st["I"], compute_dtype=torch.bfloat16)
    with torch.no_grad():
        m.gate_up_proj.copy_(st["gate_up_packed"])
        m.down_proj.copy_(st["down_packed"])
        m.gate_up_absmax.copy_(st["gate_up_absmax"])
        m.down_absmax.copy_(st["down_absmax"])
    with torch.no_grad():
        got = m(case["x"], case["idx"], case["w"])
    ref = M.reference_forward(st, case["x"], case["idx"], case["w"], torch.bfloat16)
    assert torch.equal(got, ref)


def test_enable_fast_skips_cpu_storage_and_reports_reasons(e4b, capsys):
    m = e4b.Experts4bit.from_float(torch.randn(4, 128, 64), torch.randn(4, 64, 64))
    lm = e4b.ExpertsLoRA(m)
    assert e4b.enable_fast(lm, verbose=True) == 0
    out = capsys.readouterr().out
    assert "storage not on CUDA" in out
    assert e4b.disable_fast(lm) == 0


def test_lora_params_and_init(e4b):
    m = e4b.Experts4bit.from_float(torch.randn(4, 128, 64), torch.randn(4, 64, 64))
    lm = e4b.ExpertsLoRA(m, r=8, alpha=16)
    assert lm.gate_up_lora_A.shape == (4, 8, 64) and lm.gate_up_lora_B.shape == (4, 128, 8)
    assert lm.down_lora_A.shape == (4, 8, 64) and lm.down_lora_B.shape == (4, 64, 8)
    assert lm.scaling == 2.0 and not lm.gate_up_lora_B.any()
    assert not any(p.requires_grad for p in m.parameters())
    with pytest.raises(ValueError):
        e4b.ExpertsLoRA(m, r=0)


def test_fused_path_fails_loudly_without_cuda(e4b):
    x = torch.zeros(1, 64, dtype=torch.bfloat16)
    with pytest.raises(RuntimeError, match="CUDA"):
        e4b.ops.moe_forward(x, torch.zeros(1, 2, dtype=torch.long), torch.ones(1, 2), torch.zeros(4, 10, dtype=torch.uint8),
                            torch.zeros(4, 1), torch.zeros(4, 10, dtype=torch.uint8), torch.zeros(4, 1), 4, 64)
