"""CPU: pin the oracle against the published NF4 table and the reference's golden vectors."""
import os

import numpy as np
import pytest
import torch

import cases as C
from oracle import moe as M
from oracle import nf4 as N

GOLD = os.path.join(os.path.dirname(__file__), "golden")


def _load(name):
    return dict(np.load(os.path.join(GOLD, f"{name}.npz")))


def _u16(t):
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def test_codebook_matches_paper_construction():
    v = N.nf4_codebook_from_construction()
    assert np.abs(v - N.NF4_CODE.astype(np.float64)).max() < 2e-7
    assert N.NF4_CODE[7] == 0.0 and N.NF4_CODE[0] == -1.0 and N.NF4_CODE[15] == 1.0
    assert np.all(np.diff(N.NF4_CODE) > 0)


def test_quantize_pack_convention_and_roundtrip():
    # every code at block scale 1: element i of a block gets code i % 16
    w = torch.from_numpy(np.tile(N.NF4_CODE, 4)).reshape(1, 64)
    packed, absmax = N.quantize_nf4(w)
    assert absmax.tolist() == [1.0]
    q = N.unpack_nf4(packed)
    assert q.tolist() == [i % 16 for i in range(64)]
    # first element in the HIGH nibble
    assert packed[0] == (0 << 4) | 1 and packed[7] == (14 << 4) | 15
    back = N.dequantize_nf4_f32(packed, absmax)
    assert np.array_equal(back, np.tile(N.NF4_CODE, 4))


def test_quantize_midpoint_tie_goes_low_and_zero_block():
    t = N.nf4_thresholds()
    w = np.zeros(64, np.float32)
    w[0] = 1.0                    # absmax = 1
    w[1] = t[9]                   # exactly on the midpoint between codes 9 and 10
    w[2] = np.nextafter(t[9], np.float32(2))
    packed, am = N.quantize_nf4(torch.from_numpy(w).reshape(1, 64))
    q = N.unpack_nf4(packed)
    assert q[1] == 9 and q[2] == 10 and q[3] == 7
    p0, a0 = N.quantize_nf4(torch.zeros(1, 64))
    assert a0.tolist() == [0.0] and set(N.unpack_nf4(p0).tolist()) == {7}


@pytest.mark.parametrize("name", C.CASES)
def test_case_inputs_rebuild_identically(name):
    g = _load(name)
    case = C.build(name)
    for k, v in C.input_digests(case).items():
        assert str(g[k]) == v, (name, k)


@pytest.mark.parametrize("name", C.CASES)
def test_oracle_matches_reference_golden(name):
    g = _load(name)
    case = C.build(name)
    st = case["st"]
    # dequant: bit-exact with the reference's _dequantize_expert
    n1 = 2 * st["I"] if st["has_gate"] else st["I"]
    for e in (0, st["E"] - 1):
        gu = M.dequant_expert(st["gate_up_packed"], st["gate_up_absmax"], e, (n1, st["H"]))
        assert np.array_equal(_u16(gu), g[f"dequant_gu_e{e}"])
        dn = M.dequant_expert(st["down_packed"], st["down_absmax"], e, (st["H"], st["I"]))
        assert np.array_equal(_u16(dn), g[f"dequant_dn_e{e}"])
    # permutation: the reference driver's segment table
    order, token_rows, top_pos, counts, offsets = M.permute(case["idx"], st["E"])
    active = torch.nonzero(counts).view(-1)
    assert counts[active].tolist() == g["sizes"].tolist()
    assert active.tolist() == g["expert_ids"].tolist()
    # reference loop and fused driver: bit-exact restatements (same CPU kernels)
    ref = M.reference_forward(st, case["x"], case["idx"], case["w"], torch.bfloat16, case["lora"])
    assert np.array_equal(_u16(ref), g["ref_loop"]) or case["x"].shape[0] == 1
    drv = M.fused_driver_forward(st, case["x"], case["idx"], case["w"], torch.bfloat16, case["lora"])
    assert np.array_equal(_u16(drv), g["ref_fused_driver"])
    o32 = M.fp32_oracle(st, case["x"], case["idx"], case["w"], case["lora"])
    assert np.allclose(o32.numpy(), g["fp32_oracle"], rtol=1e-5, atol=1e-5 * np.abs(g["fp32_oracle"]).max())
    # the reference's bf16 loop is itself within the parity bar of the fp32 anchor
    ref_g = torch.from_numpy(g["ref_loop"].view(np.int16)).view(torch.bfloat16)
    mx, _ = M.rel_errors(ref_g, torch.from_numpy(g["fp32_oracle"]))
    assert mx < 3e-2


def test_decode_branch_is_close_to_loop():
    """The reference's single-token path (lora.py:409-460) sums in routing order; the
    restated mask loop sums in expert order -- equal up to fp32 rounding."""
    g = _load("lora_decode")
    case = C.build("lora_decode")
    ref = M.reference_forward(case["st"], case["x"], case["idx"], case["w"], torch.bfloat16, case["lora"])
    ref_g = torch.from_numpy(g["ref_loop"].view(np.int16)).view(torch.bfloat16)
    assert M.rel_errors(ref, ref_g)[0] < 1e-2


def test_router_known_answer_and_golden():
    g = _load("router")
    v, i = M.deterministic_topk(torch.from_numpy(g["tie_logits"]), 3)
    assert i.tolist() == [[1, 2, 4]] == g["tie_idx"].tolist()
    logits = torch.from_numpy(g["logits"])
    for k in (1, 2, 8):
        v, i = M.deterministic_topk(logits, k)
        assert np.array_equal(i.numpy(), g[f"topk{k}_idx"]) and np.array_equal(v.numpy(), g[f"topk{k}_vals"])
        for kind in (M.SOFTMAX_THEN_TOPK, M.TOPK_THEN_SOFTMAX):
            for norm in (False, True):
                w, i = M.route_on_host(logits, k, kind, norm)
                assert np.array_equal(i.numpy(), g[f"route_{kind}_{int(norm)}_k{k}_idx"])
                assert np.array_equal(w.numpy(), g[f"route_{kind}_{int(norm)}_k{k}_w"])


def test_olmoe_like_routing_golden():
    g = _load("olmoe_like")
    case = C.build("olmoe_like")
    logits = M.router_logits_f32(case["x"], case["router_w"])
    w, i = M.route_on_host(logits, 8)
    assert np.array_equal(i.numpy(), g["route_idx"]) and np.array_equal(w.numpy(), g["route_w"])
    assert np.array_equal(i.numpy(), case["idx"].numpy())


def test_scatter_combine_is_order_fixed():
    torch.manual_seed(0)
    T, k, H = 5, 3, 16
    idx = torch.randint(0, 4, (T, k))
    order, token_rows, top_pos, counts, offsets = M.permute(idx, 4)
    down = torch.randn(T * k, H).to(torch.bfloat16)
    w = torch.rand(T, k)[token_rows, top_pos]
    out = M.scatter_combine(down, w, order, T, k, torch.float32)
    ref = torch.zeros(T, H)
    for r in range(T * k):
        ref[token_rows[r]] += down[r].float() * w[r]
    assert torch.allclose(out, ref, atol=1e-6)


def test_fp8_block_dequant_matches_definition():
    g = torch.Generator().manual_seed(0)
    w = (torch.randn(256, 384, generator=g) * 3).to(torch.float8_e4m3fn)
    s = torch.rand(2, 3, generator=g) + 0.5
    out = M.fp8_block_dequant(w.view(torch.uint8), s, 128, torch.float32)
    assert torch.equal(out[:128, 128:256], w[:128, 128:256].float() * s[0, 1])
