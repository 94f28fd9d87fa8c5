"""GPU: each stage of the fused path against the CPU oracle, through the C ABI.

Integer/byte/index stages (quantize, dequantize, top-k indices, permutation)
must be bit-exact; floating-point stages carry their tolerance in the test.
"""
import numpy as np
import pytest
import torch

import cases as C
from oracle import moe as M
from oracle import nf4 as N

pytestmark = pytest.mark.gpu
DEV = torch.device("cuda:0")


@pytest.fixture(scope="module")
def ops(e4b):
    assert e4b._native.available(), "libe4b.so must be built (no fallback)"
    return e4b.ops


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32, torch.float16])
@pytest.mark.parametrize("n", [64, 64 * 1000, 2048 * 2048])
def test_dequantize_bit_exact(ops, dtype, n):
    g = torch.Generator().manual_seed(n)
    packed = torch.randint(0, 256, (n // 2,), dtype=torch.uint8, generator=g)
    absmax = torch.rand(n // 64, generator=g) * 3
    absmax[::7] = 0.0
    got = ops.nf4_dequantize(packed.to(DEV), absmax.to(DEV), (n,), dtype).cpu()
    ref = torch.from_numpy(N.dequantize_nf4_f32(packed.numpy(), absmax.numpy())).to(dtype)
    assert torch.equal(got.view(torch.uint8), ref.view(torch.uint8))


@pytest.mark.parametrize("dtype", [torch.bfloat16, torch.float32])
def test_quantize_bit_exact_device_and_host(ops, dtype):
    g = torch.Generator().manual_seed(1)
    w = (torch.randn(96, 640, generator=g) * 0.02).to(dtype)
    w[3, :64] = 0.0                                   # an all-zero block
    t = N.nf4_thresholds()
    w[5, :64] = torch.from_numpy(np.r_[t, np.ones(64 - 15, np.float32)]).to(dtype)  # values on midpoints
    p_ref, a_ref = N.quantize_nf4(w)
    p_dev, a_dev = ops.nf4_quantize(w.to(DEV))
    p_host, a_host = ops.nf4_quantize(w)
    assert np.array_equal(p_dev.cpu().numpy(), p_ref) and np.array_equal(a_dev.cpu().numpy(), a_ref)
    assert np.array_equal(p_host.numpy(), p_ref) and np.array_equal(a_host.numpy(), a_ref)


@pytest.mark.parametrize("name", ["small", "olmoe_like", "ragged"])
def test_dequantize_matches_reference_golden(ops, name):
    import os
    g = dict(np.load(os.path.join(os.path.dirname(__file__), "golden", f"{name}.npz")))
    case = C.build(name)
    st = case["st"]
    e = st["E"] - 1
    got = ops.nf4_dequantize(st["gate_up_packed"][e].to(DEV), st["gate_up_absmax"][e].to(DEV),
                             (2 * st["I"], st["H"]), torch.bfloat16).cpu()
    assert np.array_equal(got.view(torch.int16).numpy().view(np.uint16), g[f"dequant_gu_e{e}"])


@pytest.mark.parametrize("T,E,k,H", [(1, 64, 8, 2048), (37, 128, 8, 2048), (300, 8, 2, 4096), (5, 256, 8, 7168),
                                     (64, 64, 1, 256)])
@pytest.mark.parametrize("kind,norm", [(0, False), (0, True), (1, False)])
def test_router_topk_bit_exact_on_same_logits(ops, T, E, k, H, kind, norm):
    g = torch.Generator().manual_seed(T * 7 + E)
    x = torch.randn(T, H, generator=g).to(torch.bfloat16)
    wr = (torch.randn(E, H, generator=g) * 0.02).to(torch.bfloat16)
    wr[E // 2] = wr[E // 3]                      # exact logit ties between two experts
    w, idx, logits = ops.router_topk(x.to(DEV), wr.to(DEV), k, kind, norm, return_logits=True)
    logits = logits.cpu()
    ref_logits = M.router_logits_f32(x, wr)
    assert torch.allclose(logits, ref_logits, rtol=1e-4, atol=1e-4)
    # bit-exact indices on identical fp32 logits (the tie rule)
    kname = M.SOFTMAX_THEN_TOPK if kind == 0 else M.TOPK_THEN_SOFTMAX
    rw, ridx = M.route_on_host(logits, k, kname, norm)
    assert torch.equal(idx.cpu(), ridx)
    torch.testing.assert_close(w.cpu(), rw, rtol=2e-6, atol=1e-7)


@pytest.mark.parametrize("wdt,xdt", [(torch.float32, torch.float16), (torch.float16, torch.bfloat16),
                                     (torch.float32, torch.bfloat16)])
def test_router_mixed_dtypes_split_k(ops, wdt, xdt):
    """Weights of another type than the activations, on the K-split tensor-core path."""
    T, E, k, H = 100, 16, 4, 1024
    g = torch.Generator().manual_seed(11)
    x = torch.randn(T, H, generator=g).to(xdt)
    wr = (torch.randn(E, H, generator=g) * 0.02).to(wdt)
    w, idx, logits = ops.router_topk(x.to(DEV), wr.to(DEV), k, 0, False, return_logits=True)
    logits = logits.cpu()
    # the kernel rounds the weights to the activation type; the oracle sees the same values
    ref_logits = M.router_logits_f32(x, wr.to(xdt))
    assert torch.allclose(logits, ref_logits, rtol=1e-4, atol=1e-4)
    rw, ridx = M.route_on_host(logits, k, M.SOFTMAX_THEN_TOPK, False)
    assert torch.equal(idx.cpu(), ridx)


def test_router_tie_known_answer(ops):
    """engines/cpu_router.py tie rule: logits [1,3,3,.5,3,2], k=3 -> [1,2,4]."""
    logits = torch.tensor([[1.0, 3.0, 3.0, 0.5, 3.0, 2.0]])
    # x = e_0 (one-hot), W_r[:, 0] = logits -> fp32 logits are exactly the vector
    H = 64
    x = torch.zeros(1, H, dtype=torch.bfloat16)
    x[0, 0] = 1.0
    wr = torch.zeros(6, H, dtype=torch.bfloat16)
    wr[:, 0] = logits[0].to(torch.bfloat16)
    w, idx = ops.router_topk(x.to(DEV), wr.to(DEV), 3)
    assert idx.cpu().tolist() == [[1, 2, 4]]


@pytest.mark.parametrize("T,k,E", [(1, 8, 64), (5, 8, 64), (4096, 8, 128), (8192, 2, 8), (16384, 8, 256),
                                   (33, 4, 16), (0, 2, 4), (3, 3, 1000), (1100, 8, 1000), (2049, 4, 3)])
def test_permute_bit_exact(ops, T, k, E):
    g = torch.Generator().manual_seed(T + E)
    idx = torch.randint(0, E, (T, k), generator=g)
    if T > 4:
        idx[: T // 2] = idx[0]                     # many equal rows -> long equal runs
    order, inv, offsets = ops.permute(idx.to(DEV), E)
    r_order, tok, pos, counts, r_off = M.permute(idx, E)
    assert torch.equal(order.cpu().long(), r_order)
    assert torch.equal(offsets.cpu().long(), r_off)
    inv_ref = torch.empty_like(r_order)
    inv_ref[r_order] = torch.arange(T * k)
    assert torch.equal(inv.cpu().long(), inv_ref)


@pytest.mark.parametrize("E,NN,K,m,epi", [(4, 256, 128, 1, 0), (8, 512, 1024, 3, 1), (3, 128, 2048, 8, 2),
                                           (5, 256, 768, 13, 1), (4, 128, 128, 40, 0), (2, 4096, 1024, 1, 0),
                                           # prefill-sized groups: the tcgen05 kernel
                                           (4, 512, 256, 300, 1), (3, 256, 512, 200, 0), (6, 384, 768, 150, 2)])
def test_grouped_gemm_vs_fp32(ops, E, NN, K, m, epi):
    g = torch.Generator().manual_seed(E * NN + K + m)
    w = torch.randn(E, NN, K, generator=g) * 0.05
    packed, absmax = N.quantize_stack(w)
    counts = torch.randint(0, m + 1, (E,), generator=g)
    counts[0] = m
    R = int(counts.sum())
    a = torch.randn(R, K, generator=g).to(torch.bfloat16)
    offsets = torch.zeros(E + 1, dtype=torch.int32)
    offsets[1:] = torch.cumsum(counts, 0)
    out = ops.grouped_nf4_gemm(a.to(DEV), packed.view(E, NN, K // 2).to(DEV), absmax.view(E, NN, K // 64).to(DEV),
                               offsets.to(DEV), epilogue=epi).cpu().float()
    Wf = M.dequant_stack_f32(packed, absmax, (NN, K))
    ref = torch.empty(R, NN // 2 if epi == 1 else NN)
    for e in range(E):
        lo, hi = int(offsets[e]), int(offsets[e + 1])
        y = a[lo:hi].float() @ Wf[e].t()
        if epi == 1:
            y = torch.nn.functional.silu(y[:, : NN // 2]) * y[:, NN // 2:]
        elif epi == 2:
            y = torch.nn.functional.silu(y)
        ref[lo:hi] = y
    mx, mean = M.rel_errors(out, ref)
    assert mx <= 1e-2 and mean <= 2e-3, (mx, mean)


@pytest.mark.parametrize("T,k,H", [(1, 8, 2048), (7, 2, 4096), (64, 8, 128)])
def test_combine_fixed_order(ops, T, k, H):
    g = torch.Generator().manual_seed(T)
    E = 16
    idx = torch.randint(0, E, (T, k), generator=g)
    order, tok, pos, counts, off = M.permute(idx, E)
    rows = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    w = torch.rand(T, k, generator=g)
    inv = torch.empty(T * k, dtype=torch.int32)
    inv[order] = torch.arange(T * k, dtype=torch.int32)
    got = ops.combine(rows.to(DEV), inv.to(DEV), w.to(DEV), T, k, torch.float32).cpu()
    ref = M.scatter_combine(rows, w[tok, pos], order, T, k, torch.float32)
    torch.testing.assert_close(got, ref, rtol=1e-6, atol=1e-6)


@pytest.mark.parametrize("T,k,H", [(5, 4, 64), (33, 8, 128), (1, 2, 2048)])
def test_combine_bit_exact_against_slot_order_fma(ops, T, k, H):
    """The combine's contract is bit identity, not a tolerance: out[t] = fma(row_k-1, w_k-1, ...
    fma(row_0, w_0, 0)) in fp32, slot by slot (the fixed order of fast.py:260-278). The model
    evaluates each fma as one rounding of the exact product-plus-sum (the product of two fp32
    values is exact in fp64; the sum is rounded once to fp64 and once to fp32, which differs from
    a single rounding only at exact fp32 ties, vanishingly rare on random data)."""
    import numpy as np
    g = torch.Generator().manual_seed(100 + T)
    E = 16
    idx = torch.randint(0, E, (T, k), generator=g)
    order, tok, pos, counts, off = M.permute(idx, E)
    rows = torch.randn(T * k, H, generator=g).to(torch.bfloat16)
    w = torch.rand(T, k, generator=g)
    inv = torch.empty(T * k, dtype=torch.int32)
    inv[order] = torch.arange(T * k, dtype=torch.int32)
    got = ops.combine(rows.to(DEV), inv.to(DEV), w.to(DEV), T, k, torch.float32).cpu().numpy()
    r64 = rows.float().numpy().astype(np.float64)
    w64 = w.numpy().astype(np.float64)
    acc = np.zeros((T, H), dtype=np.float32)
    for s in range(k):
        prod = r64[inv[torch.arange(T) * k + s].long().numpy()] * w64[:, s:s + 1]
        acc = (prod + acc.astype(np.float64)).astype(np.float32)
    assert np.array_equal(got, acc)


@pytest.mark.parametrize("K", [128, 768, 2048])
def test_gemv_matches_fp16_code_model_to_one_ulp(ops, K):
    """The decode GEMV computes sum_b absmax_b * sum_i fp16(code_i) * fp16(x_i) with fp32 tensor-core
    accumulation; check it against that model (evaluated in fp64) to within one bf16 ulp of the
    output plus an accumulation floor of 2^-16 of the row's scale (tensor-core fp32 sums are not
    round-to-nearest, which shows on outputs near zero)."""
    E, NN, m = 2, 256, 5
    g = torch.Generator().manual_seed(K)
    w = torch.randn(E, NN, K, generator=g) * 0.05
    packed, absmax = N.quantize_stack(w)
    a = torch.randn(E * m, K, generator=g).to(torch.bfloat16)
    offsets = torch.tensor([0, m, 2 * m], dtype=torch.int32)
    out = ops.grouped_nf4_gemm(a.to(DEV), packed.view(E, NN, K // 2).to(DEV), absmax.view(E, NN, K // 64).to(DEV),
                               offsets.to(DEV)).cpu().double()
    q = torch.from_numpy(N.unpack_nf4(packed.numpy().reshape(-1)).astype(np.int64)).view(E, NN, K)
    c16 = torch.from_numpy(N.NF4_CODE).to(torch.float16).double()
    Wm = (c16[q].view(E, NN, K // 64, 64) * absmax.double().view(E, NN, K // 64, 1)).view(E, NN, K)
    model = torch.cat([a[e * m:(e + 1) * m].double() @ Wm[e].t() for e in range(E)])
    ulp = model.abs().float().to(torch.bfloat16).float().double() * 2.0 ** -7
    floor = 2.0 ** -16 * model.abs().amax(dim=1, keepdim=True)
    assert ((out - model).abs() <= ulp + floor).all()


def test_gemv_rows_beyond_fp16_range_are_scaled_exactly(ops):
    E, NN, K = 1, 128, 256
    g = torch.Generator().manual_seed(5)
    w = torch.randn(E, NN, K, generator=g) * 0.05
    packed, absmax = N.quantize_stack(w)
    a = torch.randn(3, K, generator=g)
    a[1] *= 1e6                                 # far beyond fp16's 65504
    a = a.to(torch.bfloat16)
    offsets = torch.tensor([0, 3], dtype=torch.int32)
    out = ops.grouped_nf4_gemm(a.to(DEV), packed.view(E, NN, K // 2).to(DEV), absmax.view(E, NN, K // 64).to(DEV),
                               offsets.to(DEV)).cpu().float()
    ref = a.float() @ M.dequant_stack_f32(packed, absmax, (NN, K))[0].t()
    for r in range(3):
        mx, mean = M.rel_errors(out[r], ref[r])
        assert mx <= 1e-2 and mean <= 2e-3, (r, mx, mean)


def test_bounded_wait_reports_timeout_and_context_survives(ops):
    """A wait on a copy that never comes runs out after its iteration cap, reports
    E4B_ERR_TIMEOUT through the error word, and the context keeps working."""
    import importlib
    import time
    N = importlib.import_module("experts4bit-qlora_b200._native")
    ws = torch.zeros(1024, dtype=torch.uint8, device=DEV)
    t0 = time.perf_counter()
    N.check(N.lib().e4b_selftest_wait_timeout(ws.data_ptr(), ws.numel(), torch.cuda.current_stream().cuda_stream),
            "e4b_selftest_wait_timeout")
    torch.cuda.synchronize()
    assert time.perf_counter() - t0 < 30.0
    assert ws[4:8].view(torch.int32).item() == 0          # the wait did not complete
    assert N.read_device_error(ws) == N.E4B_ERR_TIMEOUT
    # the context is still usable
    x = torch.randn(64, device=DEV)
    assert torch.isfinite(x.sum()).item()
