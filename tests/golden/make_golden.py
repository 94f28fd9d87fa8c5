"""Regenerate the golden fixtures by running the REFERENCE's own Python on CPU.

Run in the build container only (it imports experts4bit-qlora from its source
tree, which does not exist on the GPU box):

    python tests/golden/make_golden.py [/path/to/experts4bit-qlora]

bitsandbytes and grouped-nf4-gemm are not installed there, so two stand-ins are
put on the import path: ``oracle/bnb_shim`` (the oracle's NF4 codec behind
bitsandbytes' function names) and an in-process ``nf4_grouped`` whose
``gemm_4bit_grouped`` is a per-segment fp32 dequant-matmul, so the reference's
own ``engines/fast.py`` driver (permutation, LoRA-on-sorted-rows, combine) runs
unmodified. Everything else -- ``ExpertsNbit.forward``, ``ExpertsLoRA.forward``
and ``_forward_decode``, ``cpu_router.deterministic_topk`` / ``route_on_host``
-- is the reference's code as shipped.
"""
from __future__ import annotations

import os
import sys
import types

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))


def _bf16_u16(t):
    return t.detach().contiguous().to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def main(ref_root: str) -> None:
    sys.path[:0] = [os.path.join(REPO, "oracle", "bnb_shim"), REPO, ref_root, HERE]
    import cases as C
    from oracle.nf4 import dequantize_nf4_f32

    calls = []

    def gemm_4bit_grouped(a, packed, absmax, sizes, expert_ids):
        calls.append((list(sizes), list(expert_ids)))
        E, N, Kh = packed.shape
        out = torch.empty(a.shape[0], N, dtype=a.dtype)
        off = 0
        for n, e in zip(sizes, expert_ids):
            w = torch.from_numpy(dequantize_nf4_f32(packed[e].reshape(-1).numpy(),
                                                    absmax[e].reshape(-1).numpy())).reshape(N, Kh * 2)
            out[off:off + n] = (a[off:off + n].float() @ w.t()).to(a.dtype)
            off += n
        return out

    sys.modules["nf4_grouped"] = types.SimpleNamespace(gemm_4bit_grouped=gemm_4bit_grouped)

    from experts4bit_qlora import Experts4bit, ExpertsLoRA
    from experts4bit_qlora.engines import cpu_router as cr
    from experts4bit_qlora.engines import fast

    for name in C.CASES:
        case = C.build(name)
        st = case["st"]
        mod = Experts4bit.from_float(case["gate_up_f"], case["down_f"], compute_dtype=torch.bfloat16,
                                     has_gate=st["has_gate"])
        # the reference quantized through the shim: its bytes must be the case's bytes
        assert torch.equal(mod.gate_up_proj.data, st["gate_up_packed"]), name
        assert torch.equal(mod.down_absmax, st["down_absmax"]), name
        x, idx, w = case["x"], case["idx"], case["w"]
        out = {}
        if case["lora"] is None:
            target = mod
            fused = fast.fused_experts_forward
        else:
            L = case["lora"]
            target = ExpertsLoRA(mod, r=L["r"], alpha=L["alpha"], dtype=L["gate_up_A"].dtype)
            with torch.no_grad():
                for k in ("gate_up_A", "gate_up_B", "down_A", "down_B"):
                    getattr(target, k.replace("_A", "_lora_A").replace("_B", "_lora_B")).copy_(L[k])
            target.eval()
            fused = fast.fused_experts_lora_forward
        with torch.no_grad():
            out["ref_loop"] = _bf16_u16(target(x, idx, w))
            calls.clear()
            target._e4b_fast_ref = target.forward
            out["ref_fused_driver"] = _bf16_u16(fused(target, x, idx, w))
            sizes, eids = calls[0]
            out["sizes"] = np.array(sizes, dtype=np.int64)
            out["expert_ids"] = np.array(eids, dtype=np.int64)
            # fp32 anchor (tests/test_fast.py:49-68) computed with the reference's own dequant
            xf = x.float()
            o32 = torch.zeros(x.shape[0], st["H"])
            for e in range(st["E"]):
                wgu = mod._dequantize_expert(mod.gate_up_proj, mod.gate_up_absmax, mod._gate_up_shape, e, torch.float32)
                wdn = mod._dequantize_expert(mod.down_proj, mod.down_absmax, mod._down_shape, e, torch.float32)
                tok, pos = torch.where(idx == e)
                if not len(tok):
                    continue
                h = xf[tok] @ wgu.t()
                if case["lora"] is not None:
                    L = case["lora"]
                    h = h + L["scaling"] * ((xf[tok] @ L["gate_up_A"][e].float().t()) @ L["gate_up_B"][e].float().t())
                if mod.has_gate:
                    g, u = h.chunk(2, -1)
                    h = mod.act_fn(g) * u
                else:
                    h = mod.act_fn(h)
                d = h @ wdn.t()
                if case["lora"] is not None:
                    d = d + L["scaling"] * ((h @ L["down_A"][e].float().t()) @ L["down_B"][e].float().t())
                o32.index_add_(0, tok, d * w[tok, pos, None].float())
            out["fp32_oracle"] = o32.numpy()
            for e in (0, st["E"] - 1):
                out[f"dequant_gu_e{e}"] = _bf16_u16(mod._dequantize_expert(
                    mod.gate_up_proj, mod.gate_up_absmax, mod._gate_up_shape, e, torch.bfloat16))
                out[f"dequant_dn_e{e}"] = _bf16_u16(mod._dequantize_expert(
                    mod.down_proj, mod.down_absmax, mod._down_shape, e, torch.bfloat16))
        if case["router_w"] is not None:
            logits = x.float() @ case["router_w"].float().t()
            rw, ri = cr.route_on_host(logits, case["k"], cr._SOFTMAX_THEN_TOPK, False)
            out["route_w"] = rw.numpy()
            out["route_idx"] = ri.numpy()
        for k, v in C.input_digests(case).items():
            out[k] = np.array(v)
        np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
        print(name, {k: v.shape for k, v in out.items() if not k.startswith("sha_")})

    # router rule: the reference's tie known-answer plus seeded logits with injected ties
    g = torch.Generator().manual_seed(21)
    logits = torch.randn(64, 64, generator=g)
    logits[::3, 5] = logits[::3, 9]                     # exact ties between experts 5 and 9
    logits[1::7, :] = torch.round(logits[1::7, :])       # many-way ties
    tie = torch.tensor([[1.0, 3.0, 3.0, 0.5, 3.0, 2.0]])
    out = {"logits": logits.numpy(), "tie_logits": tie.numpy()}
    for k in (1, 2, 8):
        v, i = cr.deterministic_topk(logits, k)
        out[f"topk{k}_vals"], out[f"topk{k}_idx"] = v.numpy(), i.numpy()
        for kind in (cr._SOFTMAX_THEN_TOPK, cr._TOPK_THEN_SOFTMAX):
            for norm in (False, True):
                rw, ri = cr.route_on_host(logits, k, kind, norm)
                out[f"route_{kind}_{int(norm)}_k{k}_w"] = rw.numpy()
                out[f"route_{kind}_{int(norm)}_k{k}_idx"] = ri.numpy()
    v, i = cr.deterministic_topk(tie, 3)
    out["tie_idx"], out["tie_vals"] = i.numpy(), v.numpy()
    np.savez_compressed(os.path.join(HERE, "router.npz"), **out)
    print("router", len(out))


if __name__ == "__main__":
    main(sys.argv[1] if len(sys.argv) > 1 else os.environ.get("E4B_REFERENCE_ROOT", "../reference"))
