"""GPU: the drop-in inside its caller, a transformers OLMoE model.

A small random-init ``OlmoeForCausalLM`` (transformers' own modelling code) gets
its ``mlp.experts`` replaced by ``Experts4bit.from_float`` of the same weights, as
the reference's loader does (loader.py:699-718), and ``enable_fast`` patches them.
Checked: the MoE block's output against the HF block on the dequantized weights
(fp32 anchor bars), the patched model's logits against the unpatched loop, and a
CUDA-graph-captured greedy decode that replays the eager token stream
(``probe_capture``, engines/capture.py:177-222).
"""
from __future__ import annotations

import importlib

import pytest
import torch

from oracle import moe as M

pytestmark = pytest.mark.gpu
DEV = "cuda"


def _tiny_olmoe(e4b, layers=2, seed=0):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.OlmoeConfig(vocab_size=1024, hidden_size=512, intermediate_size=256, num_hidden_layers=layers,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=16,
                                   num_experts_per_tok=4, max_position_embeddings=256, norm_topk_prob=False)
    torch.manual_seed(seed)
    model = transformers.OlmoeForCausalLM(cfg).to(DEV, dtype=torch.bfloat16).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            layer.mlp.gate.weight.normal_(0, 0.05)
            ex = layer.mlp.experts
            ex.gate_up_proj.normal_(0, 0.02)
            ex.down_proj.normal_(0, 0.02)
    return model, cfg


def _swap_experts(e4b, model):
    for layer in model.model.layers:
        ex = layer.mlp.experts
        layer.mlp.experts = e4b.Experts4bit.from_float(ex.gate_up_proj.data, ex.down_proj.data).eval()


def test_moe_block_with_drop_in_experts(e4b):
    model, cfg = _tiny_olmoe(e4b)
    block = model.model.layers[0].mlp
    hf_experts = block.experts
    _swap_experts(e4b, model)
    ours = block.experts
    assert e4b.enable_fast(model) == cfg.num_hidden_layers
    # HF's own experts, in fp32, on the fp32 dequantized NF4 values: the function the fused layer
    # computes, evaluated without intermediate roundings
    hf32 = hf_experts.float()
    with torch.no_grad():
        for e in range(cfg.num_experts):
            hf32.gate_up_proj[e].copy_(ours._dequantize_expert(ours.gate_up_proj, ours.gate_up_absmax,
                                                               ours._gate_up_shape, e, torch.float32))
            hf32.down_proj[e].copy_(ours._dequantize_expert(ours.down_proj, ours.down_absmax, ours._down_shape,
                                                            e, torch.float32))
    for T in (1, 5, 200):
        h = torch.randn(1, T, cfg.hidden_size, device=DEV).to(torch.bfloat16)
        with torch.no_grad():
            got = block(h)
            flat = h.view(-1, cfg.hidden_size)
            _, w, idx = block.gate(flat)
            prev = torch.backends.cuda.matmul.allow_tf32
            torch.backends.cuda.matmul.allow_tf32 = False
            anchor = hf32(flat.float(), idx, w.float())
            torch.backends.cuda.matmul.allow_tf32 = prev
        mx, mean = M.rel_errors(got.view(-1, cfg.hidden_size).float(), anchor)
        assert mx <= 1e-2 and mean <= 2e-3, (T, mx, mean)


def test_patched_model_logits_follow_the_reference_loop(e4b):
    model, cfg = _tiny_olmoe(e4b, seed=1)
    _swap_experts(e4b, model)
    ids = torch.randint(0, cfg.vocab_size, (1, 24), device=DEV)
    with torch.no_grad():
        ref = model(input_ids=ids).logits.float()
        assert e4b.enable_fast(model) == cfg.num_hidden_layers
        got = model(input_ids=ids).logits.float()
        assert e4b.disable_fast(model) == cfg.num_hidden_layers
        again = model(input_ids=ids).logits.float()
    assert torch.equal(ref, again)
    mx, mean = M.rel_errors(got, ref)
    assert mx <= 3e-2 and mean <= 5e-3, (mx, mean)


def test_probe_capture_replays_the_eager_stream(e4b):
    capture = importlib.import_module("experts4bit-qlora_b200.capture")
    model, cfg = _tiny_olmoe(e4b, seed=2)
    _swap_experts(e4b, model)
    e4b.enable_fast(model)
    ids = torch.randint(0, cfg.vocab_size, (1, 12), device=DEV)
    rep = capture.probe_capture(model, ids, max_new_tokens=12)
    assert rep["captured"], rep["error"]
    if not rep["matches_eager"]:  # a photo finish is allowed only when replay equals eager bit for bit
        assert rep["teacher_forced"]["max_abs_delta"] == 0.0, rep
    dec, first = capture.capture_decode(model, ids, max_length=ids.shape[-1] + 10)
    toks = [int(first)]
    for _ in range(5):
        toks.append(int(dec.step(torch.tensor([[toks[-1]]], device=DEV))))
    again = dec.reset(ids)
    assert int(again) == toks[0]
