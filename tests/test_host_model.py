"""CPU: the drop-in module inside transformers' OLMoE block (the caller the fused path
serves: ``self.experts(hidden, top_k_index, top_k_weights)``, modeling_olmoe.py).

``Experts4bit.from_float`` of the HF experts' weights replaces ``mlp.experts``; its
reference forward (the loop ``enable_fast`` falls back to) must equal HF's own
experts running on the dequantized NF4 values, and the model must run end to end.
"""
from __future__ import annotations

import pytest
import torch


def _tiny(seed=0):
    transformers = pytest.importorskip("transformers")
    cfg = transformers.OlmoeConfig(vocab_size=256, hidden_size=256, intermediate_size=128, num_hidden_layers=2,
                                   num_attention_heads=4, num_key_value_heads=4, num_experts=8, num_experts_per_tok=2,
                                   max_position_embeddings=64)
    torch.manual_seed(seed)
    model = transformers.OlmoeForCausalLM(cfg).to(torch.bfloat16).eval()
    with torch.no_grad():
        for layer in model.model.layers:
            layer.mlp.gate.weight.normal_(0, 0.05)
            layer.mlp.experts.gate_up_proj.normal_(0, 0.02)
            layer.mlp.experts.down_proj.normal_(0, 0.02)
    return model, cfg


def test_reference_loop_inside_the_hf_block(e4b):
    model, cfg = _tiny()
    block = model.model.layers[0].mlp
    hf = block.experts
    ours = e4b.Experts4bit.from_float(hf.gate_up_proj.data, hf.down_proj.data).eval()
    with torch.no_grad():
        for e in range(cfg.num_experts):  # HF's experts on the dequantized NF4 values
            hf.gate_up_proj[e].copy_(ours._dequantize_expert(ours.gate_up_proj, ours.gate_up_absmax,
                                                             ours._gate_up_shape, e, torch.bfloat16))
            hf.down_proj[e].copy_(ours._dequantize_expert(ours.down_proj, ours.down_absmax, ours._down_shape, e,
                                                          torch.bfloat16))
    h = torch.randn(1, 7, cfg.hidden_size).to(torch.bfloat16)
    with torch.no_grad():
        ref = block(h)
        block.experts = ours
        got = block(h)
    assert got.dtype == ref.dtype and got.shape == ref.shape
    d = (got.float() - ref.float()).abs().max() / ref.float().abs().max()
    assert d <= 1e-2, float(d)


def test_model_runs_end_to_end_with_drop_in_experts(e4b):
    model, cfg = _tiny(seed=1)
    for layer in model.model.layers:
        ex = layer.mlp.experts
        layer.mlp.experts = e4b.Experts4bit.from_float(ex.gate_up_proj.data, ex.down_proj.data).eval()
    ids = torch.randint(0, cfg.vocab_size, (1, 9))
    with torch.no_grad():
        out = model(input_ids=ids).logits
    assert out.shape == (1, 9, cfg.vocab_size) and torch.isfinite(out.float()).all()
    sd = model.state_dict()
    assert any(k.endswith("mlp.experts.gate_up_absmax") for k in sd)
