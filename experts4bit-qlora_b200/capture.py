"""CUDA-graph capture of a model's decode step, and a probe of whether it replays correctly.

Drop-in for ``experts4bit_qlora.engines.capture`` (capture.py:37-139 ``CapturedDecoder`` /
``capture_decode``, :177-222 ``probe_capture``). The fused expert layers of this package
never synchronise the host (device permutation, device error words, fixed launch shapes),
so a decode step of a model whose experts are patched with ``enable_fast`` captures as
one graph: with a ``StaticCache`` every step has the same shapes, so ONE graph serves a
whole generation and a step is a token copy, a replay and a position bump.

A graph that captured a stale pointer replays without error and returns plausible
tokens, so ``probe_capture`` compares the replayed greedy stream with an incremental
eager decode run by the same rule (raw argmax, fixed length), and on a mismatch
re-runs both teacher-forced to tell a tie from a capture defect.
"""
from __future__ import annotations

import torch


def _static_cache(model, max_length: int, batch: int = 1):
    from transformers import StaticCache
    cfg = model.config.get_text_config() if hasattr(model.config, "get_text_config") else model.config
    return StaticCache(config=cfg, max_batch_size=batch, max_cache_len=max_length, device=model.device,
                       dtype=next(model.parameters()).dtype)


def _forward(model, ids, cache, pos):
    return model(input_ids=ids, past_key_values=cache, cache_position=pos, use_cache=True)


class CapturedDecoder:
    """One captured decode step. The graph reads its inputs by address: a step copies the
    token into ``cur_token``, replays, advances ``cache_position`` and reads ``logits``."""

    def __init__(self, model, cache, cur_token, cache_position, graph, logits):
        self.model, self.cache = model, cache
        self.cur_token, self.cache_position = cur_token, cache_position
        self.graph, self.logits = graph, logits

    def reset(self, input_ids: torch.Tensor) -> torch.Tensor:
        """Re-prefill the prompt and rewind to the post-prompt state; returns the first token.
        Needed between generations: ``step`` only advances the position."""
        self.cache.reset()
        n = input_ids.shape[-1]
        with torch.no_grad():
            out = _forward(self.model, input_ids, self.cache, torch.arange(n, device=input_ids.device))
        nxt = out.logits[:, -1:].argmax(-1)
        self.cur_token.copy_(nxt)
        self.cache_position.fill_(n)
        return nxt

    def _replay(self, token: torch.Tensor) -> None:
        # the position already names the slot this token belongs in: replay first, then advance
        self.cur_token.copy_(token.view(1, 1))
        self.graph.replay()
        self.cache_position += 1

    def logits_for(self, token: torch.Tensor) -> torch.Tensor:
        """Replay on ``token`` and return the step's logits (a copy)."""
        self._replay(token)
        return self.logits[:, -1].clone()

    def step(self, token: torch.Tensor) -> torch.Tensor:
        """Replay on ``token`` and return the greedy next token ``[1, 1]``."""
        self._replay(token)
        return self.logits[:, -1:].argmax(-1)


def capture_decode(model, input_ids, max_length: int, warmup: int = 3):
    """Prefill eagerly, then capture ONE decode step against static buffers. Returns
    ``(CapturedDecoder, first_token)``. A host sync or a data-dependent launch inside the
    step makes the capture raise: such a model is not supported, and this says so."""
    cache = _static_cache(model, max_length)
    n = input_ids.shape[-1]
    pos = torch.arange(n, device=model.device)
    with torch.no_grad():
        first = _forward(model, input_ids, cache, pos).logits[:, -1:].argmax(-1)
    cur_token = first.clone()
    cache_position = torch.tensor([n], device=model.device)
    # settle the allocator and lazy buffers on a side stream before the capture bakes addresses
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s), torch.no_grad():
        for _ in range(warmup):
            _forward(model, cur_token, cache, cache_position)
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph), torch.no_grad():
        captured = _forward(model, cur_token, cache, cache_position)
    # the warm-up and the capture wrote the cache at the first decode slot: re-prefill
    dec = CapturedDecoder(model, cache, cur_token, cache_position, graph, captured.logits)
    return dec, dec.reset(input_ids)


def _eager_greedy(model, input_ids, n_new: int, forced=None):
    """Incremental eager greedy decode against a StaticCache, by the captured path's rule
    (raw argmax, exactly ``n_new`` tokens, no stopping criteria). With ``forced``, feeds
    those tokens instead and returns each step's logits."""
    n = input_ids.shape[-1]
    cache = _static_cache(model, n + n_new + 2)
    toks, logits = [], []
    dev = input_ids.device
    with torch.no_grad():
        nxt = _forward(model, input_ids, cache, torch.arange(n, device=dev)).logits[:, -1:].argmax(-1)
        for j in range(n_new):
            tok = nxt if forced is None else torch.tensor([[forced[j]]], dtype=input_ids.dtype, device=dev)
            toks.append(int(tok))
            if j == n_new - 1:
                break
            out = _forward(model, tok, cache, torch.tensor([n + j], device=dev))
            logits.append(out.logits[0, -1].float())
            nxt = out.logits[:, -1:].argmax(-1)
    return toks, logits


def _teacher_forced_delta(model, dec, input_ids, eager_tokens) -> dict:
    """max |logits_replay - logits_eager| with both fed the same token stream."""
    out = {"max_abs_delta": None, "steps": 0, "note": None}
    try:
        _, ref = _eager_greedy(model, input_ids, len(eager_tokens), forced=eager_tokens)
        dec.reset(input_ids)
        worst, steps = 0.0, 0
        for j, t in enumerate(eager_tokens[:-1]):
            got = dec.logits_for(torch.tensor([[t]], dtype=input_ids.dtype, device=input_ids.device))
            if j < len(ref):
                worst = max(worst, float((got.float()[0] - ref[j]).abs().max()))
                steps += 1
        out["max_abs_delta"], out["steps"] = worst, steps
    except Exception as e:  # reported, not raised: the probe's answer is the report
        out["note"] = f"{type(e).__name__}: {e}"[:140]
    return out


def probe_capture(model, input_ids, max_new_tokens: int = 16) -> dict:
    """Does capture work on this model, and does replay match eager decode?"""
    report = {"captured": False, "matches_eager": None, "n_new": max_new_tokens, "error": None,
              "eager": None, "replayed": None}
    n = input_ids.shape[-1]
    try:
        report["eager"], _ = _eager_greedy(model, input_ids, max_new_tokens)
    except Exception as e:
        report["error"] = f"eager decode failed: {type(e).__name__}: {e}"
        return report
    try:
        dec, first = capture_decode(model, input_ids, max_length=n + max_new_tokens + 2)
        report["captured"] = True
    except Exception as e:
        report["error"] = f"{type(e).__name__}: {str(e)[:200]}"
        return report
    got, tok = [int(first)], first
    for _ in range(max_new_tokens - 1):
        tok = dec.step(tok)
        got.append(int(tok))
    torch.cuda.synchronize()
    report["replayed"] = got
    report["matches_eager"] = got == report["eager"]
    if not report["matches_eager"]:
        tf = _teacher_forced_delta(model, dec, input_ids, report["eager"])
        report["teacher_forced"] = tf
        i = next((j for j in range(min(len(got), len(report["eager"]))) if got[j] != report["eager"][j]), None)
        report["divergence"] = {"index": i,
                                "verdict": ("tie (replay bit-identical to eager under teacher forcing)"
                                            if tf.get("max_abs_delta") == 0.0 and tf.get("steps")
                                            else "undetermined (see teacher_forced)")}
    return report
