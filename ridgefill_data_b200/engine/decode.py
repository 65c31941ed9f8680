"""Greedy decode over filled caches (code/kva/kva.py:497-522): every decode step runs the full model
exactly (SwiftKV native: its own late-layer path)."""
from __future__ import annotations

import torch

from .scoring import check_finite


@torch.no_grad()
def step(model, tok, position, cache, arm):
    """One exact decode step: token `tok` at `position` through every layer over `cache` (appended in place).
    Returns the next-token logits [1, V] fp32."""
    native = arm is not None and arm.fill == "swiftkv_native"
    pos = torch.tensor([position], device=model.device)
    h = model.embed(torch.tensor([tok], device=model.device))
    b = None
    for i in range(model.n_layers):
        if native and i >= arm.split:
            if i == arm.split:
                b = h
            model.swift_fill(i, b, pos, cache)
            h = model.swift_layer(i, h, pos, cache)
        else:
            h = model.layer(i, h, pos, cache)
    return model.logits(h)


@torch.no_grad()
def greedy(model, ids, cache, first_logits, steps, arm, eos=()):
    """Greedy continuation of up to `steps` tokens, stopping after an EOS. Returns (tokens, 'stop' | 'length')."""
    out = []
    tok = int(check_finite(first_logits[-1], f"{arm.name} first token").argmax())
    n = ids.shape[0]
    for t in range(steps):
        out.append(tok)
        if tok in eos:
            return out, "stop"
        if t == steps - 1:
            break
        logits = step(model, tok, n + t, cache, arm)
        tok = int(check_finite(logits[-1], f"{arm.name} decode step {t + 1}").argmax())
    return out, "length"


def fork_cache(cache):
    """A per-arm fork of a cache: per-layer dict copies sharing K/V buffers (rows below every fork's length
    are never rewritten) and cloned recurrent states."""
    out = []
    for c in cache:
        d = dict(c)
        for k in ("rec", "conv"):
            if k in d and d[k] is not None:
                d[k] = d[k].clone()
        out.append(d)
    return out
