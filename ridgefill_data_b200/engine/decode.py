"""Greedy decode over filled caches (code/kva/kva.py:497-522): every decode step runs the full model
exactly (SwiftKV native: its own late-layer path)."""
from __future__ import annotations

import torch

from .scoring import check_finite


@torch.no_grad()
def step(model, tok, position, cache, arm):
    """One exact decode step: token `tok` at `position` through every layer over `cache` (appended in place).
    Returns the next-token logits [1, V] fp32."""
    dev = model.device
    pos = torch.tensor([position], device=dev)
    h = model.embed(torch.tensor([tok], device=dev))
    swift_from = arm.split if arm is not None and arm.fill == "swiftkv_native" else model.n_layers
    for i in range(swift_from):
        h = model.layer(i, h, pos, cache)
    boundary = h
    for i in range(swift_from, model.n_layers):      # SwiftKV's own late layers read the boundary state
        model.swift_fill(i, boundary, pos, cache)
        h = model.swift_layer(i, h, pos, cache)
    return model.logits(h)


@torch.no_grad()
def greedy(model, ids, cache, first_logits, steps, arm, eos=()):
    """Greedy continuation of up to `steps` tokens, stopping after an EOS. Returns (tokens, 'stop' | 'length')."""
    made = []
    start = ids.shape[0]
    nxt = int(check_finite(first_logits[-1], f"{arm.name} first token").argmax())
    while len(made) < steps:
        made.append(nxt)
        if nxt in eos:
            return made, "stop"
        if len(made) == steps:
            break
        logits = step(model, nxt, start + len(made) - 1, cache, arm)
        nxt = int(check_finite(logits[-1], f"{arm.name} decode step {len(made)}").argmax())
    return made, "length"


def fork_cache(cache):
    """A per-arm fork of a cache: per-layer dict copies sharing K/V buffers (rows below every fork's length
    are never rewritten) and cloned recurrent states."""
    forks = []
    for entry in cache:
        fork = dict(entry)
        fork.update({k: fork[k].clone() for k in ("rec", "conv") if fork.get(k) is not None})
        forks.append(fork)
    return forks
