"""Greedy decode over filled caches (code/kva/kva.py:497-522): every decode step runs the full model
exactly (SwiftKV native: its own late-layer path). On the B200 model a run of GRAPH_MIN_STEPS or more tokens replays
one CUDA graph of the device-position decode step (engine/decode_graph.py) instead of eager steps: the same kernels
and arithmetic, without the per-step host launches (RF_DECODE_GRAPH=0 keeps the eager steps)."""
from __future__ import annotations

import os

import torch

from .scoring import check_finite

GRAPH_MIN_STEPS = 16


def _graph_for(model, cache, steps, arm):
    """A decode graph for one sequence when the model and arm allow one, else None. The cache's recurrent states
    are replaced by copies first: the graph updates them in place, and other holders of the old tensors (a fork's
    parent, a snapshot) must not see that."""
    if (os.environ.get("RF_DECODE_GRAPH") == "0" or steps < GRAPH_MIN_STEPS or model.device.type != "cuda"
            or not hasattr(model, "decode_step_dev") or getattr(model, "tp", None) is not None
            or getattr(model.cfg, "moe", False) or (arm is not None and arm.fill == "swiftkv_native")):
        return None
    from .decode_graph import DecodeGraph
    for entry in cache:
        for k in ("rec", "conv"):
            if entry.get(k) is not None:
                entry[k] = entry[k].clone()
    try:
        return DecodeGraph(model, [cache], headroom=steps)
    except NotImplementedError:
        return None


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
    dg = _graph_for(model, cache, steps, arm)
    while len(made) < steps:
        made.append(nxt)
        if nxt in eos:
            return made, "stop"
        if len(made) == steps:
            break
        logits = dg.step([nxt]) if dg is not None else step(model, nxt, start + len(made) - 1, cache, arm)
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
