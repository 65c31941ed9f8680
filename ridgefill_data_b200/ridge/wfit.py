"""Sensitivity-weighted ridge fit (code/kva/wfit.py:1-70).

The plain fit weights every calibration row equally, but the loss from a fill follows how much later text reads
the row. This fit weights each calibration row by qfp: the attention the row receives from later rows in the
attention layers below the split, per later row (engine.select.per_later_token over engine.impact.received_mass),
with the whole calibration document as the prefix.

Weight shapes, per document over rows >= 1, then scaled to mean 1 over the document:
  qfp   qfp itself
  sqrt  qfp ** 0.5
  rank  1 / max(1 - u, RANK_FLOOR), u = the row's rank fraction by qfp (ties share their mean rank)
Row 0 (the attention sink, whose qfp is orders of magnitude above the rest) gets weight 1.
"""
from __future__ import annotations

import time

import torch

from ..engine import impact as IM
from ..engine.select import per_later_token
from .stats import RidgeStats

SHAPES = ("qfp", "sqrt", "rank")
RANK_FLOOR = 0.1


def rank_fraction(x):
    """Mean rank of each value among x (0-based, ties share their mean rank) divided by len(x)."""
    _, inverse, counts = torch.unique(x, return_inverse=True, return_counts=True)
    mean_rank = counts.cumsum(0) - (counts + 1) / 2
    return mean_rank.double()[inverse] / x.numel()


def row_weights(qfp, shape):
    """Fit weights [n] fp64 of one document's rows from their qfp [n]."""
    q = qfp.double().cpu()
    if shape == "qfp":
        s = q[1:]
    elif shape == "sqrt":
        s = q[1:].clamp_min(0).sqrt()
    elif shape == "rank":
        s = 1 / (1 - rank_fraction(q[1:])).clamp_min(RANK_FLOOR)
    else:
        raise ValueError(f"weight shape {shape!r} not in {SHAPES}")
    w = torch.ones_like(q)
    if s.numel() and s.mean() > 0:
        w[1:] = s / s.mean()
    return w


@torch.no_grad()
def doc_pass(model, ids, split, stride, late):
    """One exact forward of a document. By layer `split` its qfp [n] (fp64 CPU) is complete; late(i, h, qfp)
    then sees every late layer's input rows h (i >= split)."""
    n = ids.shape[0]
    pos = torch.arange(n, device=model.device)
    recv = torch.zeros(n, dtype=torch.float64)
    qfp = []

    def hook(i, h):
        if i == "final":
            return
        if i < split and model.layer_types[i] == "attn":
            x = model.in_norm(h, model.W[i]["ln1"])
            q = model.queries(i, x, pos)
            k, _ = IM.attn_kv(model, i, x, pos)
            recv.add_(IM.received_mass(q, k, model.scale, stride=stride))
        if i >= split:
            if not qfp:
                qfp.append(per_later_token(recv, n))
            late(i, h, qfp[0])
    model.forward_exact(ids.to(model.device), hook=hook)


def capture_weighted(model, docs, split, shape="rank", stride=1, device=None, log=print):
    """RidgeStats for one split with every calibration row weighted by its qfp shape (the fit then runs as for
    the plain statistics: EigenFit / CholeskyFit over the returned state)."""
    L, H = model.n_layers, model.hidden
    st = RidgeStats(split, range(split, L), H, device or model.device)
    t0 = time.time()
    for j, d in enumerate(docs):
        def late(i, h, qfp):
            if i == split:
                st.begin(h, w=row_weights(qfp, shape).float())
            st.add_layer(i, h)
        doc_pass(model, torch.as_tensor(d["ids"]), split, stride, late)
        if log and (j % 10 == 0 or j == len(docs) - 1):
            log(f"weighted capture {j + 1}/{len(docs)} ({time.time() - t0:.0f}s)")
    return st
