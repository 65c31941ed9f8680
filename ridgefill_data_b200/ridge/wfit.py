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
    first_rank = counts.cumsum(0) - counts                 # 0-based rank of each distinct value's first copy
    shared = first_rank + (counts - 1) / 2
    return shared.double()[inverse] / x.numel()


_SHAPE_FNS = {
    "qfp": lambda q: q,
    "sqrt": lambda q: q.clamp_min(0).sqrt(),
    "rank": lambda q: (1 - rank_fraction(q)).clamp_min(RANK_FLOOR).reciprocal(),
}


def row_weights(qfp, shape):
    """Fit weights [n] fp64 of one document's rows from their qfp [n]: the shape of rows 1.. scaled to mean 1,
    and weight 1 for row 0."""
    if shape not in _SHAPE_FNS:
        raise ValueError(f"unknown weight shape {shape!r} (one of {SHAPES})")
    q = qfp.double().cpu()
    shaped = _SHAPE_FNS[shape](q[1:])
    weights = torch.ones_like(q)
    if shaped.numel() > 0:
        mean = shaped.mean()
        if mean > 0:
            weights[1:] = shaped / mean
    return weights


class _QfpTap:
    """A forward hook that sums, over the attention layers below the split, the mass each row receives from
    later rows; from the split on it hands each late layer's input rows to `late` with the finished qfp."""

    def __init__(self, model, n, split, stride, late):
        self.model, self.n, self.split, self.stride, self.late = model, n, split, stride, late
        self.pos = torch.arange(n, device=model.device)
        self.received = torch.zeros(n, dtype=torch.float64)
        self.qfp = None

    def __call__(self, i, h):
        if i == "final":
            return
        m = self.model
        if i < self.split:
            if m.layer_types[i] == "attn":
                x = m.in_norm(h, m.W[i]["ln1"])
                keys, _ = IM.attn_kv(m, i, x, self.pos)
                self.received.add_(IM.received_mass(m.queries(i, x, self.pos), keys, m.scale, stride=self.stride))
            return
        if self.qfp is None:
            self.qfp = per_later_token(self.received, self.n)
        self.late(i, h, self.qfp)


@torch.no_grad()
def doc_pass(model, ids, split, stride, late):
    """One exact forward of a document. By layer `split` its qfp [n] (host fp64) is complete; late(i, h, qfp)
    then sees the input rows h of every late layer i >= split."""
    model.forward_exact(ids.to(model.device), hook=_QfpTap(model, ids.shape[0], split, stride, late))


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
