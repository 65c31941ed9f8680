"""Mixture-of-experts entry points (csrc/moe.cu): router top-k, expert alignment + row gather, the expert-grouped
tcgen05 GEMM (SwiGLU or plain epilogue) and the weighted combine."""
from __future__ import annotations

import torch

from ._ext import ext


def router_topk(logits, E, k, norm=True):
    """logits [n, >= E] fp32 -> (idx [n, k] int32, weights [n, k] fp32): softmax over the first E columns,
    top-k (ties to the lower expert), weights renormalised when norm."""
    n = logits.shape[0]
    idx = torch.empty(n, k, dtype=torch.int32, device=logits.device)
    w = torch.empty(n, k, dtype=torch.float32, device=logits.device)
    ext().router_topk(logits, E, k, idx, w, bool(norm))
    return idx, w


def align(idx, E, x, e0=0):
    """Expert-sorted copy of the rows routed to experts [e0, e0 + E): returns (xp [n k, d], pos [n, k] (-1 for
    slots whose expert is elsewhere), seg_start [E + 1], tile_start [E + 1])."""
    n, k = idx.shape
    dev = x.device
    i32 = dict(dtype=torch.int32, device=dev)
    counts = torch.empty(E, **i32)
    rank = torch.empty(n, k, **i32)
    seg = torch.empty(E + 1, **i32)
    tiles = torch.empty(E + 1, **i32)
    pos = torch.empty(n, k, **i32)
    xp = torch.empty(n * k, x.shape[1], dtype=torch.bfloat16, device=dev)
    ext().moe_align(idx, e0, E, counts, rank, seg, tiles, pos, x, xp)
    return xp, pos, seg, tiles


def grouped(xp, w, seg, tiles, swiglu):
    """Per expert segment: xp_e w_e^T (w [E, N, K]); SwiGLU over gate/up rows interleaved per 128 when swiglu."""
    N = w.shape[1]
    out = torch.empty(xp.shape[0], N // 2 if swiglu else N, dtype=torch.bfloat16, device=xp.device)
    ext().grouped_gemm(xp, w, seg, tiles, out, bool(swiglu), ext().error_word(xp.device.index or 0))
    return out


def combine(h, y, pos, w, ys=None, gate_logit=None, n=None, d=None, out=None):
    """h (or zeros when h is None) + sum_k w y[pos] (+ sigmoid(gate) ys), into `out` when given."""
    if out is None and h is not None:
        out = torch.empty_like(h)
    elif out is None:
        out = torch.empty(n, d, dtype=torch.bfloat16, device=y.device)
    ext().moe_combine(h, y, pos, w, ys, gate_logit, out)
    return out
