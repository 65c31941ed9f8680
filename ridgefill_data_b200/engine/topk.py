"""Deterministic block top-k for block-sparse attention selection (code/engine-fix/PATCHES.md: the determinism fix
of the external engine's sparse-attention select).

Per row of block scores [rows, cols] with `visible[r]` live columns: select the k highest visible scores with ties
at the k-th value taken lowest index first, NaN scores never selected, and emit the chosen block indices in
ascending order padded with -1 (so the downstream expansion and its reductions see one canonical order). The
k-th value comes from torch.topk values only (deterministic), and ranks among tied blocks from a cumulative sum,
so the result equals sorting by (score descending, index ascending) and taking the first k, independent of the
top-k kernel's internal order.
"""
from __future__ import annotations

import torch


def block_topk(scores, k, visible=None):
    """(indices [rows, k] int64 ascending, -1 padded; counts [rows]) of the selected blocks."""
    rows, cols = scores.shape
    s = scores.float()
    col = torch.arange(cols, device=s.device)
    live = torch.ones(rows, cols, dtype=torch.bool, device=s.device) if visible is None else \
        col[None, :] < torch.as_tensor(visible, device=s.device)[:, None]
    live &= ~torch.isnan(s)
    masked = torch.where(live, s, torch.full_like(s, -torch.inf))
    n_live = live.sum(1)
    kk = min(k, cols)
    if kk == 0:
        return torch.full((rows, k), -1, dtype=torch.long, device=s.device), torch.zeros(rows, dtype=torch.long,
                                                                                       device=s.device)
    kth = torch.topk(masked, kk, dim=1).values[:, kk - 1:kk]                    # k-th largest live value
    above = live & (masked > kth)
    tied = live & (masked == kth)
    need = (torch.clamp(n_live, max=kk) - above.sum(1))[:, None]              # ties still to take
    take_tied = tied & (tied.long().cumsum(1) <= need)
    chosen = above | take_tied
    counts = chosen.sum(1)
    key = torch.where(chosen, col[None, :].expand(rows, cols), torch.full_like(col[None, :].expand(rows, cols), cols))
    idx = key.sort(dim=1).values[:, :kk]
    idx = torch.where(idx == cols, torch.full_like(idx, -1), idx)
    if kk < k:
        idx = torch.cat((idx, torch.full((rows, k - kk), -1, dtype=idx.dtype, device=idx.device)), 1)
    return idx, counts


def reference_topk(scores, k, visible=None):
    """Plain-Python restatement: sort live, non-NaN columns by (score desc, index asc), keep k, ascending."""
    out = []
    for r, row in enumerate(scores.tolist()):
        n = len(row) if visible is None else int(visible[r])
        cand = [(-v, j) for j, v in enumerate(row[:n]) if v == v]
        pick = sorted(j for _, j in sorted(cand)[:k])
        out.append(pick + [-1] * (k - len(pick)))
    return torch.tensor(out, dtype=torch.long)
