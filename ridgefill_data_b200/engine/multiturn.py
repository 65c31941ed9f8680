"""Carried-cache turns and deferred repair (the semantics of code/kva/multiturn.py:148-255).

A document is prefilled once, possibly with RidgeFill, and its cache is kept for later turns:

* `extend` runs new rows exactly on top of the cache and `decode` generates greedily from it;
* `repair` pays the skipped late-layer work back for the first R cached rows: layers >= split run exactly over
  those rows from their exact split-layer inputs, on a scratch cache, the way a chunked prefill of the rows would;
  attention layers keep the cached K/V of rows >= R, and a GDN layer's state is replaced only when R covers every
  row it has absorbed;
* `repair_selected` recomputes chosen prefix rows through layers >= split with every other row read as filled
  (the computation of finish(exact_rows=...)), and writes those rows' K/V into the cache; GDN states stay.

Repairs swap whole per-layer cache entries and never write into a cached tensor, so forks that share the
cache's storage are left as they were.
"""
from __future__ import annotations

import torch


def _positions(model, start, count):
    return torch.arange(start, start + count, device=model.device)


def extend(model, cache, ids, start, split=None, before=None):
    """Run rows `ids` exactly at positions start, start + 1, ... on top of `cache`.

    before(low), if given, is called as the rows reach layer `split`, with low = {layer < split: that layer's input
    rows}. Returns (logits of the last row, the rows' layer-`split` inputs or None)."""
    ids = torch.as_tensor(ids, device=model.device)
    pos = _positions(model, start, ids.shape[0])
    h = model.embed(ids)
    inputs = {}
    at_split = None
    for i in range(model.n_layers):
        if i == split:
            at_split = h
            if before is not None:
                before(inputs)
        elif split is not None and before is not None and i < split:
            inputs[i] = h
        h = model.layer(i, h, pos, cache)
    return model.logits(h[-1:]), at_split


def decode(model, cache, logits, start, steps, eos=(), split=None):
    """Greedy generation of at most `steps` tokens; each generated token except the last is fed back at positions
    start, start + 1, .... Returns (ids, "stop" on an eos id or "length", the fed rows' layer-`split` inputs
    stacked, or None)."""
    eos = set(eos)
    ids, fed = [], []
    nxt = int(logits[-1].argmax())
    finish = "length"
    for t in range(steps):
        ids.append(nxt)
        if nxt in eos:
            finish = "stop"
            break
        if len(ids) == steps:
            break
        lg, hb = extend(model, cache, [nxt], start + t, split)
        if hb is not None:
            fed.append(hb)
        nxt = int(lg[-1].argmax())
    return ids, finish, (torch.cat(fed) if fed else None)


def cached_rows(cache, layer):
    """Rows held by one layer's cache entry (attention: 'n'; GDN: 'len')."""
    entry = cache[layer]
    return entry["n"] if "n" in entry else entry.get("len", 0)


def repair_rows(r, P, H):
    """Rows a deferred repair of share r covers: every cached row (H) at r >= 1, else round(r * P)."""
    if r >= 1 and P > 0:
        return H
    return round(r * P)


def _fresh_kv(model, k, v):
    entry = {}
    model._append_kv(entry, k, v)
    return entry


def repair(model, cache, hb, split, rows):
    """Exact recomputation of layers >= split over cached rows [0, rows) from their layer-split inputs hb."""
    held = cached_rows(cache, split)
    if rows < 0 or rows > held or rows > hb.shape[0]:
        raise ValueError(f"cannot repair {rows} rows: the cache holds {held}, {hb.shape[0]} split inputs given")
    if not rows:
        return
    scratch = model.new_cache()
    pos = _positions(model, 0, rows)
    h = hb[:rows].to(model.device)
    for i in range(split, model.n_layers):
        h = model.layer(i, h, pos, scratch)
        new, old = scratch[i], cache[i]
        if model.layer_types[i] == "attn":
            k = torch.cat([new["k"], old["k"][:, rows:]], dim=1)
            v = torch.cat([new["v"], old["v"][:, rows:]], dim=1)
            cache[i] = _fresh_kv(model, k, v)
        elif old["len"] == rows:
            cache[i] = {"conv": new["conv"], "rec": new["rec"], "len": rows}
        scratch[i] = {}


def fill_inputs(model, arm, i, b):
    """Layer i's filled inputs of rows whose layer-split inputs are b, under the arm's fill."""
    kind = arm.fill_of(model.layer_types[i])
    if kind == "identity":
        return b
    if kind == "proj":
        return arm.projector(i, b)
    raise ValueError(f"fill {kind!r} has no per-layer inputs to recompute from")


def repair_selected(model, cache, arm, b, rows):
    """Recompute prefix rows `rows` through layers >= arm.split over the filled prefix (b: every prefix row's
    layer-split input) and write their K/V into the cache."""
    if not len(rows):
        return
    sel = torch.as_tensor(rows, dtype=torch.long, device=model.device)
    b = b.to(model.device)
    pos = _positions(model, 0, b.shape[0])
    scratch = model.new_cache()
    cur = b.index_select(0, sel)
    for i in range(arm.split, model.n_layers):
        base = fill_inputs(model, arm, i, b)
        x = base.index_copy(0, sel, cur.to(base.dtype))
        nxt = model.layer_rows(i, x, pos, sel, scratch)
        if model.layer_types[i] == "attn":
            got, old = scratch[i], cache[i]
            k = old["k"].index_copy(1, sel, got["k"].index_select(1, sel))
            v = old["v"].index_copy(1, sel, got["v"].index_select(1, sel))
            cache[i] = _fresh_kv(model, k, v)
        scratch[i] = {}
        cur = nxt
