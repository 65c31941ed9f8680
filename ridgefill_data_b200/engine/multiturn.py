"""Multi-turn use of a carried cache and deferred repair (code/kva/multiturn.py:148-255 semantics).

A pasted document is prefilled once (possibly approximately) and cached; later turns extend the cache exactly
(extend), decode greedily (decode), and may pay the skipped late-layer work back:
  repair            layers >= split recomputed exactly over rows [0, R) from their exact layer-split inputs, on a
                    scratch cache, as chunked prefill of those rows would (R = round(r P), every cached row at r = 1)
  repair_selected   chosen prefix rows recomputed through layers >= split by finish(exact_rows=...)'s computation
                    over the other rows as filled; their K/V replace the cached ones (GDN states stay)
Both replace cache list entries only, never a tensor in place, so forks of the cache stay intact.
"""
from __future__ import annotations

import torch


def extend(model, cache, ids, start, split=None, before=None):
    """Exact forward of new rows at positions start, ... on top of cache. before(low): called once the rows
    have passed layers < split with their inputs there. Returns (last-row logits, the rows' split inputs)."""
    ids = torch.as_tensor(ids, device=model.device)
    pos = torch.arange(start, start + ids.shape[0], device=model.device)
    h, hb, low = model.embed(ids), None, {}
    for i in range(model.n_layers):
        if i == split:
            hb = h
            if before is not None:
                before(low)
        if before is not None and split is not None and i < split:
            low[i] = h
        h = model.layer(i, h, pos, cache)
    return model.logits(h[-1:]), hb


def decode(model, cache, logits, start, steps, eos=(), split=None):
    """Greedy decode feeding rows from start. Returns (ids, 'stop' | 'length', fed rows' split inputs)."""
    out, hb = [], []
    tok = int(logits[-1].argmax())
    reason = "length"
    for t in range(steps):
        out.append(tok)
        if tok in eos:
            reason = "stop"
            break
        if t == steps - 1:
            break
        lg, b = extend(model, cache, [tok], start + t, split)
        hb.append(b)
        tok = int(lg[-1].argmax())
    return out, reason, (torch.cat(hb) if hb and split is not None else None)


def cached_rows(cache, layer):
    c = cache[layer]
    return c.get("n", c.get("len", 0))


def repair_rows(r, P, H):
    return H if P > 0 and r >= 1 else round(r * P)


def _put_kv(model, cache, i, k, v):
    new = {}
    model._append_kv(new, k, v)
    cache[i] = new


def repair(model, cache, hb, split, rows):
    H = cached_rows(cache, split)
    if not 0 <= rows <= H or hb.shape[0] < rows:
        raise ValueError(f"repair of {rows} rows: {H} cached, {hb.shape[0]} inputs")
    if rows == 0:
        return
    pos = torch.arange(rows, device=model.device)
    tmp = model.new_cache()
    h = hb[:rows].to(model.device)
    for i in range(split, model.n_layers):
        h = model.layer(i, h, pos, tmp)
        c, t = cache[i], tmp[i]
        if model.layer_types[i] == "attn":
            _put_kv(model, cache, i, torch.cat((t["k"], c["k"][:, rows:]), 1), torch.cat((t["v"], c["v"][:, rows:]), 1))
        elif rows == c["len"]:
            cache[i] = dict(conv=t["conv"], rec=t["rec"], len=rows)
        tmp[i] = {}


def fill_inputs(model, arm, i, b):
    f = arm.fill_of(model.layer_types[i])
    if f == "proj":
        return arm.projector(i, b)
    if f == "identity":
        return b
    raise ValueError(f"no fill inputs for fill {f!r}")


def repair_selected(model, cache, arm, b, rows):
    if len(rows) == 0:
        return
    P = b.shape[0]
    r = torch.as_tensor(rows, dtype=torch.long, device=model.device)
    pos = torch.arange(P, device=model.device)
    b = b.to(model.device)
    hr = b[r]
    tmp = model.new_cache()
    for i in range(arm.split, model.n_layers):
        x = fill_inputs(model, arm, i, b)
        hr_next = model.layer_rows(i, x.index_copy(0, r, hr.to(x.dtype)), pos, r, tmp)
        if model.layer_types[i] == "attn":
            c, t = cache[i], tmp[i]
            _put_kv(model, cache, i, c["k"].index_copy(1, r, t["k"][:, r]), c["v"].index_copy(1, r, t["v"][:, r]))
        tmp[i] = {}
        hr = hr_next
