"""Layer-major RidgeFill prefill (the computation of code/kva/kva.py:282-460, reordered by causality).

run_lower runs layers < split exactly over all N prompt rows; every arm at that split shares the result. finish
then walks the late layers i >= split. At each one the prefix rows [0, P) only write layer i's cache: K/V of an
attention layer, conv window and delta-rule state of a GDN layer, computed from a stand-in for the layer's input
(the ridge-predicted x_i, the split input itself, SwiftKV's K/V, the K/V fold, ...). The exact tail rows [P, N)
then run the whole layer against that cache.

When every late layer's prefix fill is a plain projector or identity fill, the fills depend on h_S alone and not
on each other. The B200 model then writes all of them in one batched, fused fill (fill_batch) before the tail
walks the layers.
"""
from __future__ import annotations

import torch

from ..ridge.projector import Projector
from .arm import ORACLE_RESCALE, TAIL_RESCALE

_EPS = 1e-30


def context_input(b, mix, split, k):
    """Context projector input: the split rows b followed by the mixer outputs of layers split-1, ..., split-k."""
    cols = [b]
    cols += [mix[split - j].to(b.device, b.dtype) for j in range(1, k + 1)]
    return torch.cat(cols, dim=-1)


def _keep_split(model, h, device):
    if device is not None:
        return h.to(device)
    return model.stable(h) if hasattr(model, "stable") else h


def run_lower(model, ids, splits, hs_device=None, hook=None, mix=None, tick=None, reserve=64, maps=None):
    """Exact forward through layers < max(splits).

    Returns ({split: layer-split input rows [N, H]}, a cache whose layers < max(splits) are filled). hook(i, h) sees
    every layer input, mix(i, a) every mixer output; tick(i) runs before layer i (a scheduler's slot for other
    work between layers); `reserve` cache rows past the prompt are preallocated so decode appends in place; maps: the
    arm's projector, told that a prompt starts (streamed maps begin their copies, overlapping these layers)."""
    wanted = {splits} if isinstance(splits, int) else set(splits)
    if maps is not None and hasattr(maps, "begin") and model.device.type == "cuda":
        maps.begin(model.device)
    ids = ids.to(model.device)
    n = ids.shape[0]
    if hasattr(model, "reserve"):
        model.reserve(n + reserve)
    pos = torch.arange(n, device=model.device)
    cache = model.new_cache()
    kept = {}
    h = model.embed(ids)
    last = max(wanted)
    for i in range(last):
        if i in wanted:
            kept[i] = _keep_split(model, h, hs_device)
        if hook is not None:
            hook(i, _keep_split(model, h, None))
        if tick is not None:
            tick(i)
        h = model.layer(i, h, pos, cache, mix=mix)
    kept[last] = _keep_split(model, h, hs_device)
    return kept, cache


def late_inputs_row0(model, ids, split):
    """True late-layer inputs of position 0, which attends to itself only."""
    return oracle_layers(model, ids[:1], split)


def oracle_layers(model, ids, first):
    got = {}

    def grab(i, h):
        if i != "final" and i >= first:
            got[i] = h
    model.forward_exact(ids, hook=grab)
    return got


def oracle_tap(store, first, rows, device="cpu"):
    """A forward hook storing rows [0, rows) of every layer input from layer `first` on (the true late inputs)."""
    def tap(i, h):
        if i == "final" or i < first:
            return
        store[i] = h[:rows].to(device)
    return tap


def kv_target(model, i, h):
    """[k | v] before RoPE, [tokens, 2 * kv_heads * head_dim], of layer i for inputs h (the K/V fold's target)."""
    reads = model.reads(i, h)
    return torch.cat([reads["k"].flatten(1), reads["v"].flatten(1)], dim=1)


def splice_kv(model, i, x, xo, part):
    """(k, v) before RoPE with `part` ('k' or 'v') read from the true inputs xo and the other from the fill x."""
    filled, true = model.reads(i, x), model.reads(i, xo)
    out = {"k": filled["k"], "v": filled["v"]}
    out[part] = true[part]
    return out["k"], out["v"]


def rescale_kv(model, i, x, mode, xo=None, scale=None):
    """(k, v) before RoPE filled from x, with the half named by mode[0] rescaled per row and KV head:
    knorm / vnorm take the norm of the true inputs' half, kdir takes the true direction at the filled norm,
    ktail / vtail multiply by `scale` [kv_heads, 1]."""
    filled = model.reads(i, x)
    half = mode[0]
    got = filled[half].float()
    if scale is not None:
        got = got * scale
    else:
        true = model.reads(i, xo)[half].float()
        n_fill = got.norm(dim=-1, keepdim=True)
        n_true = true.norm(dim=-1, keepdim=True)
        if mode == "kdir":
            got = true * (n_fill / n_true.clamp_min(_EPS))
        else:
            got = got * (n_true / n_fill.clamp_min(_EPS))
    out = {"k": filled["k"], "v": filled["v"]}
    out[half] = got.to(filled[half].dtype)
    return out["k"], out["v"]


def tail_scale(model, i, h_true, x_fill, part):
    """[kv_heads, 1]: the tail rows' mean ratio of the true to the filled norm of layer i's K or V."""
    true = model.reads(i, h_true)[part].float().norm(dim=-1)
    fill = model.reads(i, x_fill)[part].float().norm(dim=-1)
    return (true / fill.clamp_min(_EPS)).mean(0).unsqueeze(1)


def _problems(arm, model, n, P, oracle, rows, fill_reuse, mix):
    """Yield a message for every option combination finish() does not define."""
    tail = n - P
    R, part, tb, rs = arm.refresh, arm.exact_part, arm.tail_bias_from, arm.rescale
    if arm.context and (mix is None or not arm.uses("proj") or arm.uses("swiftkv") or arm.uses("kvfold")):
        yield "a context arm fills from a projector and needs the lower layers' mixer outputs (mix)"
    if rows is not None:
        ordered = bool((rows.diff() > 0).all())
        if fill_reuse is not None or arm.fill == "swiftkv" or arm.uses("kvfold") or int(rows[-1]) >= P \
                or not ordered:
            yield "exact rows must be increasing prefix rows, without fill reuse, swiftkv or kvfold"
    if R is not None:
        ok = arm.split <= R < model.n_layers - 1 and arm.fill == "proj" and not arm.fill_by_type \
            and fill_reuse is None and not arm.f1 and not arm.st \
            and getattr(arm.refresh_projector, "split", None) == R + 1
        if not ok:
            yield (f"refresh at layer {R} needs split <= R < n_layers - 1, fill 'proj', a refresh_projector fitted "
                   "at R + 1, and no fill reuse, f1 or st")
    if part is not None and (part not in ("k", "v") or oracle is None or rows is not None or R is not None
                             or fill_reuse is not None):
        yield "exact_part ('k' or 'v') reads the true late inputs (oracle) and excludes exact rows, refresh, reuse"
    if tb is not None and (arm.context or R is not None or fill_reuse is not None):
        yield "tail_bias_from excludes context, refresh and fill reuse"
    skip = arm.tail_bias_skip_last
    if (skip and tb is None) or (tb is not None and not 0 <= skip < tail):
        yield f"tail_bias_skip_last={skip} needs tail_bias_from and must lie in [0, {tail})"
    if rs is not None:
        allowed = rs in ORACLE_RESCALE + TAIL_RESCALE and arm.fill == "proj" and not arm.f1 and part is None \
            and rows is None and R is None and fill_reuse is None
        if not allowed or (rs in ORACLE_RESCALE and oracle is None) or (rs in TAIL_RESCALE and arm.context):
            yield (f"rescale {rs!r}: one of {ORACLE_RESCALE + TAIL_RESCALE} on a 'proj' fill (the first three read "
                   "the oracle, the tail ones take no context), without f1, exact_part, exact rows, refresh, reuse")
    rskip = arm.rescale_skip_last
    if (rskip and rs not in TAIL_RESCALE) or (rs in TAIL_RESCALE and not 0 <= rskip < tail):
        yield f"rescale_skip_last={rskip} needs a tail rescale and must lie in [0, {tail})"


def _plain_batchable(arm, model, P, rows, fill_reuse, row0, fill_store):
    """Every late prefix fill is a plain projector / identity fill that reads h_S only, so a model with
    fill_batch can write them all at once."""
    if P <= 0 or not hasattr(model, "fill_batch") or arm.fill not in ("proj", "identity"):
        return False
    extras = (arm.fill_by_type, rows, fill_reuse, row0, arm.refresh, arm.tail_bias_from, arm.exact_part,
              arm.rescale)
    return all(e is None for e in extras) and not arm.context


class _LateLayers:
    """finish()'s state for one arm while it walks the late layers."""

    def __init__(self, model, ids, h_split, arm, oracle, rows, row_inputs, mix):
        self.model, self.arm, self.oracle, self.row_inputs = model, arm, oracle, row_inputs
        n = ids.shape[0]
        self.n = n
        self.P = P = arm.prefix_len(n)
        self.pos = torch.arange(n, device=model.device)
        self.h_split = h_split
        self.b = h_split[:P]                    # prefix rows' layer-split inputs
        self.h = h_split[P:]                    # the exact tail, advanced layer by layer
        self.rows = rows
        self.hr = h_split[rows] if rows is not None else None      # exact rows, advanced layer by layer
        self.src = self.b                       # what the projector reads (context columns / refreshed rows)
        if arm.context:
            lower_mix = {j: mix[j][:P] for j in range(arm.split - arm.context, arm.split)}
            self.src = context_input(self.b, lower_mix, arm.split, arm.context)
        self.row0 = late_inputs_row0(model, ids, arm.split) if (arm.f1 and P > 0) else None
        self.n_bias = n - P - arm.tail_bias_skip_last
        self.n_scale = n - P - arm.rescale_skip_last

    # -- stand-in inputs of one late layer
    def projected(self, i):
        a = self.arm
        refreshed = a.refresh is not None and i > a.refresh
        proj = a.refresh_projector if refreshed else a.projector
        on_device = getattr(self.model, "project_map", None)      # the B200 model's own GEMM
        x = on_device(proj, i, self.src) if on_device is not None and isinstance(proj, Projector) \
            else proj(i, self.src)
        if a.tail_bias_from is None or i < a.tail_bias_from:
            return x, None
        # self.h holds the tail's layer-i inputs: the mean tail residual of the map is added to every prefix row
        predicted = a.projector(i, self.h_split[self.P:self.n - a.tail_bias_skip_last]).float()
        bias = (self.h[:self.n_bias].float() - predicted).mean(0).to(x.dtype)
        return x + bias, bias

    def stand_in(self, i, fill):
        if fill == "proj":
            return self.projected(i)
        if fill == "identity":
            return self.b, None
        if fill == "oracle":
            return self.oracle[i][:self.P].to(self.b.device), None
        raise ValueError(f"unknown fill {fill!r}")

    # -- writing layer i's prefix cache
    def write(self, i, cache):
        fill = self.arm.fill_of(self.model.layer_types[i])
        handler = {"swiftkv": self._swift, "kvfold": self._kvfold, "none": self._none}.get(fill, self._computed)
        handler(i, fill, cache)

    def _swift(self, i, fill, cache):
        self.model.swift_fill(i, self.b, self.pos[:self.P], cache)

    def _kvfold(self, i, fill, cache):
        if self.model.layer_types[i] != "attn" or self.row0 is not None:
            raise ValueError("the K/V fold writes attention layers only (GDN layers via fill_by_type), without f1")
        k, v = self.arm.kvfold.kv(i, self.b)
        self.model.fill_kv(i, k, v, self.pos[:self.P], cache)

    def _none(self, i, fill, cache):
        if self.row0 is not None:
            raise ValueError("fill 'none' cannot take f1")
        if self.rows is None:
            return
        if self.row_inputs is not None:         # only the exact rows reach this layer
            self.row_inputs[i] = self.hr
        self.hr = self.model.layer(i, self.hr, self.pos[self.rows], cache)

    def _computed(self, i, fill, cache):
        m, a, P = self.model, self.arm, self.P
        ppos = self.pos[:P]
        x, bias = self.stand_in(i, fill)
        if self.row0 is not None:
            x = torch.cat((self.row0[i], x[1:]), 0)
        if self.rows is not None:
            if self.row_inputs is not None:
                self.row_inputs[i] = self.hr
            x = x.index_copy(0, self.rows, self.hr.to(x.dtype))
        attn = m.layer_types[i] == "attn"
        if i == a.refresh:
            self.src = m.layer(i, x, ppos, cache)
            if self.rows is not None:
                self.hr = self.src[self.rows]
        elif self.rows is not None:
            self.hr = m.layer_rows(i, x, ppos, self.rows, cache)
        elif a.exact_part is not None and attn:
            m.fill_kv(i, *splice_kv(m, i, x, self.oracle[i][:P].to(x.device), a.exact_part), ppos, cache)
        elif a.rescale is not None and attn:
            m.fill_kv(i, *self._rescaled(i, x, bias), ppos, cache)
        else:
            m.fill(i, x, ppos, cache)

    def _rescaled(self, i, x, bias):
        a, m = self.arm, self.model
        if a.rescale not in TAIL_RESCALE:
            return rescale_kv(m, i, x, a.rescale, xo=self.oracle[i][:self.P].to(x.device))
        tail_fill = a.projector(i, self.h_split[self.P:self.n - a.rescale_skip_last])
        if bias is not None:
            tail_fill = tail_fill + bias
        factor = tail_scale(m, i, self.h[:self.n_scale], tail_fill, a.rescale[0])
        return rescale_kv(m, i, x, a.rescale, scale=factor)


def _swiftkv_native(model, h_split, arm, keep, keep_cache, cache, n):
    if arm.split != model.swift_layers:
        raise ValueError(f"native SwiftKV runs only at its own split ({model.swift_layers})")
    pos = torch.arange(n, device=model.device)
    first = n - keep
    h = h_split[first:]
    for i in range(arm.split, model.n_layers):
        model.swift_fill(i, h_split, pos, cache)
        h = model.swift_layer(i, h, pos[first:], cache)
        if not keep_cache:
            cache[i] = {}
    return model.logits(h), cache, arm.prefix_len(n)


def finish(model, ids, h_split, lower_cache, arm, keep, oracle=None, keep_cache=True, fill_store=None,
           fill_reuse=None, exact_rows=None, row_inputs=None, hook=None, mix=None, timer=None, tick=None):
    """Layers >= arm.split for one arm; returns (logits of the last `keep` rows [keep, V] fp32, cache, P).

    oracle: true late inputs (oracle fills, exact_part, oracle rescales); fill_store / fill_reuse: save or reuse
    the prefix fills per layer; exact_rows: prefix rows recomputed exactly through the late layers over the others
    as filled (row_inputs receives their per-layer inputs); hook(i, h): the tail's layer inputs; tick(i): runs
    before the tail enters late layer i; timer: a stage timer around the batched fill. The arm's own options are
    documented in engine/arm.py."""
    n = ids.shape[0]
    split = arm.split
    if hasattr(model, "reserve"):
        model.reserve(n + 64)
    h_split = h_split.to(model.device)
    cache = [dict(c) for c in lower_cache[:split]]
    cache += [{} for _ in range(split, model.n_layers)]
    if arm.fill == "swiftkv_native":
        return _swiftkv_native(model, h_split, arm, keep, keep_cache, cache, n)
    P = arm.prefix_len(n)
    if keep > n - P:
        raise ValueError(f"{keep} logit rows asked from an exact tail of {n - P}")
    rows = None
    if exact_rows is not None and len(exact_rows):
        rows = torch.as_tensor(exact_rows, dtype=torch.long, device=model.device)
    for problem in _problems(arm, model, n, P, oracle, rows, fill_reuse, mix):
        raise ValueError(problem)
    run = _LateLayers(model, ids, h_split, arm, oracle, rows, row_inputs, mix)
    tail_pos = run.pos[P:]

    batched = _plain_batchable(arm, model, P, rows, fill_reuse, run.row0, fill_store)
    if batched:
        late = list(range(split, model.n_layers))
        proj = arm.projector if arm.fill == "proj" else None
        if timer is None:
            model.fill_batch(late, run.b, run.pos[:P], cache, proj)
        else:
            with timer.stage("fill"):
                model.fill_batch(late, run.b, run.pos[:P], cache, proj)

    stable = getattr(model, "stable", None)
    for i in range(split, model.n_layers):
        if P > 0:
            if fill_reuse is not None:
                have = fill_reuse[i].get("n", P)
                if have != P:
                    raise ValueError(f"the reused fill of layer {i} holds {have} rows; this arm fills {P}")
                cache[i] = dict(fill_reuse[i])
            elif not batched:
                run.write(i, cache)
            if fill_store is not None:
                fill_store[i] = dict(cache[i])
            st = arm.st.get(i) if arm.st else None
            if st is not None:
                cache[i]["rec"] = cache[i]["rec"] + st.to(cache[i]["rec"])
        if hook is not None:
            hook(i, stable(run.h) if stable is not None else run.h)
        if tick is not None:
            tick(i)
        run.h = model.layer(i, run.h, tail_pos, cache)
        if not keep_cache:
            cache[i] = {}
    return model.logits(run.h[-keep:]), cache, P


def prefill(model, ids, arm, keep=1, **kw):
    """Full prefill of one arm (run_lower, then finish): (logits [keep, V], cache, P)."""
    if arm.split is None or arm.fill == "exact":
        n = ids.shape[0]
        logits, cache = model.forward_exact(ids.to(model.device),
                                            keep=torch.arange(n - keep, n, device=model.device))
        return logits, cache, 0
    hs, lower = run_lower(model, ids, [arm.split], maps=arm.projector)
    return finish(model, ids, hs[arm.split], lower, arm, keep, **kw)
