"""Layer-major RidgeFill prefill (code/kva/kva.py:282-460 semantics).

  1. run_lower: layers < split run exactly on all N prompt rows (shared by every arm at that split);
  2. finish: for each late layer i >= split, the prefix rows [0, P) only fill layer i's cache (from a
     predicted input, SwiftKV's K/V, the K/V fold, ...), then the exact tail rows [P, N) run the full layer
     over that cache (attention over all N cached rows; the GDN recurrence continues from the filled state).
This is the engine's chunk-major computation reordered by causality. With the B200 model the fills of all
late layers are independent of each other (each reads only h_S), so finish() batches the ridge maps of
every late layer into one fused fill (models/b200.py: fill_batch) before the tail walks the layers.
"""
from __future__ import annotations

import torch

from .arm import ORACLE_RESCALE, TAIL_RESCALE


def context_input(b, mix, split, k):
    """The context projector's input rows [b, c_{split-1}, .., c_{split-k}]."""
    return torch.cat([b] + [mix[split - j].to(b.device, b.dtype) for j in range(1, k + 1)], -1)


def run_lower(model, ids, splits, hs_device=None, hook=None, mix=None, tick=None, reserve=64):
    """Exact forward up to max(splits). Returns ({split: h_split [N, H]}, cache with layers < max(splits)
    filled). hook(i, h): every layer input; mix(i, a): every mixer output; tick(i): called before layer i with no
    tensor (a scheduler's point to run other work between layers); reserve: cache rows kept free past the prompt
    (decode steps append there without copying)."""
    if isinstance(splits, int):
        splits = [splits]
    ids = ids.to(model.device)
    pos = torch.arange(ids.shape[0], device=model.device)
    if hasattr(model, "reserve"):
        model.reserve(ids.shape[0] + reserve)
    cache = model.new_cache()
    h = model.embed(ids)
    hs = {}
    top = max(splits)
    stable = getattr(model, "stable", lambda t: t)
    for i in range(top):
        if i in splits:
            hs[i] = stable(h) if hs_device is None else h.to(hs_device)
        if hook is not None:
            hook(i, stable(h))
        if tick is not None:
            tick(i)
        h = model.layer(i, h, pos, cache, mix=mix)
    hs[top] = stable(h) if hs_device is None else h.to(hs_device)
    return hs, cache


def late_inputs_row0(model, ids, split):
    """Exact late-layer inputs of position 0 (it depends on itself only)."""
    got = {}
    model.forward_exact(ids[:1], hook=lambda i, h: got.__setitem__(i, h) if i != "final" and i >= split else None)
    return got


def oracle_tap(store, first, rows, device="cpu"):
    """hook(i, h) keeping rows [0, rows) of every layer input i >= first (the true late inputs)."""
    def hook(i, h):
        if i != "final" and i >= first:
            store[i] = h[:rows].to(device)
    return hook


def kv_target(model, i, h):
    """Pre-RoPE [k | v] [tokens, 2 * kv_heads * head_dim] of layer inputs h (the K/V fold's target)."""
    r = model.reads(i, h)
    return torch.cat((r["k"].flatten(1), r["v"].flatten(1)), 1)


def splice_kv(model, i, x, xo, part):
    """Pre-RoPE (k, v): `part` from the true inputs xo, the other half from the filled inputs x."""
    f, e = model.reads(i, x), model.reads(i, xo)
    return (e["k"], f["v"]) if part == "k" else (f["k"], e["v"])


def rescale_kv(model, i, x, mode, xo=None, scale=None):
    """Pre-RoPE (k, v) filled from x with one half rescaled per row and KV head: knorm / vnorm to the norm of
    the true inputs xo, kdir xo's direction at the filled norm, ktail / vtail times scale [kv_heads, 1]."""
    f = model.reads(i, x)
    part = mode[0]
    a = f[part].float()
    if scale is None:
        t = model.reads(i, xo)[part].float()
        na, nt = a.norm(dim=-1, keepdim=True), t.norm(dim=-1, keepdim=True)
        a = t * (na / nt.clamp_min(1e-30)) if mode == "kdir" else a * (nt / na.clamp_min(1e-30))
    else:
        a = a * scale
    a = a.to(f[part].dtype)
    return (a, f["v"]) if part == "k" else (f["k"], a)


def tail_scale(model, i, h_true, x_fill, part):
    """[kv_heads, 1]: mean over tail rows of ||true|| / ||filled|| of layer i's K or V."""
    t = model.reads(i, h_true)[part].float().norm(dim=-1)
    f = model.reads(i, x_fill)[part].float().norm(dim=-1)
    return (t / f.clamp_min(1e-30)).mean(0)[:, None]


def _validate(arm, model, n, P, oracle, rows, fill_reuse, mix):
    split, R, part, tb, rs = arm.split, arm.refresh, arm.exact_part, arm.tail_bias_from, arm.rescale
    if arm.context and (mix is None or not arm.uses("proj") or arm.uses("swiftkv") or arm.uses("kvfold")):
        raise ValueError("context arms fill from a projector and need the lower mixer outputs (mix)")
    if rows is not None and (fill_reuse is not None or arm.fill == "swiftkv" or arm.uses("kvfold")
                             or int(rows[-1]) >= P or bool((rows.diff() <= 0).any())):
        raise ValueError("exact rows: sorted unique rows < P, no fill reuse, not swiftkv or kvfold")
    if R is not None and (not split <= R < model.n_layers - 1 or arm.fill != "proj" or arm.fill_by_type
                          or fill_reuse is not None or arm.f1 or arm.st
                          or getattr(arm.refresh_projector, "split", None) != R + 1):
        raise ValueError("refresh R: split <= R < L - 1, fill 'proj', a refresh_projector of split R + 1; no fill "
                         "reuse, f1 or st")
    if part is not None and (part not in ("k", "v") or oracle is None or rows is not None or R is not None
                             or fill_reuse is not None):
        raise ValueError("exact_part 'k' | 'v' reads the true late inputs (oracle); no exact rows, refresh or reuse")
    if tb is not None and (arm.context or R is not None or fill_reuse is not None):
        raise ValueError("tail_bias_from: no context, refresh or fill reuse")
    skip = arm.tail_bias_skip_last
    if (tb is None and skip) or (tb is not None and not 0 <= skip < n - P):
        raise ValueError(f"tail_bias_skip_last {skip}: needs tail_bias_from and 0 <= it < the tail ({n - P})")
    if rs is not None and (rs not in ORACLE_RESCALE + TAIL_RESCALE or arm.fill != "proj" or arm.f1
                           or part is not None or rows is not None or R is not None or fill_reuse is not None
                           or (rs in ORACLE_RESCALE and oracle is None) or (rs in TAIL_RESCALE and arm.context)):
        raise ValueError("rescale knorm | kdir | vnorm (oracle) | ktail | vtail (no context): fill 'proj'; no f1, "
                         "exact_part, exact rows, refresh or fill reuse")
    rskip = arm.rescale_skip_last
    if (rs not in TAIL_RESCALE and rskip) or (rs in TAIL_RESCALE and not 0 <= rskip < n - P):
        raise ValueError(f"rescale_skip_last {rskip}: needs rescale ktail | vtail and 0 <= it < the tail ({n - P})")


def _plain_batchable(arm, model, P, rows, fill_reuse, row0, fill_store):
    """True when every late layer's prefix fill is a plain projector or identity fill (no per-layer
    dependence on the tail): the B200 model then runs all fills as one batch."""
    return (P > 0 and hasattr(model, "fill_batch") and arm.fill in ("proj", "identity") and arm.fill_by_type is None
            and rows is None and fill_reuse is None and row0 is None and not arm.context and arm.refresh is None
            and arm.tail_bias_from is None and arm.exact_part is None and arm.rescale is None)


def finish(model, ids, h_split, lower_cache, arm, keep, oracle=None, keep_cache=True, fill_store=None,
           fill_reuse=None, exact_rows=None, row_inputs=None, hook=None, mix=None, timer=None, tick=None):
    """Layers >= arm.split for one arm. keep: number of final rows whose logits to return. Returns
    (logits [keep, V] fp32, cache, P). tick(i): called before late layer i's tail rows run. See the module doc and
    engine/arm.py for the options."""
    n = ids.shape[0]
    split = arm.split
    P = arm.prefix_len(n)
    pos = torch.arange(n, device=model.device)
    if hasattr(model, "reserve"):
        model.reserve(n + 64)
    h_split = h_split.to(model.device)
    cache = [dict(c) for c in lower_cache[:split]] + [dict() for _ in range(model.n_layers - split)]
    if arm.fill == "swiftkv_native":
        if split != model.swift_layers:
            raise ValueError(f"SwiftKV native runs at its own split {model.swift_layers}")
        q0 = n - keep
        h = h_split[q0:]
        for i in range(split, model.n_layers):
            model.swift_fill(i, h_split, pos, cache)
            h = model.swift_layer(i, h, pos[q0:], cache)
            if not keep_cache:
                cache[i] = {}
        return model.logits(h), cache, P
    if keep > n - P:
        raise ValueError(f"keep {keep} rows > exact tail {n - P}")
    rows = None
    if exact_rows is not None and len(exact_rows) > 0:
        rows = torch.as_tensor(exact_rows, dtype=torch.long, device=model.device)
    _validate(arm, model, n, P, oracle, rows, fill_reuse, mix)
    b = h_split[:P]
    h = h_split[P:]
    bx = b
    if arm.context:
        bx = context_input(b, {j: mix[j][:P] for j in range(split - arm.context, split)}, split, arm.context)
    row0 = late_inputs_row0(model, ids, split) if (arm.f1 and P > 0) else None
    hr = h_split[rows] if rows is not None else None
    R, part, tb, rs = arm.refresh, arm.exact_part, arm.tail_bias_from, arm.rescale
    t_mean = n - P - arm.tail_bias_skip_last
    t_scale = n - P - arm.rescale_skip_last

    batched = _plain_batchable(arm, model, P, rows, fill_reuse, row0, fill_store)
    if batched:
        late = list(range(split, model.n_layers))
        if timer is not None:
            with timer.stage("fill"):
                model.fill_batch(late, b, pos[:P], cache, arm.projector if arm.fill == "proj" else None)
        else:
            model.fill_batch(late, b, pos[:P], cache, arm.projector if arm.fill == "proj" else None)

    for i in range(split, model.n_layers):
        if P > 0 and fill_reuse is not None:
            if fill_reuse[i].get("n", P) != P:
                raise ValueError(f"reused fill of layer {i} has {fill_reuse[i]['n']} rows, P = {P}")
            cache[i] = dict(fill_reuse[i])
        elif P > 0 and not batched:
            fill = arm.fill_of(model.layer_types[i])
            if fill == "swiftkv":
                model.swift_fill(i, b, pos[:P], cache)
            elif fill == "kvfold":
                if model.layer_types[i] != "attn" or row0 is not None:
                    raise ValueError("kvfold fills attention layers only (fill_by_type for GDN layers), without f1")
                model.fill_kv(i, *arm.kvfold.kv(i, b), pos[:P], cache)
            elif fill == "none":
                if row0 is not None:
                    raise ValueError("fill 'none' takes no f1")
                if rows is not None:                     # only the exact rows reach layer i
                    if row_inputs is not None:
                        row_inputs[i] = hr
                    hr = model.layer(i, hr, pos[rows], cache)
            else:
                bias = None
                if fill == "proj":
                    x = arm.projector(i, bx) if R is None or i <= R else arm.refresh_projector(i, bx)
                    if tb is not None and i >= tb:       # h is the tail's layer-i input before layer i runs
                        r = h[:t_mean].float() - arm.projector(i, h_split[P:n - arm.tail_bias_skip_last]).float()
                        bias = r.mean(0).to(x.dtype)
                        x = x + bias
                elif fill == "identity":
                    x = b
                elif fill == "oracle":
                    x = oracle[i][:P].to(b.device)
                else:
                    raise ValueError(fill)
                if row0 is not None:
                    x = torch.cat((row0[i], x[1:]), 0)
                if rows is not None:
                    if row_inputs is not None:
                        row_inputs[i] = hr
                    x = x.index_copy(0, rows, hr.to(x.dtype))
                if i == R:
                    bx = model.layer(i, x, pos[:P], cache)
                    if rows is not None:
                        hr = bx[rows]
                elif rows is not None:
                    hr = model.layer_rows(i, x, pos[:P], rows, cache)
                elif part is not None and model.layer_types[i] == "attn":
                    model.fill_kv(i, *splice_kv(model, i, x, oracle[i][:P].to(x.device), part), pos[:P], cache)
                elif rs is not None and model.layer_types[i] == "attn":
                    if rs in TAIL_RESCALE:
                        xt = arm.projector(i, h_split[P:n - arm.rescale_skip_last])
                        kv = rescale_kv(model, i, x, rs, scale=tail_scale(
                            model, i, h[:t_scale], xt if bias is None else xt + bias, rs[0]))
                    else:
                        kv = rescale_kv(model, i, x, rs, xo=oracle[i][:P].to(x.device))
                    model.fill_kv(i, *kv, pos[:P], cache)
                else:
                    model.fill(i, x, pos[:P], cache)
        if P > 0 and fill_store is not None:
            fill_store[i] = dict(cache[i])
        st = arm.st.get(i) if (arm.st and P > 0) else None
        if st is not None:
            cache[i]["rec"] = cache[i]["rec"] + st.to(cache[i]["rec"])
        if hook is not None:
            hook(i, model.stable(h) if hasattr(model, "stable") else h)
        if tick is not None:
            tick(i)
        h = model.layer(i, h, pos[P:], cache)
        if not keep_cache:
            cache[i] = {}
    return model.logits(h[-keep:]), cache, P


def prefill(model, ids, arm, keep=1, **kw):
    """run_lower + finish for one arm: (logits [keep, V], cache, P)."""
    if arm.fill == "exact" or arm.split is None:
        pos_keep = torch.arange(ids.shape[0] - keep, ids.shape[0], device=model.device)
        logits, cache = model.forward_exact(ids.to(model.device), keep=pos_keep)
        return logits, cache, 0
    hs, lower = run_lower(model, ids, [arm.split])
    return finish(model, ids, hs[arm.split], lower, arm, keep, **kw)
