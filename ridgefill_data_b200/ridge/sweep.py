"""The fit driver: one capture pass, ridge maps for every split (code/scripts/fit_sweep.py semantics).

1. capture   exact forward over the calibration documents; for every split S and late layer i >= S the
             shifted sums of (h_S -> layer i's input), fp32 per block into fp64 accumulators (on the device
             when the model is on CUDA: the tcgen05 Gram kernel with split-bf16 operands).
2. per split ridge maps for the lambda grid (EigenFit on the CPU, or CholeskyFit on the device), then
             lambda chosen on held-out documents by the mean read cosine of the late layers' reads (pre-RoPE
             K/V, or the GDN in-projections) of the predicted vs the true inputs; the identity map is scored
             as a baseline.
3. outputs   the map file (Projector.save), the fit record JSON (provenance, rows, docs, lambda_star,
             mean_read_cos, per_layer_read_cos, projector, projector_sha256) and optionally the sufficient
             statistics (.pt) for refits without recapture.
"""
from __future__ import annotations

import time
from pathlib import Path

import torch
import torch.nn.functional as F

from ..utils import prov
from .fit import CholeskyFit, EigenFit
from .projector import Projector, meta_of
from .stats import RidgeStats

LAMBDAS = (1e-4, 3e-4, 1e-3, 3e-3, 0.01, 0.03, 0.1, 0.3, 1.0)


class StaleProjector(RuntimeError):
    """A map file exists that was fitted on another calibration list (its recorded rows differ)."""


def stale_projectors(paths, rows):
    return [(p, meta_of(p).get("rows")) for p in paths if Path(p).exists() and meta_of(p).get("rows") != str(rows)]


def _common_shifts(model, doc, splits, group):
    """Shifts (first-block means of the boundary and every late layer's input) taken from one document on rank 0
    and broadcast, so every rank's sums share them and can simply be added."""
    import torch.distributed as dist
    L, H = model.n_layers, model.hidden
    lo = min(splits)
    buf = torch.zeros(L - lo + 1, H, dtype=torch.float32, device=model.device)
    if dist.get_rank(group) == 0:
        got = {}
        with torch.no_grad():
            model.forward_exact(torch.as_tensor(doc["ids"]).to(model.device),
                                hook=lambda i, h: got.__setitem__(i, h[:8192].float().mean(0)) if i != "final" else None)
        for i in range(lo, L):
            buf[i - lo] = got[i]
    dist.broadcast(buf, src=dist.get_global_rank(group, 0) if group is not None else 0, group=group)
    return {i: buf[i - lo] for i in range(lo, L)}


def unit_rms(model, h):
    """h / rms(h) in fp32 (rms with the model's norm eps): the direction a late layer's input norm keeps."""
    hf = h.float()
    return hf * torch.rsqrt(hf.square().mean(-1, keepdim=True) + model.eps)


def capture(model, docs, splits, device=None, log=print, group=None, unitrms=False, kvfold=False):
    """{S: RidgeStats} over the documents (forward_exact with a capture hook). With a process group the documents
    are split over the ranks (data parallel), every rank uses rank 0's shifts, and the fp64 sums are added over
    the ranks at the end (one reduction per statistic: each rank keeps its partial sums on the device until then).
    unitrms / kvfold: also the sums of the extra targets (same capture pass), returned as stats["unitrms"][S] (x =
    h_S, targets y_i / rms(y_i)) and stats["kvfold"][S] (x = h_S / rms(h_S), targets the pre-RoPE [k | v] of
    every late attention layer, with their per-feature sums of squares "sq")."""
    L, H = model.n_layers, model.hidden
    dev = device or model.device
    stats = {S: RidgeStats(S, range(S, L), H, dev) for S in splits}
    extra = {}
    if (unitrms or kvfold) and group is not None:
        raise ValueError("the unit-RMS and K/V-fold sums are captured on one process (no data-parallel capture)")
    if unitrms:
        extra["unitrms"] = {S: RidgeStats(S, range(S, L), H, dev) for S in splits}
    if kvfold:
        from ..engine.prefill import kv_target
        kv_dim = 2 * model.n_kv * model.head_dim
        extra["kvfold"] = {S: RidgeStats(S, [i for i in range(S, L) if model.layer_types[i] == "attn"], H, dev,
                                         out_dim=kv_dim) for S in splits}
        sq = {S: {i: torch.zeros(kv_dim, dtype=torch.float64, device=dev) for i in extra["kvfold"][S].layers}
              for S in splits}
    if group is not None:
        import torch.distributed as dist
        shifts = _common_shifts(model, docs[0], splits, group)
        for S, st in stats.items():
            st.cx = shifts[S].to(dev)
            st.cy = {i: shifts[i].to(dev) for i in range(S, L)}
        rank, world = dist.get_rank(group), dist.get_world_size(group)
        docs = docs[rank::world]
    t0 = time.time()
    with torch.no_grad():
        for j, d in enumerate(docs):
            def hook(i, h):
                if i == "final":
                    return
                if i in stats:
                    stats[i].begin(h)
                    if unitrms:
                        extra["unitrms"][i].begin(h)
                    if kvfold:
                        extra["kvfold"][i].begin(unit_rms(model, h))
                u = unit_rms(model, h) if unitrms else None
                kv = kv_target(model, i, h) if kvfold and model.layer_types[i] == "attn" else None
                for S, st in stats.items():
                    if S <= i:
                        st.add_layer(i, h)
                        if unitrms:
                            extra["unitrms"][S].add_layer(i, u)
                        if kv is not None:
                            extra["kvfold"][S].add_layer(i, kv)
                            c = extra["kvfold"][S].cy[i].to(kv.device)
                            sq[S][i] += (kv.float() - c).double().square().sum(0).to(dev)
            model.forward_exact(torch.as_tensor(d["ids"]).to(model.device), hook=hook)
            if log and (j % 10 == 0 or j == len(docs) - 1):
                log(f"capture {j + 1}/{len(docs)} rows {int(stats[splits[0]].n)} ({time.time() - t0:.0f}s)")
    if group is not None:
        _reduce_sums(stats, group, log)
    if kvfold:
        for S, st in extra["kvfold"].items():
            st.sq = sq[S]
    stats.update(extra)
    return stats


def _reduce_sums(stats, group, log=None):
    """Sum every rank's fp64 statistics: through NVSwitch multicast (parallel/nvls.py NvlsF64Reducer, this package's
    kernel) when the GPUs offer it, else one NCCL all-reduce per tensor."""
    import torch.distributed as dist
    tensors = []
    for st in stats.values():
        n = torch.tensor([st.n], dtype=torch.float64, device=st.sx.device)
        dist.all_reduce(n, group=group)
        st.n = float(n.item())
        tensors += [st.sx, st.sxx] + list(st.sy.values()) + list(st.sxy.values())
    reducer = None
    if tensors and tensors[0].is_cuda and dist.get_backend(group) == "nccl":
        try:
            from ..parallel.nvls import NvlsF64Reducer, NvlsUnavailable
            reducer = NvlsF64Reducer(group)
        except (NvlsUnavailable, RuntimeError) as e:       # no multicast objects on these GPUs
            if log:
                log(f"fp64 sums through NCCL ({e})")
    if reducer is not None:
        try:
            reducer.allreduce_(tensors)
            from ..ops._ext import check_errors
            torch.cuda.synchronize()
            check_errors()
        finally:
            reducer.close()
        return
    for t in tensors:
        dist.all_reduce(t, group=group)


def read_cos(model, i, pred, true):
    """Mean over the layer's read tensors of the per-row-per-head cosine (code/scripts/fit_sweep.py:308-312)."""
    p, t = model.reads(i, pred), model.reads(i, true)
    if all(p[r].is_cuda and p[r].dtype == torch.bfloat16 for r in t):
        from ..ops.kernels import row_cosine                         # one warp per row (csrc/reduce.cu)
        return sum(row_cosine(p[r], t[r]).mean().item() for r in t) / len(t)
    return sum(F.cosine_similarity(p[r].float(), t[r].float(), dim=-1).mean().item() for r in t) / len(t)


def select_lambda(model, held, S, maps, lams):
    """Per candidate (each lambda, and 'identity'): {str(c): {layer: mean read cos}} over held documents."""
    late = list(range(S, model.n_layers))
    cand = list(lams) + ["identity"]
    sums = {c: {i: 0.0 for i in late} for c in cand}
    count = 0
    with torch.no_grad():
        for d in held:
            got = {}
            model.forward_exact(torch.as_tensor(d["ids"]).to(model.device),
                                hook=lambda i, h: got.__setitem__(i, h) if i != "final" and i >= S else None)
            count += 1
            for i in late:
                for c in cand:
                    if c == "identity":
                        x = got[S]
                    else:
                        w, b = maps[c][i]
                        x = F.linear(got[S], w.to(got[S].device, got[S].dtype), b.to(got[S].device, got[S].dtype))
                    sums[c][i] += read_cos(model, i, x, got[i])
    per_layer = {str(c): {i: v / count for i, v in s.items()} for c, s in sums.items()}
    mean = {c: sum(v.values()) / len(v) for c, v in per_layer.items()}
    best = max(lams, key=lambda lam: mean[str(lam)])
    return best, mean, per_layer


def fit_select_lean(model, stats_state, S, lams, held, solver="cholesky", center=True):
    """The per-split solve and held-out lambda choice without holding every lambda's maps: the held documents'
    true late inputs are captured once, each lambda's maps are solved, scored (mean read cosine, as
    select_lambda) and dropped, and only the best lambda's maps are kept (on the host). Returns (best, mean,
    per_layer, {best: {i: (weight, bias)}}). For full-size models, where every lambda's maps of every late layer
    would not fit next to the model and the statistics."""
    L = model.n_layers
    late = list(range(S, L))
    held_in = []
    with torch.no_grad():
        for d in held:
            got = {}
            model.forward_exact(torch.as_tensor(d["ids"]).to(model.device),
                                hook=lambda i, h: got.__setitem__(i, h) if i != "final" and i >= S else None)
            held_in.append(got)
        per_layer = {"identity": {i: sum(read_cos(model, i, g[S], g[i]) for g in held_in) / len(held_in)
                                  for i in late}}
        fit_ = CholeskyFit(stats_state, center=center, device=model.device) if solver == "cholesky" \
            else EigenFit(stats_state, center=center)
        best, best_maps = None, None
        for lam in lams:
            maps = fit_.layers(late, [lam])[lam] if solver == "cholesky" else \
                {i: fit_.layer(i, [lam])[lam] for i in late}
            scores = {}
            for i in late:
                w, b = maps[i]
                tot = 0.0
                for g in held_in:
                    x = F.linear(g[S], w.to(g[S].device, g[S].dtype), b.to(g[S].device, g[S].dtype))
                    tot += read_cos(model, i, x, g[i])
                scores[i] = tot / len(held_in)
            per_layer[str(lam)] = scores
            if best is None or sum(scores.values()) > sum(per_layer[str(best)].values()):
                best = lam
                best_maps = {i: (w.cpu(), b.cpu()) for i, (w, b) in maps.items()}
            del maps
    mean = {c: sum(v.values()) / len(v) for c, v in per_layer.items()}
    return best, mean, per_layer, {best: best_maps}


def fit_split(stats_state, S, L, lams, solver="eigen", center=True, device=None):
    """{lam: {i: (weight, bias)}} fp32 maps of split S."""
    late = list(range(S, L))
    if solver == "eigen":
        fit = EigenFit(stats_state, center=center)
        maps = {lam: {} for lam in lams}
        for i in late:
            for lam, wb in fit.layer(i, lams).items():
                maps[lam][i] = wb
        return maps
    fit = CholeskyFit(stats_state, center=center, device=device)
    return fit.layers(late, lams)


def select_lambda_kv(model, held, S, fold_maps, lams):
    """K/V-fold lambda selection: per candidate, the mean over held documents, late attention layers and K / V of
    the per-row-per-head cosine between the fold's prediction and the true pre-RoPE K / V."""
    from ..engine.prefill import kv_target
    late = [i for i in range(S, model.n_layers) if model.layer_types[i] == "attn"]
    sums = {lam: {i: 0.0 for i in late} for lam in lams}
    count = 0
    hd = model.head_dim
    with torch.no_grad():
        for d in held:
            got = {}
            model.forward_exact(torch.as_tensor(d["ids"]).to(model.device),
                                hook=lambda i, h: got.__setitem__(i, h) if i != "final" and i >= S else None)
            u = unit_rms(model, got[S])
            count += 1
            for i in late:
                true = kv_target(model, i, got[i]).float().unflatten(-1, (-1, hd))
                for lam in lams:
                    w, b = fold_maps[lam][i]
                    pred = F.linear(u, w.to(u.device), b.to(u.device)).unflatten(-1, (-1, hd))
                    sums[lam][i] += F.cosine_similarity(pred, true, dim=-1).mean().item()
    per_layer = {str(lam): {i: v / count for i, v in s.items()} for lam, s in sums.items()}
    mean = {c: sum(v.values()) / max(1, len(v)) for c, v in per_layer.items()}
    return max(lams, key=lambda lam: mean[str(lam)]), mean, per_layer


def _now(model):
    """Wall seconds after the device has finished its queued work (stage boundaries of the fit's timings)."""
    if model.device.type == "cuda":
        torch.cuda.synchronize(model.device)
    return time.perf_counter()


def fit(model, docs, splits, lambdas=LAMBDAS, held=None, out_dir=None, name=None, solver=None, center=True,
        save_stats=False, log=print, meta_extra=None, group=None, unitrms=False, kvfold=False, timings=None,
        lean=False):
    """Fit maps for every split. Returns {S: dict(projector, lambda_star, mean_read_cos, per_layer_read_cos,
    record)}; writes files when out_dir is given. unitrms: also the unit-RMS-target maps of the same capture,
    saved as <name>-sweep-s<S>-unitrms with the raw fit as its control <name>-sweep-s<S>-rawctl
    (results[S]["unitrms"]); kvfold: also the K/V fold (pre-RoPE [k | v] of every late attention layer straight
    from the unit-RMS boundary state), saved as <name>-kvfold-s<S> (results[S]["kvfold"]). timings: a dict that
    receives the stage seconds (capture_s with the Gram sums and their reduction; per split fit_s<S> for the solves
    over the lambda grid and select_s<S> for the held-out lambda choice). lean: solve, score and drop one lambda at a
    time (fit_select_lean; results[S]["maps"] then holds only the chosen lambda), for full-size models; with lean
    the solves and the scoring are timed together as fit_s<S>."""
    splits = sorted(int(s) for s in splits)
    name = name or model.cfg.name or "model"
    L = model.n_layers
    rows = sum(len(d["ids"]) for d in docs)
    out_dir = Path(out_dir) if out_dir else None
    raw_suffix = "-rawctl" if (unitrms or kvfold) else ""
    proj_path = (lambda S, sfx=raw_suffix: out_dir / f"{name}-sweep-s{S}{sfx}.safetensors") if out_dir else None
    if out_dir:
        out_dir.mkdir(parents=True, exist_ok=True)
        paths = [proj_path(S) for S in splits] + ([proj_path(S, "-unitrms") for S in splits] if unitrms else [])
        stale = stale_projectors(paths, rows)
        if stale:
            raise StaleProjector("fitted on another calibration list: " + ", ".join(f"{p} ({r})" for p, r in stale))
    solver = solver or ("cholesky" if model.device.type == "cuda" else "eigen")
    t_cap = _now(model)
    stats = capture(model, docs, splits, log=log, group=group, unitrms=unitrms, kvfold=kvfold)
    if timings is not None:
        timings["capture_s"] = _now(model) - t_cap
    extra = {k: stats.pop(k) for k in ("unitrms", "kvfold") if k in stats}
    results = {}
    for S in sorted(splits, reverse=True):
        t0 = time.time()
        state = stats[S].state()
        if out_dir and save_stats:
            more = {}
            if unitrms:
                u = extra["unitrms"][S].state()
                more["unitrms"] = dict(cy=u["cy"], sy=u["sy"], sxy=u["sxy"])
            if kvfold:
                more["kvfold"] = dict(extra["kvfold"][S].state(), sq={i: v.cpu() for i, v in
                                                                      extra["kvfold"][S].sq.items()})
            torch.save(dict(state, dtype="float64", docs=[d["name"] for d in docs], model=name, **more),
                       out_dir / f"{name}-s{S}.pt")
        t_fit = _now(model)
        if lean and held:
            del stats[S]                                  # the device sums are no longer needed (state is on host)
            best, mean, per_layer, maps = fit_select_lean(model, state, S, lambdas, held, solver, center)
            t_sel = _now(model)
        else:
            maps = fit_split(state, S, L, lambdas, solver, center, model.device)
            t_sel = _now(model)
            if held:
                best, mean, per_layer = select_lambda(model, held, S, maps, lambdas)
            else:
                best, mean, per_layer = lambdas[len(lambdas) // 2], {}, {}
        if timings is not None:
            timings[f"fit_s{S}"] = t_sel - t_fit
            if not (lean and held):
                timings[f"select_s{S}"] = _now(model) - t_sel
        if model.device.type == "cuda":
            torch.cuda.empty_cache()
        W = {i: maps[best][i][0].to(torch.bfloat16).cpu() for i in range(S, L)}
        B = {i: maps[best][i][1].to(torch.bfloat16).cpu() for i in range(S, L)}
        meta = dict(model=name, model_commit="", lam=best, rows=rows, taps=S, sweep=True, note="",
                    calib_exclude_sha256="", code_commit=prov.COMMIT_AT_START, code_dirty=prov.DIRTY_AT_START,
                    docs=len(docs), **(meta_extra or {}))
        proj = Projector(S, W, B, {k: str(v) for k, v in dict(meta, split=S).items()})
        record = dict(rows=rows, docs=len(docs), lambda_star=best, mean_read_cos=mean,
                      per_layer_read_cos=per_layer, solver=solver, center=center)
        write = out_dir is not None and (group is None or __import__("torch.distributed").distributed.get_rank(group) == 0)
        if write:
            path = proj_path(S)
            proj.save(path, meta)
            record.update(provenance=prov.provenance(name, dict(split=S, lambdas=list(lambdas), sweep_splits=splits,
                                                                held=[d["name"] for d in held or []])),
                          projector=str(path), projector_sha256=prov.sha256(path))
            prov.write_json(out_dir / f"fit-sweep-{name}-s{S}.json", record)
        if log:
            log(f"S={S}: lambda* {best} read cos {mean.get(str(best), float('nan')):.4f} "
                f"(identity {mean.get('identity', float('nan')):.4f}) in {time.time() - t0:.1f}s")
        results[S] = dict(projector=proj, lambda_star=best, mean_read_cos=mean, per_layer_read_cos=per_layer,
                          record=record, maps=maps)
        if unitrms:
            results[S]["unitrms"] = _fit_extra(model, extra["unitrms"][S].state(), S, lambdas, held, solver, center,
                                               "unitrms", name, rows, docs, meta, out_dir, proj_path, write, log)
        if kvfold:
            results[S]["kvfold"] = _fit_kvfold(model, extra["kvfold"][S], S, lambdas, held, name, rows, docs,
                                               meta, out_dir, write, log)
    return results


def _fit_extra(model, state, S, lambdas, held, solver, center, kind, name, rows, docs, meta, out_dir, proj_path,
               write, log):
    """The unit-RMS-target maps of split S: same grid and held-out selection as the raw fit."""
    L = model.n_layers
    maps = fit_split(state, S, L, lambdas, solver, center, model.device)
    best, mean, per_layer = (select_lambda(model, held, S, maps, lambdas) if held
                             else (lambdas[len(lambdas) // 2], {}, {}))
    W = {i: maps[best][i][0].to(torch.bfloat16).cpu() for i in range(S, L)}
    B = {i: maps[best][i][1].to(torch.bfloat16).cpu() for i in range(S, L)}
    m = dict(meta, lam=best, target="y / rms(y)")
    proj = Projector(S, W, B, {k: str(v) for k, v in dict(m, split=S).items()})
    record = dict(rows=rows, docs=len(docs), lambda_star=best, mean_read_cos=mean, per_layer_read_cos=per_layer,
                  target="y / rms(y)")
    if write:
        path = proj_path(S, "-unitrms")
        proj.save(path, m)
        record.update(projector=str(path), projector_sha256=prov.sha256(path))
        prov.write_json(out_dir / f"fit-sweep-{name}-s{S}-{kind}.json", record)
    if log:
        log(f"S={S} {kind}: lambda* {best} read cos {mean.get(str(best), float('nan')):.4f}")
    return dict(projector=proj, lambda_star=best, mean_read_cos=mean, record=record)


def _fit_kvfold(model, st, S, lambdas, held, name, rows, docs, meta, out_dir, write, log):
    """The K/V fold of split S: ridge from the unit-RMS boundary state to every late attention layer's pre-RoPE
    [k | v] (EigenFit: the outputs are narrower than the input), lambda by held-out K / V cosine."""
    from .projector import KVFold
    state = st.state()
    fit_ = EigenFit(state, center=True)
    maps = {lam: {} for lam in lambdas}
    for i in st.layers:
        for lam, wb in fit_.layer(i, lambdas).items():
            maps[lam][i] = wb
    best, mean, per_layer = (select_lambda_kv(model, held, S, maps, lambdas) if held
                             else (lambdas[len(lambdas) // 2], {}, {}))
    W = {i: maps[best][i][0].to(torch.bfloat16).cpu() for i in st.layers}
    B = {i: maps[best][i][1].to(torch.bfloat16).cpu() for i in st.layers}
    m = dict(meta, lam=best, target="pre-RoPE [k | v] from b / rms(b)")
    fold = KVFold(S, W, B, model.n_kv, model.eps, {k: str(v) for k, v in dict(m, split=S).items()})
    record = dict(rows=rows, docs=len(docs), lambda_star=best, mean_kv_cos=mean, per_layer_kv_cos=per_layer,
                  layers=st.layers)
    if write:
        path = out_dir / f"{name}-kvfold-s{S}.safetensors"
        fold.save(path, m)
        record.update(projector=str(path), projector_sha256=prov.sha256(path))
        prov.write_json(out_dir / f"fit-kvfold-{name}-s{S}.json", record)
    if log:
        log(f"S={S} kvfold: lambda* {best} K/V cos {mean.get(str(best), float('nan')):.4f}")
    return dict(projector=fold, lambda_star=best, mean_kv_cos=mean, record=record)
