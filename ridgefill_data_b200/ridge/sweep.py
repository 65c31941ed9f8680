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


def capture(model, docs, splits, device=None, log=print, group=None):
    """{S: RidgeStats} over the documents (forward_exact with a capture hook). With a process group the documents
    are split over the ranks (data parallel), every rank uses rank 0's shifts, and the fp64 sums are added over
    the ranks at the end (one reduction per statistic: each rank keeps its partial sums on the device until then)."""
    L, H = model.n_layers, model.hidden
    dev = device or model.device
    stats = {S: RidgeStats(S, range(S, L), H, dev) for S in splits}
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
                for S, st in stats.items():
                    if S <= i:
                        st.add_layer(i, h)
            model.forward_exact(torch.as_tensor(d["ids"]).to(model.device), hook=hook)
            if log and (j % 10 == 0 or j == len(docs) - 1):
                log(f"capture {j + 1}/{len(docs)} rows {int(stats[splits[0]].n)} ({time.time() - t0:.0f}s)")
    if group is not None:
        import torch.distributed as dist
        for st in stats.values():
            n = torch.tensor([st.n], dtype=torch.float64, device=st.sx.device)
            dist.all_reduce(n, group=group)
            st.n = float(n.item())
            for t in [st.sx, st.sxx] + list(st.sy.values()) + list(st.sxy.values()):
                dist.all_reduce(t, group=group)
    return stats


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


def fit(model, docs, splits, lambdas=LAMBDAS, held=None, out_dir=None, name=None, solver=None, center=True,
        save_stats=False, log=print, meta_extra=None, group=None):
    """Fit maps for every split. Returns {S: dict(projector, lambda_star, mean_read_cos, per_layer_read_cos,
    record)}; writes files when out_dir is given."""
    splits = sorted(int(s) for s in splits)
    name = name or model.cfg.name or "model"
    L = model.n_layers
    rows = sum(len(d["ids"]) for d in docs)
    out_dir = Path(out_dir) if out_dir else None
    proj_path = (lambda S: out_dir / f"{name}-sweep-s{S}.safetensors") if out_dir else None
    if out_dir:
        out_dir.mkdir(parents=True, exist_ok=True)
        stale = stale_projectors([proj_path(S) for S in splits], rows)
        if stale:
            raise StaleProjector("fitted on another calibration list: " + ", ".join(f"{p} ({r})" for p, r in stale))
    solver = solver or ("cholesky" if model.device.type == "cuda" else "eigen")
    stats = capture(model, docs, splits, log=log, group=group)
    results = {}
    for S in sorted(splits, reverse=True):
        t0 = time.time()
        state = stats[S].state()
        if out_dir and save_stats:
            torch.save(dict(state, dtype="float64", docs=[d["name"] for d in docs], model=name),
                       out_dir / f"{name}-s{S}.pt")
        maps = fit_split(state, S, L, lambdas, solver, center, model.device)
        if held:
            best, mean, per_layer = select_lambda(model, held, S, maps, lambdas)
        else:
            best, mean, per_layer = lambdas[len(lambdas) // 2], {}, {}
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
    return results
