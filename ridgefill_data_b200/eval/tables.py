"""Result tables from the evaluation CLI's per-prompt records (the role of code/finals/tables.py): for every arm,
the mean of a metric and its paired difference to a reference arm with a BCa interval (eval/stats.py), the
two-sided p-value by interval inversion, Holm-adjusted over the table's arms, optionally a non-inferiority verdict
against a declared margin; rendered as Markdown or LaTeX.

    python -m ridgefill_data_b200.eval.tables RESULTS/TASK --metric nll --ref exact [--latex] [--upper 0.01]

Records are the JSON files evaluate.py writes (one per prompt: {"name", "runs": {arm: {metric: value}}}); only
prompts where every arm and the reference hold a finite value enter (the pairing unit), and the table says how many.
"""
from __future__ import annotations

import argparse
import json
import math
from pathlib import Path

import numpy as np

from . import stats as ST


def load_records(directory):
    return [json.loads(p.read_text()) for p in sorted(Path(directory).glob("*.json"))]


DERIVED = ("nll", "nll_novel", "nll_key", "correct", "turn2_correct", "turn1_correct")


def metric_value(rec, arm, metric, threshold=2.0):
    """One arm's value of `metric` on one record: a scalar field of the run, or a metric derived from the
    evaluation record's fields: nll (mean -logprob over the scored tokens), nll_novel (the novel-token mask of a
    graded prompt), nll_key (key tokens: exact log-prob above the tail-only one by more than `threshold` nats),
    correct / turn1_correct / turn2_correct (0 / 1). None when the record does not hold it."""
    run = rec.get("runs", {}).get(arm)
    if run is None:
        return None
    v = run.get(metric)
    if isinstance(v, bool):
        return float(v)
    if isinstance(v, (int, float)):
        return float(v) if math.isfinite(float(v)) else None
    lp = run.get("logprobs")
    if metric == "nll" and lp:
        return -sum(lp) / len(lp)
    if metric == "nll_novel" and lp and "novel" in rec:
        xs = [-x for x, m in zip(lp, rec["novel"]) if m]
        return sum(xs) / len(xs) if xs else None
    if metric == "nll_key" and lp and "tail_only" in rec and "exact" in rec["runs"]:
        tail = rec["tail_only"]["logprobs"] if isinstance(rec["tail_only"], dict) else rec["tail_only"]
        ex = rec["runs"]["exact"]["logprobs"]
        xs = [-x for x, e, t in zip(lp, ex, tail) if e - t > threshold]
        return sum(xs) / len(xs) if xs else None
    if metric in ("turn1_correct", "turn2_correct") and "turns" in run:
        k = int(metric[4]) - 1
        return float(run["turns"][k]["correct"]) if len(run["turns"]) > k else None
    return None


def paired_table(records, metric, ref, arms=None, n_resamples=ST.N_RESAMPLES, upper=None, lower=None):
    """[{arm, n, mean, ref_mean, delta, lo, hi, p, p_holm, noninferior}] over the prompts where every arm has the
    metric."""
    arms = arms or sorted({a for r in records for a in r.get("runs", {})} - {ref})
    rows, units = [], []
    for r in records:
        vals = {a: metric_value(r, a, metric) for a in arms + [ref]}
        if all(v is not None for v in vals.values()):
            units.append((r.get("name"), vals))
    if len(units) < 2:
        raise ST.StatsError(f"{metric}: {len(units)} complete prompts; at least 2 needed")
    ref_vals = np.array([v[ref] for _, v in units])
    pvals = {}
    for a in arms:
        x = np.array([v[a] for _, v in units])
        d = x - ref_vals
        res = ST.bca(d, n_resamples=n_resamples)
        row = dict(arm=a, n=len(units), mean=float(x.mean()), ref_mean=float(ref_vals.mean()), delta=res.estimate,
                   lo=res.lo, hi=res.hi, p=ST.pvalue(res), degenerate=res.degenerate)
        if upper is not None or lower is not None:
            ni = ST.noninferiority(d, upper=upper, lower=lower, n_resamples=n_resamples)
            row.update(noninferior=ni.passed, ni_bound=ni.hi if upper is not None else ni.lo)
        rows.append(row)
        pvals[a] = row["p"]
    adj = ST.holm(pvals)
    for row in rows:
        row["p_holm"] = adj[row["arm"]]
    return rows


def _fmt(x, digits=4):
    return "-" if x is None else f"{x:.{digits}f}"


def markdown(rows, metric, ref):
    head = f"| arm | n | {metric} | {ref} | delta | 95% BCa | p (Holm) |"
    if any("noninferior" in r for r in rows):
        head += " non-inferior |"
    lines = [head, "|" + "---|" * (head.count("|") - 1)]
    for r in rows:
        line = (f"| {r['arm']} | {r['n']} | {_fmt(r['mean'])} | {_fmt(r['ref_mean'])} | {_fmt(r['delta'])} | "
                f"[{_fmt(r['lo'])}, {_fmt(r['hi'])}] | {_fmt(r['p_holm'], 3)} |")
        if "noninferior" in r:
            line += f" {'yes' if r['noninferior'] else 'no'} |"
        lines.append(line)
    return "\n".join(lines)


def latex(rows, metric, ref):
    ni = any("noninferior" in r for r in rows)
    cols = "lrrrrrr" + ("c" if ni else "")
    esc = lambda s: str(s).replace("_", "\\_").replace("%", "\\%")  # noqa: E731
    out = [f"\\begin{{tabular}}{{{cols}}}", "\\toprule",
           f"arm & $n$ & {esc(metric)} & {esc(ref)} & $\\Delta$ & 95\\% BCa & $p_\\text{{Holm}}$"
           + (" & NI" if ni else "") + " \\\\", "\\midrule"]
    for r in rows:
        line = (f"{esc(r['arm'])} & {r['n']} & {_fmt(r['mean'])} & {_fmt(r['ref_mean'])} & {_fmt(r['delta'])} & "
                f"[{_fmt(r['lo'])}, {_fmt(r['hi'])}] & {_fmt(r['p_holm'], 3)}")
        if ni:
            line += " & " + ("\\checkmark" if r.get("noninferior") else "--")
        out.append(line + " \\\\")
    out += ["\\bottomrule", "\\end{tabular}"]
    return "\n".join(out)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("results")
    ap.add_argument("--metric", required=True)
    ap.add_argument("--ref", default="exact")
    ap.add_argument("--arms")
    ap.add_argument("--latex", action="store_true")
    ap.add_argument("--upper", type=float)
    ap.add_argument("--lower", type=float)
    ap.add_argument("--resamples", type=int, default=ST.N_RESAMPLES)
    a = ap.parse_args(argv)
    rows = paired_table(load_records(a.results), a.metric, a.ref, a.arms.split(",") if a.arms else None,
                        a.resamples, a.upper, a.lower)
    print(latex(rows, a.metric, a.ref) if a.latex else markdown(rows, a.metric, a.ref))
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
