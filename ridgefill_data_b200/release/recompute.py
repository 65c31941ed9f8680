"""Recompute published numbers from evaluation records and print them as claim lines (the role of the reference's
per-claim recompute scripts, recompute/*.py, driven by recompute/run_all.sh and checked by recompute/gate.py).

A spec (JSON or YAML) lists claims; each names a folder of per-prompt records written by the evaluation CLI
({"name", "runs": {arm: {metric: value}}}) and what to print from it:

    claims:
      - id: S7.llama.ridgefill.nll      # kind "interval": <id>.delta / .ci_lo / .ci_hi (BCa, paired against ref)
        results: results/llama/nll
        metric: nll
        arm: ridgefill
        ref: exact
        kind: interval
        digits: 3
      - {id: S7.llama.n, results: results/llama/nll, metric: nll, arm: ridgefill, ref: exact, kind: n}
      - {id: S7.llama.exact.mean, results: results/llama/nll, metric: nll, arm: exact, kind: mean, digits: 4}
      - {id: S7.llama.ridgefill.p, results: ..., kind: p_holm, digits: 3}   # Holm over the arms listed in `arms`
      - {id: LB9.share, results: ..., metric: identical, arm: ridgefill, kind: share, digits: 1}  # 100 * mean

Intervals use the declared resample count and seed of eval/stats.py, so a rerun prints the same strings; paths are
relative to --root. `python -m ridgefill_data_b200.release.recompute SPEC [--root DIR] > claims.out`, then
`python -m ridgefill_data_b200.release.claims claims.out --claims claims.csv`.
"""
from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from ..eval import stats as ST
from ..eval import tables as TB
from .claims import Claims, fixed, signed

KINDS = ("interval", "n", "mean", "ref_mean", "delta", "p", "p_holm", "share", "count")


def load_spec(path):
    text = Path(path).read_text()
    if str(path).endswith((".yaml", ".yml")):
        import yaml
        spec = yaml.safe_load(text)
    else:
        spec = json.loads(text)
    items = spec["claims"] if isinstance(spec, dict) else spec
    for c in items:
        if c.get("kind", "interval") not in KINDS:
            raise ValueError(f"claim {c.get('id')}: unknown kind {c.get('kind')!r} (one of {KINDS})")
        for k in ("id", "results", "metric"):
            if k not in c:
                raise ValueError(f"claim {c.get('id')}: missing {k!r}")
    return items


def _values(records, metric, arm):
    out = {}
    for r in records:
        v = TB.metric_value(r, arm, metric)
        if v is not None:
            out[r.get("name")] = v
    return out


class Recompute:
    def __init__(self, root=".", claims=None):
        self.root = Path(root)
        self.claims = claims or Claims()
        self._records = {}
        self._tables = {}

    def records(self, folder):
        if folder not in self._records:
            path = self.root / folder
            if not path.is_dir():
                raise FileNotFoundError(f"missing input: {path}")
            self._records[folder] = TB.load_records(path)
        return self._records[folder]

    def table(self, c):
        arms = tuple(c.get("arms") or [c["arm"]])
        key = (c["results"], c["metric"], c.get("ref", "exact"), arms, c.get("upper"), c.get("lower"))
        if key not in self._tables:
            rows = TB.paired_table(self.records(c["results"]), c["metric"], c.get("ref", "exact"), list(arms),
                                   upper=c.get("upper"), lower=c.get("lower"))
            self._tables[key] = {r["arm"]: r for r in rows}
        return self._tables[key][c["arm"]]

    def one(self, c):
        kind, d = c.get("kind", "interval"), int(c.get("digits", 3))
        if kind in ("mean", "share", "count"):
            vals = _values(self.records(c["results"]), c["metric"], c["arm"])
            if kind == "count":
                return self.claims.add(c["id"], str(int(sum(vals.values()))))
            if not vals:
                raise ST.StatsError(f"claim {c['id']}: no finite {c['metric']} for {c['arm']}")
            m = float(np.mean(list(vals.values())))
            return self.claims.add(c["id"], fixed(100.0 * m if kind == "share" else m, d))
        row = self.table(c)
        if kind == "interval":
            return self.claims.interval(c["id"], row["delta"], row["lo"], row["hi"], d, sign=c.get("signed", True))
        if kind == "n":
            return self.claims.add(c["id"], str(row["n"]))
        if kind == "delta":
            return self.claims.add(c["id"], signed(row["delta"], d))
        return self.claims.add(c["id"], fixed(row[kind], d))

    def run(self, items):
        for c in items:
            self.one(c)
        return self.claims


def main(argv=None):
    ap = argparse.ArgumentParser(description="recompute claims from evaluation records")
    ap.add_argument("spec")
    ap.add_argument("--root", default=".")
    a = ap.parse_args(argv)
    Recompute(a.root, Claims(stream=sys.stdout)).run(load_spec(a.spec))
    return 0


if __name__ == "__main__":
    sys.exit(main())
