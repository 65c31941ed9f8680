"""Claim lines and the claims gate (recompute/common.py:52-74 formats, recompute/gate.py:1-45 gate).

A claim line is `<id>\\t<value>`: exactly one TAB, no newline, the value printed as the publication prints it. Lines
without a TAB are human commentary. The gate compares the claim lines of a run with a CSV of expected values
(columns `id`, `expected`, optional others) by exact string match and reports four kinds of failure: a mismatched
value, a claim the run did not print, a claim printed twice, and a printed claim the CSV does not list.

    python -m ridgefill_data_b200.release.claims OUTPUT --claims claims.csv      # exit 0 only when all match
"""
from __future__ import annotations

import argparse
import csv
import sys
from dataclasses import dataclass, field
from pathlib import Path


class ClaimError(ValueError):
    pass


def fixed(x, digits):
    """Fixed-point text; a value that rounds to zero has no sign ("0.00", never "-0.00")."""
    s = f"{float(x):.{digits}f}"
    return s[1:] if s.startswith("-") and float(s) == 0.0 else s


def signed(x, digits):
    """Fixed-point text with an explicit sign ("+0.012", "-0.004"); zero after rounding is unsigned."""
    s = fixed(abs(float(x)), digits)
    if float(s) == 0.0:
        return s
    return ("+" if float(x) > 0 else "-") + s


def line(key, value):
    """The claim line for (key, value); refuses a TAB in either or a newline in the value."""
    key, value = str(key), str(value)
    if not key or "\t" in key or "\n" in key or "\t" in value or "\n" in value:
        raise ClaimError(f"claim {key!r}: empty id, or a TAB / newline in the id or value")
    return f"{key}\t{value}"


class Claims:
    """Collects claim lines in order (and optionally echoes them to a stream)."""

    def __init__(self, stream=None):
        self.lines = []
        self.stream = stream

    def add(self, key, value):
        s = line(key, value)
        self.lines.append(s)
        if self.stream is not None:
            print(s, file=self.stream, flush=True)
        return s

    def interval(self, key, estimate, lo, hi, digits, sign=True):
        """Three claims: key.delta, key.ci_lo, key.ci_hi."""
        f = signed if sign else fixed
        for suffix, v in (("delta", estimate), ("ci_lo", lo), ("ci_hi", hi)):
            self.add(f"{key}.{suffix}", f(v, digits))

    def text(self):
        return "".join(s + "\n" for s in self.lines)


def read_expected(path):
    with open(path, newline="") as f:
        rows = list(csv.DictReader(f))
    if rows and ("id" not in rows[0] or "expected" not in rows[0]):
        raise ClaimError(f"{path}: needs the columns id and expected")
    out = {}
    for r in rows:
        if r["id"] in out:
            raise ClaimError(f"{path}: duplicate id {r['id']}")
        out[r["id"]] = r["expected"]
    return out


def parse_output(text):
    """[(key, value)] of the claim lines of a run's output; commentary lines (no TAB) are skipped."""
    out = []
    for s in text.splitlines():
        if "\t" in s:
            k, v = s.split("\t", 1)
            out.append((k, v))
    return out


@dataclass
class GateReport:
    total: int
    mismatched: dict = field(default_factory=dict)    # id -> (expected, got)
    missing: list = field(default_factory=list)
    twice: list = field(default_factory=list)
    unlisted: dict = field(default_factory=dict)      # id -> got

    @property
    def passed(self):
        return not (self.mismatched or self.missing or self.twice or self.unlisted)

    @property
    def matched(self):
        return self.total - len(self.mismatched) - len(self.missing)

    def lines(self):
        out = [f"MISMATCH {k}: expected {e!r}, got {g!r}" for k, (e, g) in self.mismatched.items()]
        out += [f"MISSING  {k}" for k in self.missing]
        out += [f"TWICE    {k}" for k in self.twice]
        out += [f"UNLISTED {k}: {g!r}" for k, g in self.unlisted.items()]
        out.append(f"gate: {self.matched} of {self.total} claims match; {len(self.mismatched)} mismatched, "
                   f"{len(self.missing)} missing, {len(self.twice)} printed twice, {len(self.unlisted)} unlisted")
        return out


def gate(expected, printed):
    """Compare {id: expected} with [(id, value)] printed by a run."""
    got, twice = {}, []
    for k, v in printed:
        if k in got and k not in twice:
            twice.append(k)
        got[k] = v
    rep = GateReport(total=len(expected), twice=twice)
    for k, e in expected.items():
        if k not in got:
            rep.missing.append(k)
        elif got[k] != e:
            rep.mismatched[k] = (e, got[k])
    rep.unlisted = {k: v for k, v in got.items() if k not in expected}
    return rep


def main(argv=None):
    ap = argparse.ArgumentParser(description="exact-match gate of claim lines against a claims CSV")
    ap.add_argument("output", type=Path, help="a run's output (claim lines: id<TAB>value)")
    ap.add_argument("--claims", type=Path, required=True)
    a = ap.parse_args(argv)
    for p in (a.output, a.claims):
        if not p.is_file():
            print(f"missing input: {p}", file=sys.stderr)
            return 2
    rep = gate(read_expected(a.claims), parse_output(a.output.read_text()))
    print("\n".join(rep.lines()))
    return 0 if rep.passed else 1


if __name__ == "__main__":
    sys.exit(main())
