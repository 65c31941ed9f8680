"""Corpus overlap checks (code/kva/impact_corpus.py): word n-gram fingerprints, overlap counts against reference
sets, within-document repetition, near-duplicate rejection and the scored-window cut points of a document.

A gram is N = 50 consecutive whitespace-separated words of decoded text (JSON files contribute each string value on
its own). Each word gets a stable 64-bit id (blake2b of its UTF-8 bytes), and a gram's fingerprint is a Rabin-Karp
style polynomial of its word ids modulo 2^64, computed for every window at once with numpy; reference sets of tens
of millions of grams then fit in sorted uint64 arrays searched with searchsorted.
"""
from __future__ import annotations

import csv
import hashlib
import json
from pathlib import Path

import numpy as np

GRAM = 50
_MULT = np.uint64(0x100000001B3)          # odd 64-bit multiplier (the FNV prime)
_ids = {}

FRACS = (0.5, 0.75, 1.0)                  # window ends as fractions of the document
MIN_CUT = 8192                            # the shortest window (tokens)
GAP = 1024                                # the least distance between two windows' ends


def word_ids(words):
    out = np.empty(len(words), np.uint64)
    for i, w in enumerate(words):
        v = _ids.get(w)
        if v is None:
            v = _ids[w] = int.from_bytes(hashlib.blake2b(w.encode("utf-8", "surrogatepass"), digest_size=8).digest(),
                                         "little")
        out[i] = v
    return out


def grams(text, n=GRAM):
    """Fingerprints of every word n-gram of text, in order."""
    w = word_ids(text.split())
    m = len(w) - n + 1
    if m <= 0:
        return np.zeros(0, np.uint64)
    h = np.zeros(m, np.uint64)
    with np.errstate(over="ignore"):
        for k in range(n):
            h = h * _MULT + w[k:k + m]
    return h


def strings_of(obj):
    """Every string value of a parsed JSON object (keys excluded)."""
    if isinstance(obj, str):
        yield obj
    elif isinstance(obj, dict):
        for v in obj.values():
            yield from strings_of(v)
    elif isinstance(obj, list):
        for v in obj:
            yield from strings_of(v)


def _pieces(path):
    """The texts of a file: a .txt whole, a .json / .jsonl file as its decoded string values."""
    path = Path(path)
    raw = path.read_text(encoding="utf-8", errors="ignore")
    if path.suffix == ".json":
        return list(strings_of(json.loads(raw)))
    if path.suffix == ".jsonl":
        return [piece for line in raw.splitlines() if line.strip() for piece in strings_of(json.loads(line))]
    return [raw]


def _union(arrays):
    arrays = list(arrays)
    return np.unique(np.concatenate(arrays)) if arrays else np.zeros(0, np.uint64)


def file_grams(path):
    """Distinct fingerprints of a file (each of its texts fingerprinted on its own)."""
    return _union(grams(piece) for piece in _pieces(path))


def reference(paths, texts=()):
    """Sorted distinct fingerprints of reference files and texts."""
    return _union([file_grams(p) for p in paths] + [grams(t) for t in texts])


def shared(g, ref):
    """How many distinct fingerprints of g occur in the sorted array ref."""
    distinct = np.unique(g)
    if distinct.size == 0 or ref.size == 0:
        return 0
    return int(np.isin(distinct, ref, assume_unique=True).sum())


def self_repeat(g):
    """Share of a document's gram positions that repeat an earlier gram of the same document (boilerplate)."""
    if len(g) == 0:
        return 0.0
    return 1.0 - np.unique(g).size / len(g)


class Seen:
    """Accepted documents' grams, for exact and near-duplicate rejection within a corpus."""

    def __init__(self):
        self.owner = {}

    def containment(self, g):
        """(largest share of g's distinct grams found in one accepted document, that document)."""
        counts = {}
        u = np.unique(g).tolist()
        for x in u:
            d = self.owner.get(x)
            if d is not None:
                counts[d] = counts.get(d, 0) + 1
        if not counts:
            return 0.0, None
        best = max(counts, key=counts.get)
        return counts[best] / len(u), best

    def add(self, name, g):
        for x in np.unique(g).tolist():
            self.owner.setdefault(x, name)


def cut_points(n, fracs=FRACS, min_cut=MIN_CUT, gap=GAP):
    """Window ends of a document of n tokens: each fraction of n raised to min_cut, kept when at least `gap` away
    from every end already kept (longest first, so the document's own end is always one). Ascending."""
    kept = []
    for frac in sorted(fracs, reverse=True):
        end = max(min_cut, round(frac * n))
        far_enough = min((abs(end - k) for k in kept), default=gap) >= gap
        if end <= n and far_enough:
            kept.append(end)
    return sorted(kept)


def read_tsv(path):
    with open(path, newline="") as f:
        return [dict(row) for row in csv.DictReader(f, dialect="excel-tab")]


def write_tsv(path, rows, fields=None):
    columns = list(fields) if fields else list(rows[0])
    with open(path, "w", newline="") as f:
        out = csv.DictWriter(f, columns, extrasaction="ignore", dialect="excel-tab")
        out.writeheader()
        out.writerows(rows)


def overlap_report(calib, evaluation, n=GRAM):
    """Calibration-vs-evaluation overlap (the calibration exclusion check): for every calibration document
    {name: text}, the number of its distinct word n-grams that also occur in any evaluation text, and the share of
    its grams. Returns rows sorted by shared count (largest first)."""
    ref = np.unique(np.concatenate([grams(t, n) for t in evaluation.values()])) if evaluation else np.zeros(0, np.uint64)
    rows = []
    for name, text in calib.items():
        g = grams(text, n)
        k = shared(g, ref)
        rows.append(dict(name=name, grams=int(len(np.unique(g))), shared=k,
                         share=k / max(1, len(np.unique(g)))))
    return sorted(rows, key=lambda r: (-r["shared"], r["name"]))


def _texts(paths):
    out = {}
    for p in map(Path, paths):
        for f in (sorted(p.rglob("*")) if p.is_dir() else [p]):
            if f.is_file() and f.suffix in (".txt", ".json", ".jsonl"):
                out[str(f)] = "\n".join(_pieces(f))
    return out


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="calibration-vs-evaluation word n-gram overlap")
    ap.add_argument("--calib", nargs="+", required=True, help="calibration files or directories")
    ap.add_argument("--eval", nargs="+", required=True, help="evaluation files or directories")
    ap.add_argument("--n", type=int, default=GRAM)
    ap.add_argument("--tsv")
    a = ap.parse_args(argv)
    rows = overlap_report(_texts(a.calib), _texts(a.eval), a.n)
    if a.tsv:
        write_tsv(a.tsv, rows)
    for r in rows:
        print(f"{r['shared']}\t{r['share']:.4f}\t{r['name']}")
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
