"""Corpus overlap checks (code/kva/impact_corpus.py): word n-gram fingerprints, overlap counts against reference
sets, within-document repetition, near-duplicate rejection and the scored-window cut points of a document.

A gram is N = 50 consecutive whitespace-separated words of decoded text (JSON files contribute each string value on
its own). Each word gets a stable 64-bit id (the first 8 bytes of a sha256 under this module's domain tag), and a
gram's fingerprint is the polynomial sum of its word ids in powers of an odd 64-bit constant modulo 2^64, computed
for every window at once with numpy; reference sets of tens of millions of grams then fit in sorted uint64 arrays.
"""
from __future__ import annotations

import csv
from collections import Counter
import hashlib
import json
from pathlib import Path

import numpy as np

GRAM = 50
_MULT = np.uint64(0x9E3779B97F4A7C15)     # odd 64-bit constant (2^64 / golden ratio)
_TAG = b"ridgefill-b200/word-gram/v1\x00"
_ids = {}

FRACS = (0.5, 0.75, 1.0)                  # window ends as fractions of the document
MIN_CUT = 8192                            # the shortest window (tokens)
GAP = 1024                                # the least distance between two windows' ends


def _word_id(word):
    digest = hashlib.sha256(_TAG + word.encode("utf-8", "surrogatepass")).digest()
    return int.from_bytes(digest[:8], "big")


def word_ids(words):
    """Stable 64-bit ids [len(words)] (uint64), cached per distinct word."""
    ids = [_ids.get(w) for w in words]
    for i, v in enumerate(ids):
        if v is None:
            ids[i] = _ids.setdefault(words[i], _word_id(words[i]))
    return np.array(ids, dtype=np.uint64)


def grams(text, n=GRAM):
    """Fingerprints of every word n-gram of text, in order."""
    ids = word_ids(text.split())
    windows = len(ids) - n + 1
    if windows <= 0:
        return np.zeros(0, np.uint64)
    acc = np.zeros(windows, np.uint64)
    with np.errstate(over="ignore"):
        for offset in range(n):                     # Horner's rule over the window, all windows at once
            acc = acc * _MULT + ids[offset:offset + windows]
    return acc


def strings_of(obj):
    """Every string value of a parsed JSON object (keys excluded), depth first in document order."""
    stack = [obj]
    while stack:
        item = stack.pop()
        if isinstance(item, str):
            yield item
        elif isinstance(item, dict):
            stack.extend(reversed(list(item.values())))
        elif isinstance(item, list):
            stack.extend(reversed(item))


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
    """The grams of accepted documents, for exact and near-duplicate rejection within a corpus."""

    def __init__(self):
        self.owner = {}                      # gram -> first accepted document holding it

    def containment(self, g):
        """(the largest share of g's distinct grams found in a single accepted document, that document)."""
        distinct = np.unique(g).tolist()
        hits = Counter(d for d in map(self.owner.get, distinct) if d is not None)
        if not hits:
            return 0.0, None
        doc = max(hits, key=hits.get)         # the first document to reach the top count
        return hits[doc] / len(distinct), doc

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
