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


def file_grams(path):
    """Unique fingerprints of a file: .txt as text, .json / .jsonl per decoded string value."""
    path = Path(path)
    raw = path.read_text(encoding="utf-8", errors="ignore")
    if path.suffix == ".json":
        parts = list(strings_of(json.loads(raw)))
    elif path.suffix == ".jsonl":
        parts = [s for line in raw.splitlines() if line.strip() for s in strings_of(json.loads(line))]
    else:
        parts = [raw]
    g = [grams(s) for s in parts]
    return np.unique(np.concatenate(g)) if g else np.zeros(0, np.uint64)


def reference(paths, texts=()):
    parts = [file_grams(p) for p in paths] + [grams(t) for t in texts]
    return np.unique(np.concatenate(parts)) if parts else np.zeros(0, np.uint64)


def shared(g, ref):
    """How many distinct fingerprints of g occur in the sorted array ref."""
    u = np.unique(g)
    if not len(u) or not len(ref):
        return 0
    i = np.minimum(np.searchsorted(ref, u), len(ref) - 1)
    return int((ref[i] == u).sum())


def self_repeat(g):
    """Share of a document's gram positions that repeat an earlier gram of the same document (boilerplate)."""
    return 1.0 - len(np.unique(g)) / len(g) if len(g) else 0.0


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
    cuts = []
    for f in sorted(fracs, reverse=True):
        c = max(min_cut, round(f * n))
        if c <= n and all(abs(c - k) >= gap for k in cuts):
            cuts.append(c)
    return sorted(cuts)


def read_tsv(path):
    with open(path, newline="") as f:
        return list(csv.DictReader(f, delimiter="\t"))


def write_tsv(path, rows, fields=None):
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=fields or list(rows[0]), delimiter="\t", extrasaction="ignore")
        w.writeheader()
        w.writerows(rows)


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
    for p in paths:
        p = Path(p)
        files = sorted(p.rglob("*")) if p.is_dir() else [p]
        for f in files:
            if f.is_file() and f.suffix in (".txt", ".json", ".jsonl"):
                raw = f.read_text(encoding="utf-8", errors="ignore")
                if f.suffix == ".json":
                    raw = "\n".join(strings_of(json.loads(raw)))
                elif f.suffix == ".jsonl":
                    raw = "\n".join(s for line in raw.splitlines() if line.strip() for s in strings_of(json.loads(line)))
                out[str(f)] = raw
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
