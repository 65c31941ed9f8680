"""Impact corpus: per-row first-order fill impact of calibration windows, stored per model as NPZ windows with a
checksummed index, and reduced to token-class counts and impact sums (code/impact-corpus/aggregate_classes.py:1-130
role; the impact itself is engine/impact.py).

Corpus layout, per model directory:
  index.json   {"classes": CLASSES, "n_windows": k, "windows": [{"doc", "window", "file", "sha256", "P"}]}
  <file>.npz   "impact" [P] (signed first-order impact of each prefix row) and "cls" [P] (class ids into CLASSES)
Aggregation (per model, never pooled across models): row 0 of every window is excluded; impact is cast to float32
before abs, summed in float64 within a window and with math.fsum across windows; enrichment
E_c = (sum |impact| of class c / total) / (N_c / N). Provenance: the index's sha256 and the SHA-256 of the sorted
lowercase NPZ digests, one per LF-terminated ASCII line. Two models must cover the same document set.

Token classes (a piece is the decoded text of one token): special (the tokenizer's special ids), newline (contains
a line break), space (whitespace only), number (digits after an optional leading space), punct (punctuation or
symbols only), word-start / word-start-cap (a leading space, then letters starting lower / upper case),
word-piece / word-piece-cap (letters with no leading space, lower / upper first), mixed (anything else).
"""
from __future__ import annotations

import hashlib
import io
import json
import math
from pathlib import Path

import numpy as np

CLASSES = ("special", "newline", "space", "number", "punct", "word-start", "word-start-cap", "word-piece",
           "word-piece-cap", "mixed")
PROTECTED = ("word-start-cap", "word-piece-cap", "word-piece", "mixed")


def token_class(piece, special=False):
    """Class id of one token's decoded text."""
    if special:
        return CLASSES.index("special")
    if "\n" in piece or "\r" in piece:
        return CLASSES.index("newline")
    if piece == "" or piece.isspace():
        return CLASSES.index("space")
    lead = piece[0].isspace()
    body = piece.lstrip()
    if body.isdigit():
        return CLASSES.index("number")
    if all(not c.isalnum() and not c.isspace() for c in body):
        return CLASSES.index("punct")
    if body.isalpha():
        cap = body[0].isupper()
        if lead:
            return CLASSES.index("word-start-cap" if cap else "word-start")
        return CLASSES.index("word-piece-cap" if cap else "word-piece")
    return CLASSES.index("mixed")


def classes_of(tok, ids):
    special = set(getattr(tok, "all_special_ids", None) or
                  [x for x in (getattr(tok, "bos_token_id", None), getattr(tok, "eos_token_id", None)) if x is not None])
    return np.array([token_class(tok.decode([int(t)]), int(t) in special) for t in ids], dtype=np.int8)


def window_impact(model, ids, split, P, fill_x_of, scored):
    """Signed first-order impact [P] (float64) of every prefix row of one window: the filled cache's K/V against the
    exact late layers' (engine.impact), the loss being the NLL of the last `scored` tokens."""
    import torch
    from ..engine import impact as IM
    from ..engine.prefill import run_lower
    ids = torch.as_tensor(ids).to(model.device)
    n = ids.shape[0]
    hs, _ = run_lower(model, ids, [split])
    h = hs[split]
    rows = torch.arange(n - scored - 1, n - 1, device=model.device)
    targets = ids[n - scored:]
    if n - scored - 1 < P:
        raise ValueError(f"the {scored} scored tokens must lie in the exact tail (P = {P}, n = {n})")
    true, _ = IM.exact_late(model, h, split, P, rows, targets)
    kv, gdn = IM.fill_late(model, split, P, lambda i: fill_x_of(i, h[:P]))
    res, _ = IM.impact(model, split, h[P:], P, kv, true, gdn, rows - P, targets)
    return res["impact"].numpy()


class CorpusWriter:
    """Adds windows to one model's corpus directory; close() writes index.json."""

    def __init__(self, root, model):
        self.dir = Path(root) / model
        self.dir.mkdir(parents=True, exist_ok=True)
        self.windows = []

    def add(self, doc, window, impact, cls):
        impact, cls = np.asarray(impact), np.asarray(cls)
        if impact.shape != cls.shape or impact.ndim != 1:
            raise ValueError("impact and cls are one value per prefix row")
        name = hashlib.sha256(f"{doc}|{window}".encode()).hexdigest()[:20] + ".npz"
        buf = io.BytesIO()
        np.savez(buf, impact=impact.astype(np.float64), cls=cls.astype(np.int8))
        data = buf.getvalue()
        (self.dir / name).write_bytes(data)
        self.windows.append(dict(doc=str(doc), window=int(window), file=name,
                                 sha256=hashlib.sha256(data).hexdigest(), P=int(impact.shape[0])))

    def close(self):
        idx = dict(classes=list(CLASSES), n_windows=len(self.windows), windows=self.windows)
        (self.dir / "index.json").write_text(json.dumps(idx, indent=1))
        return self.dir / "index.json"


def digest_list(digests):
    return hashlib.sha256("".join(d + "\n" for d in sorted(digests)).encode("ascii")).hexdigest()


class CorpusError(ValueError):
    pass


def aggregate_model(root, model):
    mdir = Path(root) / model
    raw = (mdir / "index.json").read_bytes()
    index = json.loads(raw)
    if tuple(index["classes"]) != CLASSES:
        raise CorpusError("the corpus uses other class definitions")
    wins = sorted(index["windows"], key=lambda w: (w["doc"], w["window"]))
    if not wins or index["n_windows"] != len(wins):
        raise CorpusError("inconsistent window count")
    if len({w["file"] for w in wins}) != len(wins):
        raise CorpusError("a file is listed twice")
    counts = np.zeros(len(CLASSES), dtype=np.int64)
    per_class = [[] for _ in CLASSES]
    totals, digests, nbytes = [], [], 0
    for w in wins:
        rel = Path(w["file"])
        if rel.is_absolute() or ".." in rel.parts or rel.suffix != ".npz":
            raise CorpusError(f"{w['file']}: a relative NPZ file name is expected")
        data = (mdir / rel).read_bytes()
        dg = hashlib.sha256(data).hexdigest()
        if dg != w["sha256"]:
            raise CorpusError(f"{w['file']}: checksum differs from the index")
        digests.append(dg)
        nbytes += len(data)
        with np.load(io.BytesIO(data), allow_pickle=False) as z:
            imp, cls = z["impact"], z["cls"]
        if imp.shape != (w["P"],) or cls.shape != imp.shape:
            raise CorpusError(f"{w['file']}: rows disagree with P")
        a = np.abs(imp[1:].astype(np.float32)).astype(np.float64)
        c = cls[1:]
        if not np.issubdtype(c.dtype, np.integer) or (c < 0).any() or (c >= len(CLASSES)).any() \
                or not np.isfinite(a).all():
            raise CorpusError(f"{w['file']}: invalid class ids or non-finite impact")
        counts += np.bincount(c, minlength=len(CLASSES))
        totals.append(float(a.sum(dtype=np.float64)))
        for k in range(len(CLASSES)):
            per_class[k].append(float(a[c == k].sum(dtype=np.float64)))
    N, S = int(counts.sum()), math.fsum(totals)
    classes = {}
    for k, label in enumerate(CLASSES):
        s_c = math.fsum(per_class[k])
        e = (s_c / S) / (counts[k] / N) if counts[k] and S > 0 and N else None
        classes[label] = dict(N_c=int(counts[k]), sum_abs_impact=s_c, enrichment=e)
    return dict(n_documents=len({w["doc"] for w in wins}), n_windows=len(wins),
                totals=dict(N=N, sum_abs_impact=S), classes=classes,
                provenance=dict(index=f"{model}/index.json", index_sha256=hashlib.sha256(raw).hexdigest(),
                                npz_count=len(digests), npz_bytes=nbytes,
                                sorted_npz_sha256_list_sha256=digest_list(digests)))


def aggregate(root, models):
    docs = [{w["doc"] for w in json.loads((Path(root) / m / "index.json").read_text())["windows"]} for m in models]
    if any(d != docs[0] for d in docs[1:]):
        raise CorpusError("the models cover different document sets")
    per = {m: aggregate_model(root, m) for m in models}
    enr = [c["enrichment"] for r in per.values() for lab, c in r["classes"].items()
           if lab in PROTECTED and c["enrichment"] is not None]
    return dict(schema="impact-corpus-classes-v1",
                method=dict(quantity="absolute first-order impact", excluded_rows="row 0 of every window",
                            enrichment="E_c = (sum_abs_impact_c / sum_abs_impact_total) / (N_c / N)",
                            protected_classes=list(PROTECTED)),
                protected_range=[min(enr), max(enr)] if enr else None, models=per)


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="token-class counts and impact sums of an impact corpus")
    ap.add_argument("--corpus-root", required=True)
    ap.add_argument("--models", required=True, help="comma-separated model directories")
    ap.add_argument("--output", required=True)
    a = ap.parse_args(argv)
    res = aggregate(a.corpus_root, a.models.split(","))
    Path(a.output).write_text(json.dumps(res, indent=2, allow_nan=False) + "\n")
    return 0


if __name__ == "__main__":
    import sys
    sys.exit(main())
