"""The locked test set builders against the reference's kva/locked.py (baseline/_ref) on one synthetic locked set
(manifest, RULER rows, LongBench rows and templates, long-prompt documents) and a character tokenizer: the prompts'
ids, needle spans, references, output budgets and continuation splits must be identical, so both harnesses score
the same rows."""
import sys
from pathlib import Path

import pytest

HERE = Path(__file__).resolve().parent
REF = HERE.parent / "baseline" / "_ref"
sys.path.insert(0, str(HERE))
from test_eval_sets import TOK, _write_set  # noqa: E402

from ridgefill_data_b200.eval import locked as LK  # noqa: E402

if (REF / "kva" / "locked.py").exists():
    sys.path.insert(0, str(REF))
    from kva import locked as RL
else:
    RL = None
pytestmark = pytest.mark.skipif(RL is None, reason="baseline/_ref not installed")

KEYS = ("name", "ids", "refs", "needles", "max_new", "metric", "task", "length", "cont_len", "split_char", "novel",
        "truncated", "source_sha256")


def _same(a, b):
    assert len(a) == len(b)
    for x, y in zip(a, b):
        for k in KEYS:
            if k in x or k in y:
                assert x.get(k) == y.get(k), (x.get("name"), k)


def _add_longbench(root):
    """Rows for every LongBench task the reference lists, its templates and budgets as the set's config files, and
    the manifest and frozen pin rewritten."""
    import hashlib
    import json
    import random
    r = random.Random(3)
    for task in RL.LONGBENCH_PROMPT:
        rows = [dict(context=" ".join(r.choice(["alpha", "beta", "gamma", "7"]) for _ in range(120)), input="which?",
                     answers=["alpha"], all_classes=["alpha", "beta"], length=120, dataset=task, _id=f"{task}{i}")
                for i in range(2)]
        (root / "longbench" / f"{task}.jsonl").write_text("\n".join(json.dumps(x) for x in rows) + "\n")
    (root / "longbench" / "dataset2prompt.json").write_text(json.dumps(RL.LONGBENCH_PROMPT))
    (root / "longbench" / "dataset2maxlen.json").write_text(json.dumps(RL.LONGBENCH_MAXLEN))
    files = sorted(p.relative_to(root).as_posix() for p in root.rglob("*")
                   if p.is_file() and p.name not in ("MANIFEST.tsv", "FROZEN.json"))
    lines = ["path\tsha256\tdomain/task"] + [f"{f}\t{hashlib.sha256((root / f).read_bytes()).hexdigest()}\t"
                                             f"{f.split('/')[0]}/x" for f in files]
    (root / "MANIFEST.tsv").write_text("\n".join(lines) + "\n")
    (root / "FROZEN.json").write_text(json.dumps(dict(
        manifest_sha256=hashlib.sha256((root / "MANIFEST.tsv").read_bytes()).hexdigest())))


def test_locked_builders_match_reference(tmp_path, monkeypatch):
    root = tmp_path / "locked"
    _write_set(root)
    _add_longbench(root)
    monkeypatch.setenv("RF_LOCKED_DIR", str(root))
    monkeypatch.setattr(RL, "LOCKED", root)
    man, rman = LK.manifest(), RL.manifest(root)
    assert man == rman
    tasks, lengths = ["niah_multikey_1", "niah_single_1"], [8192]
    for fmt in ("raw", "chat"):
        ours, _ = LK.ruler_prompts(TOK, fmt, man, tasks=tasks, lengths=lengths)
        ref, _ = RL.ruler_prompts(TOK, fmt, rman, tasks=tasks, lengths=lengths)
        _same(ours, ref)
        ours, _ = LK.longbench_prompts(TOK, fmt, man, max_len=100)
        ref, _ = RL.longbench_prompts(TOK, fmt, rman, 100)
        _same(sorted(ours, key=lambda q: q["name"]), sorted(ref, key=lambda q: q["name"]))
    ours, _ = LK.longppl_docs(TOK, man, "m")
    ref, _ = RL.longppl_docs(TOK, rman, "m", root=root)
    _same(ours, ref)
