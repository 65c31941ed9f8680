"""More of the reference's helpers as oracles (baseline/_ref/kva): non-numeric NIAH scoring, the surprisal
predictor's rank statistics, key-token readouts, attention received mass and row statistics, and the derived RULER
sets (two-key, question-first) built from one synthetic locked set."""
import random
import sys
from pathlib import Path

import numpy as np
import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

HERE = Path(__file__).resolve().parent
REF = HERE.parent / "baseline" / "_ref"
if (REF / "kva").exists():
    sys.path.insert(0, str(REF))
    from kva import impact as RI
    from kva import keytok as RKT
    from kva import niahg as RNG
    from kva import pred as RP
else:
    RI = None
pytestmark = pytest.mark.skipif(RI is None, reason="baseline/_ref not installed")

from ridgefill_data_b200.engine import impact as IM  # noqa: E402
from ridgefill_data_b200.engine import pred as PR  # noqa: E402
from ridgefill_data_b200.eval import keytok as KT  # noqa: E402
from ridgefill_data_b200.eval import niahg as NG  # noqa: E402

PIECES = ["The", "answer", "is", "Maria", "Lopez", "0x3fa9", "get_user_id", "\"", "'", "*", "-", "—", "<think>",
          "</think>", "blue harbor", "Answer:", "the special password", ".", ",", "\n", "<|im_end|>"]
FAST = settings(max_examples=200, deadline=None, derandomize=True)


@FAST
@given(st.lists(st.sampled_from(PIECES), max_size=12).map(" ".join), st.sampled_from(NG.TYPES),
       st.sampled_from(["Maria Lopez", "0x3fa9", "get_user_id", "blue harbor", "The answer is blue."]),
       st.sampled_from(["raw", "chat"]))
def test_niahg_scoring(text, typ, value, fmt):
    assert NG.extract(text) == RNG.extract(text)
    assert NG.normalize(text, typ) == RNG.normalize(text, typ)
    assert NG.edit_distance(text, value) == RNG.edit_distance(text, value)
    assert NG.score(text, value, typ, fmt) == RNG.score(text, value, typ, fmt)


def test_predictor_rank_statistics():
    g = np.random.default_rng(2)
    a, b = torch.tensor(g.normal(size=200)), torch.tensor(g.normal(size=200))
    b[::7] = a[::7]                                        # ties and partial agreement
    assert PR.spearman(a, b) == pytest.approx(RP.spearman(a, b), abs=1e-12)
    torch.testing.assert_close(PR.ranks(a), RP.ranks(a))
    for frac in (0.05, 0.2, 0.5):
        assert PR.topk_recall(a, b, frac) == pytest.approx(RP.topk_recall(a, b, frac), abs=1e-12)
    counts = torch.tensor(g.integers(0, 50, 300))
    torch.testing.assert_close(PR.log_freq(counts), RP.log_freq(counts))


def test_key_token_readout():
    g = np.random.default_rng(3)
    rec = dict(name="p", runs={a: dict(logprobs=(-g.gamma(1.0, 1.0, 64)).tolist()) for a in ("exact", "rf", "id")},
               tail_only=dict(T=100, bos=[1], logprobs=(-g.gamma(1.0, 2.0, 64)).tolist()),
               novel=(g.random(64) < 0.7).tolist())
    ours, ref = KT.readout(rec), RKT.readout(rec)
    assert ours.keys() == ref.keys() == {"rf", "id"}
    for arm in ours:
        for k in ("all", "novel", "key"):
            a, b = ours[arm][k], ref[arm][k]
            assert a["n"] == b["n"]
            assert (a["delta"] is None and b["delta"] is None) or a["delta"] == pytest.approx(b["delta"], abs=1e-9)


def test_received_mass_and_row_stats():
    g = torch.Generator().manual_seed(4)
    q = torch.randn(4, 90, 16, generator=g)
    k = torch.randn(2, 90, 16, generator=g)
    for kw in (dict(), dict(rows_below=40), dict(rows_below=40, stride=3)):
        a, b = IM.received_mass(q, k, 0.25, **kw), RI.received_mass(q, k, 0.25, **kw)
        for x, y in zip(a if isinstance(a, tuple) else (a,), b if isinstance(b, tuple) else (b,)):
            torch.testing.assert_close(x, y, rtol=1e-9, atol=1e-9)
    for x, y in zip(IM.row_stats(q, k, 0.25, local=16), RI.row_stats(q, k, 0.25, local=16)):
        torch.testing.assert_close(x, y, rtol=1e-9, atol=1e-9)


@pytest.mark.parametrize("which", ["twokey", "qfirst"])
def test_derived_sets(tmp_path, monkeypatch, which):
    sys.path.insert(0, str(HERE))
    from test_eval_sets import TOK, _write_set
    from kva import derived as RD
    from kva import locked as RL
    from ridgefill_data_b200.eval import derived as DV
    from ridgefill_data_b200.eval import locked as LK
    import hashlib
    import json
    from test_eval_sets import _ruler_row
    root = tmp_path / "locked"
    _write_set(root)
    r = random.Random(11)
    for task in DV.QFIRST_TASKS:                       # every file both builders read: each task at each length
        for L in LK.RULER_LENGTHS:
            (root / f"ruler/{task}_{L}.jsonl").write_text("\n".join(json.dumps(_ruler_row(r, i)) for i in range(2))
                                                          + "\n")
    files = sorted(p.relative_to(root).as_posix() for p in root.rglob("*")
                   if p.is_file() and p.name not in ("MANIFEST.tsv", "FROZEN.json"))
    (root / "MANIFEST.tsv").write_text("\n".join(["path\tsha256\tdomain/task"] + [
        f"{f}\t{hashlib.sha256((root / f).read_bytes()).hexdigest()}\t{f.split('/')[0]}/x" for f in files]) + "\n")
    (root / "FROZEN.json").write_text(json.dumps(dict(
        manifest_sha256=hashlib.sha256((root / "MANIFEST.tsv").read_bytes()).hexdigest())))
    monkeypatch.setenv("RF_LOCKED_DIR", str(root))
    monkeypatch.setenv("RF_DERIVED_DIR", str(tmp_path / "derived"))
    monkeypatch.setattr(RL, "LOCKED", root)
    monkeypatch.setattr(RD, "DIR", tmp_path / "derived-ref")
    ours, ref = DV.build_manifest(which), RD.build_manifest(which)
    drop = ("builder", "rule")                          # who built it, in prose; the samples and pins are equal
    assert {k: v for k, v in ours.items() if k not in drop} == {k: v for k, v in ref.items() if k not in drop}
    for d in (tmp_path / "derived", tmp_path / "derived-ref"):   # each harness reads the other's manifest
        d.mkdir(exist_ok=True)
    (tmp_path / "derived" / f"ruler-{which}.json").write_text(RD.dumps(ref))
    (tmp_path / "derived-ref" / f"ruler-{which}.json").write_text(DV.dumps(ours))
    a, _ = DV.prompts(which, TOK, "raw", LK.manifest(), lengths=[8192, 16384])
    b, _ = RD.prompts(which, TOK, "raw", RL.manifest(root), lengths=[8192, 16384])
    assert [q["name"] for q in a] == [q["name"] for q in b]
    for x, y in zip(a, b):
        for key in ("ids", "refs", "needles", "max_new", "turn_plan", "asks"):
            assert x.get(key) == y.get(key), key


def test_first_order_impact_matches_reference():
    """Per-row first-order fill impact (exact late layers, filled caches, backward through the tail) against the
    reference's kva/impact.py on the same tiny hybrid model and identity fill."""
    sys.path.insert(0, str(REF.parent))
    import reference_arm as RA
    from ridgefill_data_b200.eval.data import uniform_prompt
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.tiny import tiny_configs
    from ridgefill_data_b200.engine.prefill import run_lower
    mods = RA.import_reference()
    RK = mods[2]
    cfg = tiny_configs(8, 64)["qwen3.5-9b"]
    ours = from_config(cfg, seed=0, device="cpu", dtype=torch.float32)
    ids = uniform_prompt(96, cfg.vocab, seed=5)
    split, P, scored = 4, 64, 16
    rows = torch.arange(96 - scored - 1, 96 - 1)
    tgt = ids[96 - scored:]
    oh, _ = run_lower(ours, ids, [split])
    ot, _ = IM.exact_late(ours, oh[split], split, P, rows, tgt)
    okv, ogdn = IM.fill_late(ours, split, P, lambda i: oh[split][:P])
    ores, oloss = IM.impact(ours, split, oh[split][P:], P, okv, ot, ogdn, rows - P, tgt)
    # the reference's model in fp32 on the same seeded weights
    rm = mods[1]
    import json as _json
    import tempfile
    from pathlib import Path as _P
    from ridgefill_data_b200.models.checkpoint import RandomSource
    tmp = _P(tempfile.mkdtemp())
    (tmp / "config.json").write_text(_json.dumps(cfg.to_hf()))
    stock = rm.Checkpoint
    rm.Checkpoint = lambda path: RandomSource(cfg, seed=0, std=0.02)
    try:
        rmod = rm.model_class(tmp)(tmp, device="cpu", dtype=torch.float32)
    finally:
        rm.Checkpoint = stock
    rh, _ = RK.run_lower(rmod, ids, [split])
    rt, _ = RI.exact_late(rmod, rh[split], split, P, rows, tgt)
    rkv, rgdn = RI.fill_late(rmod, split, P, lambda i: rh[split][:P])
    rres, rloss = RI.impact(rmod, split, rh[split][P:], P, rkv, rt, rgdn, rows - P, tgt)
    assert oloss == pytest.approx(rloss, rel=1e-6)
    for k in ("impact", "err", "grad_norm"):
        torch.testing.assert_close(ores[k], rres[k], rtol=1e-4, atol=1e-7)


def test_grade_and_niah_builders_match_reference(tmp_path, monkeypatch):
    """The graded prompts (plan file, novel-token masks, short references, raw / chat, BOS dropped) and the K20
    NIAH prompts (raw, chat, mk4 distractors; the generator's seeded draws) against the reference's kva/data.py on
    the same plan, corpus and character tokenizer."""
    import json
    sys.path.insert(0, str(HERE))
    from test_eval_sets import TOK
    from kva import data as RD
    from ridgefill_data_b200.eval import text as TX
    r = random.Random(4)
    words = ["alpha", "beta", "Gamma", "delta", "7", "omega", "river", "stone", "cloud", "north", ".", ","]
    body = lambda n: " ".join(r.choice(words) for _ in range(n))  # noqa: E731
    plan = [dict(name=f"g{j}", kind="prose", text=body(400), short_start=500) for j in range(3)]
    helps = dict(rows=[dict(name=p["name"], helps=j % 2 == 0) for j, p in enumerate(plan)])
    (tmp_path / "plan-grade.json").write_text(json.dumps(plan))
    (tmp_path / "swap_summary.json").write_text(json.dumps(helps))
    monkeypatch.setattr(RD, "INPUTS", tmp_path)
    for fmt, drop in (("raw", False), ("chat", False), ("raw", True)):
        ours = TX.grade_prompts(TOK, fmt, drop_bos=drop, plan=plan, helps={x["name"]: x["helps"] for x in helps["rows"]})
        ref = RD.grade_prompts(TOK, fmt, drop_bos=drop)
        assert len(ours) == len(ref)
        for a, b in zip(ours, ref):
            for k in ("name", "ids", "short_ids", "novel", "short_tail_match", "truncated", "helps16"):
                assert a[k] == b[k], (fmt, k)
    corpus = {s: body(40000) for s in TX.NIAH_SOURCES}
    monkeypatch.setattr(RD, "corpus", lambda: corpus)
    for fmt, variant in (("raw", None), ("chat", None), ("raw", "mk4")):
        ours = TX.niah_prompts(TOK, fmt, variant=variant, text_of=corpus)
        ref = RD.niah_prompts(TOK, fmt, variant)
        assert len(ours) == len(ref) == 60
        for a, b in zip(ours, ref):
            for k in ("name", "ids", "key", "value", "needle_start", "needle_end", "depth", "distractors"):
                assert a.get(k) == b.get(k), (fmt, variant, k)
