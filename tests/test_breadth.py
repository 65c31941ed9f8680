"""CPU tests of the evaluation and engine side modules: cost model, selectors, metrics, NIAH, multi-turn
repair, key tokens, canary, config validation, CLIs."""
import json

import pytest
import torch

from ridgefill_data_b200.engine import select as SEL
from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.eval import metrics as M
from ridgefill_data_b200.eval.cost import CostModel
from ridgefill_data_b200.models.config import PRESETS


def test_cost_model_27b():
    cm = CostModel(PRESETS["qwen3.8-27b"])
    n = 16384
    s = cm.speedup(n, "proj", split=32, tail=4096)
    assert 1.3 < s < 2.0
    assert cm.speedup(n, "identity", split=32, tail=4096) > s       # no projector: cheaper
    assert cm.exact(n) > cm.ridgefill(n, 32, 4096) > cm.skip(n, 32, 4096)
    e = cm.tail_budget(n, 32, 4096)
    assert cm.skip(n, 32, 4096 + e) >= cm.ridgefill(n, 32, 4096)
    assert cm.bypass(n, 32, 4096, 0) == pytest.approx(cm.ridgefill(n, 32, 4096), rel=1e-9)
    moe = CostModel(PRESETS["flash-next"])
    assert moe.speedup(16384, "proj", split=24, tail=2048) > 1.3


def test_selector_picks():
    score = torch.tensor([0.1, 5.0, 5.0, 0.3, 2.0], dtype=torch.float64)
    assert SEL.top_rows(score, 5, 2) == [1, 2]
    rows, overlap = SEL.blend_rows(score, torch.tensor([9., 0, 0, 8, 7], dtype=torch.float64), 5, 3, 1)
    assert len(rows) == 3 and 0 in rows
    a = SEL.random_rows("p", 100, 10)
    assert a == SEL.random_rows("p", 100, 10) and len(a) == 10
    assert SEL.ranges([1, 2, 3, 7, 9, 10]) == [[1, 4], [7, 8], [9, 11]]


class _Tok:
    """A byte-level toy tokenizer: one id per character."""

    def __init__(self, text):
        self.chars = sorted(set(text))
        self.added_tokens_decoder = {}

    def __len__(self):
        return len(self.chars)

    def convert_ids_to_tokens(self, ids):
        return [self.chars[i].replace(" ", "Ġ").replace("\n", "Ċ") for i in ids]

    def decode(self, ids):
        return "".join(self.chars[i] for i in ids)

    def encode(self, text):
        return [self.chars.index(c) for c in text]


def test_content_rules():
    text = "Call John Smith at 555-1234 or visit www.example.com, then run my_function_name now"
    tok = _Tok(text)
    ids = tok.encode(text)
    tb = SEL.token_bytes(tok)
    ds = SEL.digit_ids(tok)
    P = len(ids)
    dig = SEL.digits(ids, P, ds)
    assert all(text[r].isdigit() for r in dig) and len(dig) == 7
    rx = set(SEL.regex_rows(ids, P, ds, tb))
    j, sm = text.index("John"), text.index("Smith")
    assert set(range(j, j + 4)) | set(range(sm, sm + 5)) <= rx         # a two-word name
    vb = set(SEL.verbatim_rows(ids, P, ds, tb))
    assert set(range(text.index("www"), text.index(".com") + 4)) <= vb
    assert set(range(text.index("my_function_name"), text.index("my_function_name") + 16)) <= vb


def test_choose_with_matched_arms():
    arms = [Arm("dig", split=2, tail=10, fill="proj", meta=dict(select=dict(kind="band", lo=20, hi=30))),
            Arm("rnd", split=2, tail=10, fill="proj", meta=dict(select=dict(kind="random", match="dig"))),
            Arm("tm", split=2, tail=10, fill="proj", meta=dict(select=dict(kind="tail_match", match="dig")))]
    got = SEL.choose(arms, 100, list(range(100)), "prompt")
    assert got["dig"]["rows"] == list(range(70, 80))
    assert got["rnd"]["count"] == 10 and got["tm"]["extra_tail"] == 10


def test_metrics_known_values():
    assert M.string_match_all(["the answer is 42 and 7"], [["42", "7"]]) == 100.0
    assert M.string_match_part(["nothing"], [["42"]]) == 0.0
    assert M.qa_f1_score("The cat sat", "a cat sat down") == pytest.approx(0.8)
    assert M.code_sim_score("x = 1\n", "x = 1") == 1.0
    assert 0.0 < M.rouge_score("the cat sat on the mat.", "a cat sat on a mat.") < 1.0
    assert M.longbench_row("trec", "Location\nmore", ["Location"], ["Location", "Person"]) == 1.0


def test_niah_generator():
    from ridgefill_data_b200.eval.niah import niah_correct, niah_prompt
    p = niah_prompt(2048, 4096, 0.5, seed=3)
    s, e = p["needle_start"], p["needle_end"]
    assert abs(s / 2048 - 0.5) < 0.05 and torch.equal(p["ids"][s + 4:e], p["value"])
    assert niah_correct(p["value"].tolist() + [1, 2], p["value"]) and not niah_correct([1, 2, 3], p["value"])


def test_full_repair_restores_exact(tiny_llama):
    from ridgefill_data_b200.engine import multiturn as MT
    from ridgefill_data_b200.engine.prefill import finish, run_lower
    from ridgefill_data_b200.models.base import load
    path, _ = tiny_llama
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (80,), generator=torch.Generator().manual_seed(1))
    arm = Arm("identity", split=3, tail=20, fill="identity")
    hs, lower = run_lower(m, ids, [3])
    _, cache, P = finish(m, ids, hs[3], lower, arm, 1)
    _, exact = m.forward_exact(ids)
    MT.repair(m, cache, hs[3], 3, 80)
    for i in range(3, m.n_layers):
        assert torch.allclose(cache[i]["k"], exact[i]["k"], atol=1e-5)
    lg, _ = MT.extend(m, cache, [5, 6], 80)
    lr, _ = MT.extend(m, exact, [5, 6], 80)
    assert torch.allclose(lg, lr, atol=1e-4)


def test_keytok_readout():
    from ridgefill_data_b200.eval import keytok
    rec = dict(lp=dict(exact=[-1.0, -2.0, -0.5], arm=[-1.5, -2.0, -3.0]), tail_only=[-4.0, -2.1, -0.6],
               novel=[True, False, True])
    out = keytok.readout(rec)
    assert out["arm"]["key"] == dict(delta=0.5, n=1) and out["arm"]["all"]["n"] == 3 and "exact" not in out


def test_spec_validation():
    from ridgefill_data_b200.engine import spec
    good = dict(arms=[dict(name="ex", fill="exact"), dict(name="rf", split=4, tail=256, fill="proj", projector="x")])
    spec.validate(good, 8)
    for bad in (dict(arms=[dict(name="a", fill="proj", split=9, tail=4, projector="x")]),
                dict(arms=[dict(name="a", fill="bogus")]),
                dict(arms=[dict(name="a", fill="identity", split=2, tail=0)]),
                dict(arms=[dict(name="a", fill="exact", colour="red")])):
        with pytest.raises(spec.ConfigError):
            spec.validate(bad, 8)


def test_canary_record_then_check(tmp_path, tiny_qwen35):
    from ridgefill_data_b200.models.base import load
    from ridgefill_data_b200.utils import canary
    path, _ = tiny_qwen35
    m = load(path, dtype=torch.float32)
    assert canary.check(m, tmp_path, split=4) == "recorded"
    assert canary.check(m, tmp_path, split=4) == "ok (variant 0)"
    f = next(tmp_path.glob("canary-*.json"))
    rec = json.loads(f.read_text())
    rec["variants"][0]["exact"]["sha256"] = "0" * 64
    rec["variants"][0]["exact"]["values"][0] += 1e-3
    f.write_text(json.dumps(rec))
    assert canary.check(m, tmp_path, split=4, tol=1e-2) == "ok (variant 0)"        # within the tolerance
    with pytest.raises(canary.CanaryMismatch):
        canary.check(m, tmp_path, split=4)
    assert canary.check(m, tmp_path, split=4, mode="accept") == "accepted (variant 1)"
    assert canary.check(m, tmp_path, split=4) == "ok (variant 1)"
    assert canary.check(m, tmp_path, split=4, mode="reset") == "reset"
    assert len(json.loads(f.read_text())["variants"]) == 1


def test_fit_and_evaluate_cli(tmp_path):
    from ridgefill_data_b200 import evaluate, fit
    from ridgefill_data_b200.models.config import PRESETS
    import ridgefill_data_b200.models.config as C
    C.PRESETS["cli-tiny"] = PRESETS["tiny-llama"].replace(n_layers=4, hidden=64, n_heads=2, n_kv=1, head_dim=32,
                                                          intermediate=128, vocab=512, name="cli-tiny")
    try:
        assert fit.main(["cli-tiny", "2", "--docs", "4", "--doc-len", "64", "--held", "1", "--out", str(tmp_path),
                         "--backend", "torch", "--device", "cpu", "--dtype", "fp32"]) == 0
        proj = tmp_path / "cli-tiny-sweep-s2.safetensors"
        rec = json.loads((tmp_path / "fit-sweep-cli-tiny-s2.json").read_text())
        assert proj.exists() and rec["lambda_star"] in (1e-4, 3e-4, 1e-3, 3e-3, 0.01, 0.03, 0.1, 0.3, 1.0)
        cfg = dict(model="cli-tiny", backend="torch", device="cpu", dtype="fp32", keep=4, out=str(tmp_path / "res"),
                   prompts=dict(kind="zipf", lengths=[96], count=1),
                   arms=[dict(name="exact", fill="exact"),
                         dict(name="rf", split=2, tail=16, fill="proj", projector=str(proj))])
        (tmp_path / "cfg.json").write_text(json.dumps(cfg))
        assert evaluate.main([str(tmp_path / "cfg.json"), "quality"]) == 0
        out = json.loads(next((tmp_path / "res" / "quality").glob("*.json")).read_text())
        assert out["runs"]["exact"]["kl"] == pytest.approx(0.0, abs=1e-9) and out["runs"]["rf"]["kl"] > 0
    finally:
        del C.PRESETS["cli-tiny"]


def test_cost_model_matches_the_reference(tmp_path):
    """Every MAC rule against the reference's kva/compute.py (installed in baseline/_ref) on the same shapes."""
    import sys
    from pathlib import Path
    ref_root = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (ref_root / "kva" / "compute.py").exists():
        pytest.skip("baseline/_ref not installed")
    sys.path.insert(0, str(ref_root))
    from kva import compute as RC
    for name in ("qwen3.8-27b", "llama-3.1-8b", "qwen3-8b"):
        cfg = PRESETS[name]
        d = tmp_path / name
        d.mkdir()
        (d / "config.json").write_text(json.dumps(cfg.to_hf()))
        dm, cm = RC.Dims(d), CostModel(cfg)
        for n, split, tail in ((16384, cfg.n_layers // 2, 4096), (65536, 3 * cfg.n_layers // 8, 4096), (9000, 8, 512)):
            assert cm.exact(n) == RC.exact(dm, n)
            assert cm.ridgefill(n, split, tail) == RC.kva(dm, n, split, tail)
            assert cm.ridgefill(n, split, tail, projector=False) == RC.kva(dm, n, split, tail, projector=False)
            assert cm.skip(n, split, tail) == RC.skip(dm, n, split, tail)
            assert cm.tail_budget(n, split, tail) == RC.tail_budget(dm, n, split, tail)
            assert cm.swiftkv(n, split) == RC.swiftkv(dm, n, split)
            assert cm.qattn_select(n, split) == RC.qattn_select(dm, n, split)
            for kind, kw in (("qattn", dict(budget=0.1)), ("digits", dict(rows=300)), ("tail_match", dict(rows=256))):
                assert cm.bypass_arm(n, split, tail, kind, **kw) == RC.bypass_arm(dm, n, split, tail, kind, **kw)
            assert cm.repair(split, 5000) == RC.repair(dm, split, 5000)
            assert cm.repair_selected(split, 300, n - tail) == RC.repair_selected(dm, split, 300, n - tail)
            for fill in ("proj", "identity", "kvfold"):
                assert cm.speedup(n, fill, split=split, tail=tail) == pytest.approx(
                    RC.speedup(dm, n, fill, split=split, tail=tail), rel=1e-12)
