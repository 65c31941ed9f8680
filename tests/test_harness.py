"""The research harness's evaluation sets on the CPU (tiny hybrid, character tokenizer, synthetic text): grade with
every arm option (proj / identity / none fills, pop-native's per-prompt tail, a qattn selector, reuse_fill,
tail_round), NIAH, multi-turn with repair arms, decode agreement, resume, the CLI on a harness-format config, and
the reference's own paper configs passing this framework's arm-spec validation."""
import json
import random

import pytest
import torch

from ridgefill_data_b200.eval import harness as H
from ridgefill_data_b200.eval import text as TX
from ridgefill_data_b200.eval.data import synthetic_maps
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.tiny import tiny_configs
from ridgefill_data_b200.ridge.projector import Projector

CFG = tiny_configs(8, 64)["qwen3.5-9b"]
TOK = TX.CharTokenizer()
WORDS = ["alpha", "beta", "gamma", "delta", "omega", "river", "stone", "cloud", "north", "amber", "7", "42"]


def _text(n, seed):
    r = random.Random(seed)
    return " ".join(r.choice(WORDS) for _ in range(n))


@pytest.fixture(scope="module")
def env(tmp_path_factory):
    tmp = tmp_path_factory.mktemp("harness")
    model = from_config(CFG, seed=0, device="cpu", dtype=torch.float32)
    W, B = synthetic_maps(CFG.hidden, 4, CFG.n_layers, "cpu", dtype=torch.float32)
    maps = tmp / "maps-s4.safetensors"
    Projector(4, W, B).save(maps, dict(model="tiny"))
    return tmp, model, str(maps)


def _grade_prompts():
    plan = [dict(name=f"g{j}", kind="prose", text=_text(260, j), short_start=300) for j in range(2)]
    return TX.grade_prompts(TOK, "raw", plan=plan, helps={})


def test_grade_arms(env):
    tmp, model, maps = env
    arms = [dict(name="rf", split=4, tail=600, fill="proj", projector=maps),
            dict(name="id", split=4, tail=600, fill="identity"),
            dict(name="nofill", split=4, tail=600, fill="none"),
            dict(name="pop", split=6, fill="identity", tail_from="continuation"),
            dict(name="qattn", split=4, tail=600, fill="proj", projector=maps,
                 select=dict(kind="qattn", budget=0.05)),
            dict(name="rf-again", split=4, tail=600, fill="proj", projector=maps, reuse_fill="rf"),
            dict(name="round", split=4, tail=600, fill="proj", projector=maps, tail_round=dict(base=600, block=128))]
    cfg = dict(name="t", arms=arms)
    out = tmp / "grade"
    h = H.Harness(model, TOK, cfg, "grade", out, log=lambda *_: None)
    prompts = _grade_prompts()
    assert h.run(prompts) == 2
    rec = json.loads((out / "g0.json").read_text())
    n = rec["n"]
    runs = rec["runs"]
    assert set(runs) == {"exact", "rf", "id", "nofill", "pop", "qattn", "rf-again", "round"}
    assert all(len(r["logprobs"]) == TX.SCORED for r in runs.values())
    assert runs["exact"]["P"] == 0 and runs["rf"]["P"] == n - 600
    assert runs["pop"]["P"] == n - H.KEEP and runs["pop"]["tail_from"] == "continuation"
    assert runs["rf-again"]["logprobs"] == runs["rf"]["logprobs"]
    assert runs["round"]["P"] == (n - 600) // 128 * 128
    assert runs["qattn"]["select"] == "qattn" and runs["qattn"]["n_rows"] == round(0.05 * n)
    assert runs["id"]["logprobs"] != runs["exact"]["logprobs"]
    assert "short" in rec and len(rec["short"]["logprobs"]) == TX.SCORED
    assert h.run(prompts) == 0                                   # resume: every arm complete


def test_refusals(env):
    tmp, model, maps = env
    bad = [[dict(name="a", split=4, tail=600, fill="proj", projector=maps, reuse_fill="zzz")],
           [dict(name="a", split=4, tail=600, fill="identity"), dict(name="b", split=4, tail=500, fill="identity",
                                                                      reuse_fill="a")],
           [dict(name="a", split=4, tail=100, fill="identity", tail_round=dict(base=100, block=64))],
           [dict(name="a", split=6, tail=100, fill="identity", tail_from="continuation")],
           [dict(name="a", split=6, fill="proj", projector=maps, tail=100)],               # maps of split 4
           [dict(name="a", split=4, tail=100, fill="identity", repair=0.5)]]              # repair off multiturn
    for arms in bad:
        with pytest.raises(H.EvalError):
            H.Harness(model, TOK, dict(name="t", arms=arms), "grade", tmp / "bad")
    with pytest.raises(H.EvalError):
        H.Harness(model, TOK, dict(name="t", arms=[dict(name="a", split=4, tail=9, fill="identity")]), "decode",
                  tmp / "bad")


def _mk4(n=900):
    corpus = {"prose": _text(4000, 9)}
    return TX.niah_prompts(TOK, "raw", variant="mk4", text_of=corpus, lengths=(n,), sources=("prose",))[:2]


def test_niah_and_multiturn(env):
    tmp, model, maps = env
    cfg = dict(name="t", niah_variant="mk4", multiturn_turns=2,
               arms=[dict(name="id", split=4, tail=300, fill="identity"),
                     dict(name="id-rep", split=4, tail=300, fill="identity", repair=1.0),
                     dict(name="id-repq", split=4, tail=300, fill="identity", repair=0.5, repair_by="question")])
    prompts = _mk4()
    h = H.Harness(model, TOK, dict(cfg, arms=cfg["arms"][:1]), "niah", tmp / "niah", log=lambda *_: None)
    h.run([dict(p, max_new=6) for p in prompts])
    rec = json.loads((tmp / "niah" / f"{prompts[0]['name']}.json").read_text())
    assert {"gen", "text", "correct", "needle_projected"} <= set(rec["runs"]["id"])
    hm = H.Harness(model, TOK, cfg, "multiturn", tmp / "mt", log=lambda *_: None)
    hm.run([dict(p, max_new=4) for p in prompts])
    rec = json.loads((tmp / "mt" / f"{prompts[0]['name']}.json").read_text())
    assert len(rec["turns"]) == 2 and set(rec["runs"]) == {"exact", "id", "id-rep", "id-repq"}
    for name, r in rec["runs"].items():
        assert [t["turn"] for t in r["turns"]] == [1, 2] and r["turns"][1]["new"] > 0
    assert rec["runs"]["id-rep"]["turn1_from"] == "id"                      # turn 1 shared with the base arm
    assert rec["runs"]["id-rep"]["turns"][0]["gen"] == rec["runs"]["id"]["turns"][0]["gen"]
    H_rows = rec["n"] + len(rec["runs"]["id"]["turns"][0]["gen"]) - 1
    assert rec["runs"]["id-rep"]["repair"]["rows"] == H_rows                 # r = 1: every cached row
    assert rec["runs"]["id-repq"]["repair"]["rows"] == round(0.5 * rec["runs"]["id"]["P"])


def test_decode_set(env, monkeypatch):
    tmp, model, maps = env
    cfg = dict(name="t", decode_from="grade", decode_steps=6,
               arms=[dict(name="rf", split=4, tail=300, fill="proj", projector=maps)])
    h = H.Harness(model, TOK, cfg, "decode", tmp / "dec", log=lambda *_: None)
    src = _grade_prompts()
    monkeypatch.setattr(TX, "grade_prompts", lambda tok, fmt, **kw: src)
    prompts, extra = H.set_prompts("decode", cfg, TOK, "tiny", {})
    assert extra["decode_steps"] == 6
    assert [len(q["ids"]) for q in prompts] == [len(q["ids"]) - TX.SCORED for q in src]
    h.run(prompts)
    rec = json.loads((tmp / "dec" / "g0.json").read_text())
    ex, rf = rec["runs"]["exact"], rec["runs"]["rf"]
    assert len(ex["gen"]) == 6 and len(rf["kl"]) == 6 and 0 <= rf["frac_identical"] <= 1
    assert rf["forced_top1_agree"] >= 0 and rec["n"] == len(_grade_prompts()[0]["ids"]) - TX.SCORED


def test_cli_on_harness_config(env, tmp_path, monkeypatch):
    _, _, maps = env
    from ridgefill_data_b200 import evaluate as E
    inputs = tmp_path / "inputs"
    inputs.mkdir()
    (inputs / "plan-grade.json").write_text(json.dumps(
        [dict(name="d0", kind="prose", text=_text(240, 3), short_start=200)]))
    monkeypatch.setattr(TX, "inputs_dir", lambda: inputs)
    monkeypatch.setenv("RF_CPU_DRYRUN", "1")
    cfg = dict(name="cli", model="tiny-llama", tokenizer="char", dtype="fp32", out=str(tmp_path / "res"),
               arms=[dict(name="id", split=4, tail=600, fill="identity")])
    path = tmp_path / "cfg.json"
    path.write_text(json.dumps(cfg))
    assert E.main([str(path), "grade"]) == 0
    rec = json.loads((tmp_path / "res" / "grade-cli" / "d0.json").read_text())
    assert set(rec["runs"]) == {"exact", "id"} and rec["provenance"][0]["config"]["set"] == "grade"
    with pytest.raises(SystemExit):
        E.main([str(path), "bogus"])


def test_reference_paper_configs_validate():
    """The reference's own paper configs (copied with its package into baseline/_ref) pass the arm-spec check."""
    import glob
    from pathlib import Path
    from ridgefill_data_b200.engine import spec as S
    root = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "configs" / "paper"
    files = sorted(glob.glob(str(root / "*.json")))
    if not files:
        pytest.skip("baseline/_ref holds no reference configs")
    for f in files:
        cfg = json.loads(Path(f).read_text())
        S.validate(cfg, 36 if "qwen3-8b" in cfg["model"] else 32)


def test_protocol_gate_agrees_with_reference(monkeypatch):
    """Both protocol gates (the reference's kva.protocol and engine/protocol.py) on the reference's paper configs:
    the same verdict and the same number of listed problems (the templates are refused until registered)."""
    import glob
    import sys
    from pathlib import Path
    from ridgefill_data_b200.engine import protocol as P
    from ridgefill_data_b200.utils.paths import expand
    ref_root = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    files = sorted(glob.glob(str(ref_root / "configs" / "paper" / "*.json")))
    if not files or not (ref_root / "protocol.json").exists():
        pytest.skip("baseline/_ref holds no reference configs")
    sys.path.insert(0, str(ref_root))
    from kva import paths as RPA
    from kva import protocol as RP
    monkeypatch.setenv("RF_PROTOCOL", str(ref_root / "protocol.json"))
    for f in files:
        raw = json.loads(Path(f).read_text())
        name = Path(f).name
        set_name = raw.get("decode_from") if name.startswith("decode") else "grade"
        verdicts = []
        for gate, cfg in ((RP.validate, RPA.expand(raw)), (P.validate, expand(raw))):
            try:
                gate(cfg, set_name=set_name)
                verdicts.append(("accepted", 0))
            except SystemExit as e:
                verdicts.append(("refused", str(e).count("\n  - ")))
        assert verdicts[0] == verdicts[1], (name, verdicts)
        assert verdicts[0][0] == "refused"


def test_map_files_checked_against_fit_records(tmp_path):
    """A map file named by a fit record (projector / projector_sha256) must hash to the recorded value."""
    from ridgefill_data_b200.utils.integrity import IntegrityError, recorded_sha256
    W, B = synthetic_maps(16, 2, 4, "cpu", dtype=torch.float32)
    path = tmp_path / "m-sweep-s2.safetensors"
    Projector(2, W, B).save(path, dict(model="m"))
    import hashlib
    sha = hashlib.sha256(path.read_bytes()).hexdigest()
    (tmp_path / "fit-sweep-m-s2.json").write_text(json.dumps(dict(projector=str(path), projector_sha256=sha)))
    assert recorded_sha256(path, tmp_path) == sha
    files = H.Files("cpu")
    assert files.projector(str(path)).sha256 == sha
    (tmp_path / "fit-sweep-m-s2.json").write_text(json.dumps(dict(projector=str(path), projector_sha256="0" * 64)))
    with pytest.raises(IntegrityError):
        H.Files("cpu").projector(str(path))


def test_tables_read_harness_records(env):
    """The grade records the harness writes feed the paired tables and the key-token readout directly (derived
    metrics nll / nll_novel / nll_key from the per-token log-probs)."""
    from ridgefill_data_b200.eval import keytok, tables as TB
    tmp, model, maps = env
    cfg = dict(name="t", keytoken_tail=600, arms=[dict(name="rf", split=4, tail=600, fill="proj", projector=maps),
                                                  dict(name="id", split=4, tail=600, fill="identity")])
    out = tmp / "grade-tables"
    H.Harness(model, TOK, cfg, "grade", out, log=lambda *_: None).run(_grade_prompts())
    recs = TB.load_records(out)
    rows = TB.paired_table(recs, "nll_novel", "exact", n_resamples=200)
    assert {r["arm"] for r in rows} == {"rf", "id"} and all(r["n"] == 2 for r in rows)
    r0 = recs[0]
    assert TB.metric_value(r0, "exact", "nll") == pytest.approx(-sum(r0["runs"]["exact"]["logprobs"]) / TX.SCORED)
    ro = keytok.readout(r0)
    assert set(ro) == {"rf", "id"} and ro["rf"]["all"]["n"] == TX.SCORED
    assert len(r0["tail_only"]["logprobs"]) == TX.SCORED
