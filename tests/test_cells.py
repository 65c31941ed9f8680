"""Evaluation cells: the reference's own battery cells (installed as data in baseline/_ref) through this framework's
cell checker, cell-to-config backend, arm-spec check and protocol gate, with the reference's cellcheck and
kvabackend run beside them as oracles; the TTFT runner (the speed cells' engine path) on a tiny model; preflight
refusals."""
import copy
import json
import sys
from pathlib import Path

import pytest
import torch

from ridgefill_data_b200.eval import backend as B
from ridgefill_data_b200.eval import cells as C

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
CELLS = sorted((REF / "finals" / "cells").glob("*.json"))
needs_ref = pytest.mark.skipif(not CELLS or not (REF / "protocol.json").exists(),
                               reason="baseline/_ref holds no reference cells")


def _ref_modules(monkeypatch):
    monkeypatch.setenv("KVA_REPO", str(REF))
    for p in (str(REF), str(REF / "finals" / "lib")):
        if p not in sys.path:
            sys.path.insert(0, p)
    import cellcheck
    import kvabackend
    return cellcheck, kvabackend


@needs_ref
def test_cells_check_like_the_reference(monkeypatch):
    cc, _ = _ref_modules(monkeypatch)
    schema = json.loads((REF / "finals" / "cell.schema.json").read_text())
    for f in CELLS:
        cell = json.loads(f.read_text())
        errs, warns = C.check(cell, schema)
        ref_errs = cc.validate(schema, cell, f.name)
        ref_sem, ref_warns = cc.semantic(cell) if not ref_errs else ([], [])
        assert errs == [] and len(ref_errs) + len(ref_sem) == 0, (f.name, errs)
        assert len(warns) == len(ref_warns), f.name
    base = json.loads(CELLS[0].read_text())
    broken = [("drop exact", lambda c: c["runs"][0]["arms"].remove("exact")),
              ("unknown field", lambda c: c.__setitem__("bogus", 1)),
              ("bad name", lambda c: c.__setitem__("name", "Bad Name")),
              ("duplicate run ids", lambda c: c["runs"].append(copy.deepcopy(c["runs"][0]))),
              ("wrong primary split", lambda c: c.__setitem__("split", "1/2")),
              ("tbd registration", lambda c: c.__setitem__("registration", "FINAL-TBD"))]
    for what, mutate in broken:
        cell = copy.deepcopy(base)
        mutate(cell)
        errs, warns = C.check(cell, schema)
        ref_errs = cc.validate(schema, cell, "x")
        ref_sem, ref_warns = cc.semantic(cell) if not ref_errs else ([], [])
        ours = [e.split(":")[0] for e in errs] if not ref_errs else None
        assert (len(errs) > 0) == (len(ref_errs) + len(ref_sem) > 0), what
        assert len(warns) == len(ref_warns), what
        if ref_sem:
            assert ours == [e.split(":")[0] for e in ref_sem], what
    with pytest.raises(C.SchemaError):
        C.validate({"type": "object", "oneOf": []}, {})


@needs_ref
def test_configs_equal_the_references(monkeypatch):
    _, kb = _ref_modules(monkeypatch)
    from ridgefill_data_b200.engine import protocol as P
    from ridgefill_data_b200.engine import spec as S
    p = P.load(REF / "protocol.json")
    for f in CELLS:
        cell = json.loads(f.read_text())
        ours = B.harness_configs(cell, p)
        if cell["kind"] == "speed":
            with pytest.raises(kb.HarnessGap):
                kb.harness_configs(cell)
            assert [s for _, s in ours] == ["ttft"] and ours[0][0]["ttft_lengths"] == list(B.TTFT_LENGTHS)
            continue
        theirs = kb.harness_configs(cell)
        assert [s for _, s in ours] == [s for _, s in theirs], f.name
        for (a, _), (b, _) in zip(ours, theirs):
            b = json.loads(json.dumps(b).replace("$KVA_PROJ_DIR", "$RF_PROJ_DIR").replace("$KVA_MODEL_DIR",
                                                                                          "$RF_MODEL_DIR"))
            assert {k: v for k, v in a.items() if k != "note"} == {k: v for k, v in b.items() if k != "note"}, f.name
            model = cell["model"]["name"]
            S.validate(a, p["models"][model]["layers"])


@needs_ref
def test_configs_pass_the_protocol_gate(tmp_path):
    from ridgefill_data_b200.engine import protocol as P
    p = P.load(REF / "protocol.json")
    for f in CELLS:
        cell = json.loads(f.read_text())
        ledger = tmp_path / f"{f.stem}.jsonl"
        ledger.write_text(json.dumps(dict(type="hypothesis", id=cell["registration"])) + "\n")
        for cfg, set_name in B.harness_configs(cell, p):
            if set_name == "ttft":
                continue
            src = (cfg["decode_from"] if set_name == "decode"
                   else "ruler" if cfg.get("multiturn_from") == "ruler" else set_name)
            P.validate(cfg, p=p, ledger_path=ledger, set_name=src)


@needs_ref
def test_preflight_refusals(tmp_path):
    from ridgefill_data_b200.engine import protocol as P
    p = P.load(REF / "protocol.json")
    cell = json.loads((REF / "finals" / "cells" / "llama-3.1-8b-instruct-nll.json").read_text())
    configs = B.harness_configs(cell, p)
    with pytest.raises(B.HarnessGap, match="RF_MODEL_DIR"):
        B.preflight(cell, configs, env={})
    env = dict(RF_MODEL_DIR=str(tmp_path), RF_PROJ_DIR=str(tmp_path))
    with pytest.raises(B.StaleProjector, match="does not exist"):
        B.preflight(cell, configs, env=env)
    from ridgefill_data_b200.ridge.projector import Projector
    f = cell["projector"]["files"][0]
    d = 8
    Projector(f["layer"], {i: torch.eye(d) for i in range(f["layer"], f["layer"] + 2)},
              {i: torch.zeros(d) for i in range(f["layer"], f["layer"] + 2)}).save(tmp_path / f["file"], dict(rows=5))
    with pytest.raises(B.StaleProjector, match="not the file the cell pins"):
        B.check_projector(tmp_path / f["file"], cell["projector"]["provenance"], f["sha256"])
    with pytest.raises(B.StaleProjector, match="rows"):
        B.check_projector(tmp_path / f["file"], cell["projector"]["provenance"])
    with pytest.raises(B.HarnessGap, match="DerivedManifestMismatch"):
        B.check_derived(dict(derived={"ruler-twokey": "0" * 64}), tmp_path)


def test_ttft_runner_on_a_tiny_model(tmp_path):
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.tiny import tiny_configs
    model = from_config(tiny_configs(8, 64)["qwen3.5-9b"], seed=0, device="cpu", dtype=torch.float32)
    cfg = dict(arms=[dict(name="identity-s4", split=4, tail=32, fill="identity"),
                     dict(name="nofill-s4", split=4, tail=32, fill="none"),
                     dict(name="pop-native-s6", split=6, fill="identity", tail_from="continuation")])
    n = B.run_ttft(cfg, tmp_path, model=model, repeats=2, lengths=[96, 160], log=lambda *_: None)
    assert n == 2
    rec = json.loads((tmp_path / "ttft-160.json").read_text())
    assert set(rec["runs"]) == {"exact", "identity-s4", "nofill-s4", "pop-native-s6"}
    assert rec["runs"]["identity-s4"]["P"] == 128 and rec["runs"]["pop-native-s6"]["P"] == 159
    assert all(len(r["ttft_ms"]) == 2 and r["median_ms"] > 0 for r in rec["runs"].values())
    assert rec["runs"]["exact"]["speedup_vs_exact"] == 1.0


@needs_ref
def test_registration_pins(tmp_path):
    from ridgefill_data_b200.engine import protocol as P
    from ridgefill_data_b200.release.ledger import Ledger
    p = P.load(REF / "protocol.json")
    cell = json.loads((REF / "finals" / "cells" / "qwen3-8b-ruler.json").read_text())
    pn = B.pins(cell, p)
    assert len(pn["config"]) == 3 and B.pins_of(B.pins_text(pn)) == pn
    led = Ledger(tmp_path / "ledger")
    path = tmp_path / "ledger" / "ledger.jsonl"
    assert "not a hypothesis id" in B.check_record(cell, p, path)[0]
    led.append(dict(type="hypothesis", id=cell["registration"], claim="claim text | " + B.pins_text(pn)))
    assert B.check_record(cell, p, path) == []
    changed = dict(cell, tail=2048)
    assert any(s.startswith("ConfigNotRegistered") for s in B.check_record(changed, p, path))
    led.append(dict(type="record", label=B.superseded_label(cell["registration"])))
    assert B.check_record(cell, p, path)[0].startswith("Superseded")
