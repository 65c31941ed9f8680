"""Protocol checks on a synthetic protocol file and ledger: arm kinds and their templates, protocol / battery rows,
eras, the frozen gate, locked-set rules and the returned stamp."""
import json

import pytest

from ridgefill_data_b200.engine import protocol as PR

KINDS = ["exact", "noproj", "kva", "skip", "kva+st", "noproj+qattn10", "kva+qattn10", "kva+qblind10", "pop-native",
         "swiftkv", "swiftkv-native", "kvexact", "kva+kexact", "kva+ktail", "kva+random", "kva+tailmatch",
         "skip+tailbudget"]


def _protocol(tmp_path, phase="development", version="1.1.0"):
    p = dict(version=version, phase=phase, ledger="ledger.jsonl", tails=[1024, 4096], arms={k: "" for k in KINDS},
             outside_battery=["kva+kexact", "kva+ktail", "kva+random", "kva+tailmatch", "skip+tailbudget", "kvexact"],
             blind_splits={"hyb": 12}, banned_model_substrings=["banned"],
             sets=dict(locked=["ruler", "longbench", "long-prompts"]), ruler_max_new=dict(tasks={"vt": 10}),
             models=dict(dense=dict(layers=32, kind="dense", splits=[8, 12], pop_split=22, max_len=32768),
                         hyb=dict(layers=32, kind="hybrid", splits=[8, 12], pop_split=22),
                         base=dict(layers=32, kind="dense", splits=[16], baseline_only=True)))
    path = tmp_path / "protocol.json"
    path.write_text(json.dumps(p))
    (tmp_path / "ledger.jsonl").write_text(json.dumps(dict(type="hypothesis", id="H1")) + "\n" +
                                           json.dumps(dict(type="hypothesis", id="FINAL-A")) + "\n")
    return PR.load(path)


def test_kinds_roundtrip_through_templates(tmp_path):
    p = _protocol(tmp_path)
    for model in ("dense", "hyb"):
        for kind in KINDS:
            if kind in ("exact", "swiftkv", "swiftkv-native"):
                continue
            spec = PR.template(kind, model, 12, None if kind in PR.TAILLESS else 1024, p)
            assert PR.arm_kind(spec, p) == kind, (model, kind, spec)
    assert PR.arm_kind(dict(name="x", split=8, tail=1024, fill="proj", projector="other.safetensors")) is None
    assert PR.arm_kind(dict(name="x", split=8, tail=1024, fill="identity", bogus=1)) is None
    assert PR.arm_kind(dict(name="x", split=8, fill="swiftkv_native")) == "swiftkv-native"


def test_protocol_and_battery_rows(tmp_path):
    p = _protocol(tmp_path)
    kva = PR.template("kva", "dense", 12, 1024, p)
    assert PR.protocol_row(kva, "dense", p) and PR.battery_row(kva, "dense", p)
    assert not PR.protocol_row(dict(kva, tail=777), "dense", p)
    assert not PR.protocol_row(PR.template("kva+st", "dense", 12, 1024, p), "dense", p)       # hybrids only
    assert PR.protocol_row(PR.template("kva+st", "hyb", 12, 1024, p), "hyb", p)
    assert not PR.protocol_row(PR.template("kva+qblind10", "hyb", 8, 1024, p), "hyb", p)   # blind split only
    splice = PR.template("kva+kexact", "dense", 8, 1024, p)
    assert PR.protocol_row(splice, "dense", p) and not PR.battery_row(splice, "dense", p)
    assert PR.protocol_row(PR.template("pop-native", "dense", 22, None, p), "dense", p)
    assert PR.protocol_row(PR.template("swiftkv-native", "base", 16, None, p), "base", p)
    cells = PR.battery_cells("hyb", p)
    assert (12, 1024, "kva+qblind10") in cells and (8, 1024, "kva+qblind10") not in cells
    assert (22, None, "pop-native") in cells


def test_validate(tmp_path):
    p = _protocol(tmp_path)
    ledger = tmp_path / "ledger.jsonl"
    arms = [PR.template("kva+qattn10", "dense", 12, 1024, p), PR.template("kva+random", "dense", 12, 1024, p)]
    arms[1]["select"]["match"] = arms[0]["name"]
    cfg = dict(protocol="1.1", model="/models/dense", registration=["H1"], arms=arms)
    stamp = PR.validate(cfg, p, ledger, archive=tmp_path, env={})
    assert stamp["battery"] and stamp["version"] == "1.1.0" and len(stamp["sha256"]) == 64
    bad = dict(cfg, arms=arms[1:])                                 # control without its rows arm
    with pytest.raises(SystemExit, match="outside the protocol"):
        PR.validate(bad, p, ledger, archive=tmp_path, env={})
    assert PR.validate(dict(bad, exploratory="probe"), p, ledger, archive=tmp_path, env={})["battery"] is False
    with pytest.raises(SystemExit, match="not in the ledger"):
        PR.validate(dict(cfg, registration=["H9"]), p, ledger, archive=tmp_path, env={})
    with pytest.raises(SystemExit, match="finals only"):
        PR.validate(dict(cfg, ruler_max_len=8192), p, ledger, archive=tmp_path, env={}, set_name="ruler")
    ok = PR.validate(dict(cfg, registration=["FINAL-A"], ruler_max_len=8192), p, ledger, archive=tmp_path, env={},
                     set_name="ruler")
    assert ok["registration"] == ["FINAL-A"]
    with pytest.raises(SystemExit, match="neither the current"):
        PR.validate(dict(cfg, protocol="0.9"), p, ledger, archive=tmp_path, env={})
    with pytest.raises(SystemExit, match="banned"):
        PR.validate(dict(cfg, model="/m/banned-x"), p, ledger, archive=tmp_path, env={})
    with pytest.raises(SystemExit, match="DETERMINISTIC"):
        PR.validate(cfg, p, ledger, archive=tmp_path, env={"RF_DETERMINISTIC": "0"})


def test_eras_and_frozen_gate(tmp_path):
    p = _protocol(tmp_path)
    arch = tmp_path / "arch"
    arch.mkdir()
    old = dict(json.loads((tmp_path / "protocol.json").read_text()), version="1.0.3")
    (arch / "protocol-1.0.3.json").write_text(json.dumps(old))
    (arch / "protocol-1.0.1.json").write_text(json.dumps(dict(old, version="1.0.1")))
    assert PR.era("1.0", p, arch)["version"] == "1.0.3"
    assert PR.era("1.1.7", p, arch) is p
    frozen = _protocol(tmp_path, phase="frozen")
    assert PR.frozen_gate(["H1"], frozen) and not PR.frozen_gate(["FINAL-A"], frozen)
    with pytest.raises(SystemExit):
        PR.phase(dict(version="x", phase="odd"))
