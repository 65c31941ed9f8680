"""Research-protocol checks of a run config before any GPU work (code/kva/protocol.py:1-347).

The protocol file (protocol.json: version, phase, ledger, models {name: layers, kind, splits, pop_split,
baseline_only, max_len, niah_format}, tails, arms {kind: description}, outside_battery, blind_splits, sets,
banned_model_substrings, ruler_max_new) decides which arms are protocol rows. A config must name the protocol
version it runs under (checked under that version's era: the current file for its major.minor, else the archived
protocol-<version>.json of that major.minor), the ledger hypotheses it serves, and the model; every arm must be a
protocol row, or the config states an "exploratory" reason. A frozen protocol refuses runs without a FINAL-
registration; the locked sets run only as declared finals under the current protocol.

Arm kinds are named from an arm spec's structure; the names are the protocol file's identifiers:
  base      fill identity -> noproj, proj (a sweep projector) -> kva, none -> skip, swiftkv -> swiftkv
  +rows     select == a named question-window selector (qattn5 / qblind5 / qattn10 / qblind10)
  +control  select {kind: random | tail_match, match: <rows arm>} -> +random / +tailmatch
  kva+st, kva+kexact / kva+vexact (exact_part), kva+ktail / kva+vtail (rescale), kvexact (fill oracle, or by_type
  attention oracle + GDN proj), pop-native (tail_from continuation, identity), swiftkv-native, skip+tailbudget
validate() returns the provenance stamp {version, sha256, registration, battery, exploratory_arms, exploratory}.
"""
from __future__ import annotations

import hashlib
import json
import os
import re
from pathlib import Path

from ..utils.paths import REPO

FINAL = "FINAL-"
PHASES = ("development", "frozen")
ARM_KEYS = {"name", "split", "tail", "fill", "projector", "sets", "select", "st", "reuse_fill", "tail_from",
            "exact_part", "fill_by_type", "rescale", "rescale_skip_last"}
ROW_SELECTORS = {"qattn5": {"kind": "qattn", "budget": 0.05},
                 "qblind5": {"kind": "qattn", "budget": 0.05, "window": "prefix"},
                 "qattn10": {"kind": "qattn", "budget": 0.1},
                 "qblind10": {"kind": "qattn", "budget": 0.1, "window": "prefix"}}
CONTROLS = {"random": "random", "tail_match": "tailmatch"}
BASE_OF_FILL = {"identity": "noproj", "proj": "kva", "none": "skip", "swiftkv": "swiftkv"}
SWEEP_MAP = re.compile(r"-sweep-s\d+\.safetensors$")
KVEXACT_HYBRID = {"attention": "oracle", "gdn": "proj"}
TAILLESS = ("pop-native", "swiftkv-native")
LOCKED_SETS = {"ruler": "ruler", "longbench": "longbench", "longppl": "long-prompts"}
CAPS = {"ruler": "ruler_max_len", "longbench": "longbench_max_len", "longppl": "longppl_max_len"}


class ProtocolError(SystemExit):
    pass


def protocol_file():
    return Path(os.environ.get("RF_PROTOCOL", REPO / "protocol.json"))


def load(path=None):
    raw = Path(path or protocol_file()).read_bytes()
    p = json.loads(raw)
    p["sha256"] = hashlib.sha256(raw).hexdigest()
    return p


def minor(version):
    return ".".join(str(version).split(".")[:2])


def archived(archive):
    """{major.minor: path} of the highest-patch protocol-<x.y.z>.json per minor in `archive`."""
    best = {}
    for f in Path(archive).glob("protocol-*.json"):
        v = f.name[len("protocol-"):-len(".json")]
        if re.fullmatch(r"\d+\.\d+\.\d+", v):
            key = tuple(int(x) for x in v.split("."))
            if minor(v) not in best or key > best[minor(v)][0]:
                best[minor(v)] = (key, f)
    return {k: f for k, (_, f) in best.items()}


def era(version, current, archive):
    if minor(version) == minor(current["version"]):
        return current
    path = archived(archive).get(minor(version))
    return load(path) if path else None


def phase(p):
    ph = p.get("phase", "development")
    if ph not in PHASES:
        raise ProtocolError(f"protocol {p.get('version')} phase {ph!r} is not one of {PHASES}")
    return ph


def frozen_gate(regs, p):
    """[error] for a run without a FINAL- registration under a frozen protocol."""
    if phase(p) == "frozen" and not any(str(r).startswith(FINAL) for r in regs or ()):
        return [f"protocol {p['version']} is frozen: every run needs a declared final's {FINAL}... registration"]
    return []


# ------------------------------------------------------------------------------------------ arm kinds

def _keys_within(spec, allowed):
    return set(spec) <= set(allowed) | {"name", "sets"}


def _select_kind(base, sel):
    if base == "skip":
        b = sel.get("budget")
        ok = (set(sel) == {"kind", "start", "budget"} and sel["kind"] == "start_recent" and sel["start"] == 0
              and type(sel["start"]) is int and type(b) in (int, float) and 0 < b < 1)
        return "skip+tailbudget" if ok else None
    if base not in ("kva", "noproj"):
        return None
    for suffix, want in ROW_SELECTORS.items():
        if sel == want:
            return f"{base}+{suffix}"
    if set(sel) == {"kind", "match"} and sel["kind"] in CONTROLS and isinstance(sel["match"], str):
        return f"{base}+{CONTROLS[sel['kind']]}"
    return None


def _structural_kind(spec):
    if set(spec) - ARM_KEYS:
        return None
    fill, sel = spec.get("fill", "exact"), spec.get("select")
    sweep = bool(SWEEP_MAP.search(str(spec.get("projector", ""))))
    if fill == "swiftkv_native":
        return "swiftkv-native" if _keys_within(spec, ("split", "fill")) else None
    if "tail_from" in spec:
        ok = spec["tail_from"] == "continuation" and fill == "identity" and _keys_within(spec, ("split", "fill", "tail_from"))
        return "pop-native" if ok else None
    if fill == "oracle":
        return "kvexact" if _keys_within(spec, ("split", "tail", "fill")) else None
    if fill == "by_type":
        ok = (spec.get("fill_by_type") == KVEXACT_HYBRID and sweep
              and _keys_within(spec, ("split", "tail", "fill", "fill_by_type", "projector")))
        return "kvexact" if ok else None
    base = BASE_OF_FILL.get(fill)
    if base is None or "fill_by_type" in spec or (base == "kva" and not sweep):
        return None
    if {"exact_part", "rescale", "rescale_skip_last"} & set(spec):
        if base != "kva" or not _keys_within(spec, ("split", "tail", "fill", "projector", "exact_part", "rescale",
                                                    "rescale_skip_last")):
            return None
        part, rs, skip = spec.get("exact_part"), spec.get("rescale"), spec.get("rescale_skip_last")
        if part in ("k", "v") and rs is None and skip is None:
            return f"kva+{part}exact"
        if part is None and rs in ("ktail", "vtail") and (skip is None or (type(skip) is int and skip >= 0)):
            return f"kva+{rs}"
        return None
    if spec.get("st"):
        return "kva+st" if base == "kva" and not sel else None
    return _select_kind(base, sel) if sel else base


def arm_kind(spec, p=None):
    """The protocol kind of an arm spec, or None (with p: None also for kinds p does not list)."""
    kind = _structural_kind(spec)
    return None if kind is None or (p is not None and kind not in p["arms"]) else kind


def template(kind, model, split, tail, p):
    """An arm spec of `kind` at (split, tail): arm_kind's inverse."""
    name = f"{kind}-s{split}" + ("" if tail is None else f"-t{tail}")
    proj = f"{model}-sweep-s{split}.safetensors"
    if kind == "pop-native":
        return dict(name=name, split=split, fill="identity", tail_from="continuation")
    if kind == "swiftkv-native":
        return dict(name=name, split=split, fill="swiftkv_native")
    if kind == "kvexact":
        if p["models"][model]["kind"] == "dense":
            return dict(name=name, split=split, tail=tail, fill="oracle")
        return dict(name=name, split=split, tail=tail, fill="by_type", fill_by_type=dict(KVEXACT_HYBRID), projector=proj)
    base, _, extra = kind.partition("+")
    spec = dict(name=name, split=split, tail=tail, fill={v: k for k, v in BASE_OF_FILL.items()}[base])
    if base == "kva":
        spec["projector"] = proj
    if extra in ROW_SELECTORS:
        spec["select"] = dict(ROW_SELECTORS[extra])
    elif extra in ("random", "tailmatch"):
        spec["select"] = dict(kind="random" if extra == "random" else "tail_match", match=f"{base}+qattn10")
    elif extra == "st":
        spec["st"] = "st.pt"
    elif extra in ("kexact", "vexact"):
        spec["exact_part"] = extra[0]
    elif extra in ("ktail", "vtail"):
        spec["rescale"] = extra
    elif extra == "tailbudget":
        spec["select"] = dict(kind="start_recent", start=0, budget=0.1)
    return spec


def protocol_row(spec, model, p):
    """A kind of p at one of the model's cells (split x tail grid, with each kind's own rules)."""
    kind, m = arm_kind(spec, p), p["models"].get(model)
    if kind is None or m is None:
        return False
    split = spec.get("split")
    if kind == "swiftkv":
        return bool(m.get("baseline_only"))
    if kind == "swiftkv-native":
        return bool(m.get("baseline_only")) and split in m["splits"]
    if m.get("baseline_only"):
        return False
    if kind == "pop-native":
        return split == m.get("pop_split")
    if split not in m["splits"]:
        return False
    if kind == "kva+st" and m["kind"] == "dense":
        return False
    if "+qblind" in kind and split != p.get("blind_splits", {}).get(model):
        return False
    if kind == "kvexact" and (spec.get("fill") == "oracle") != (m["kind"] == "dense"):
        return False
    return spec.get("tail") in p["tails"]


def battery_row(spec, model, p):
    return protocol_row(spec, model, p) and arm_kind(spec, p) not in p.get("outside_battery", ())


def battery_cells(model, p):
    """(split, tail, kind) of every battery row of a model in table order."""
    m = p["models"][model]
    kinds = [k for k in p["arms"] if k != "exact"]
    grid = [(s, t, k) for s in m["splits"] for t in p["tails"] for k in kinds if k not in TAILLESS]
    own = [(m.get("pop_split"), None, "pop-native")] + [(s, None, "swiftkv-native") for s in m["splits"]]
    return [(s, t, k) for s, t, k in grid + own
            if k in p["arms"] and s is not None and battery_row(template(k, model, s, t, p), model, p)]


def _row_in_config(spec, by_name, model, p):
    """protocol_row, and a matched control's target must be a rows arm of the same config, fill, split, tail."""
    if not protocol_row(spec, model, p):
        return False
    kind = arm_kind(spec, p)
    if not kind.endswith(("+random", "+tailmatch")):
        return True
    base, target = kind.split("+")[0], by_name.get(spec["select"]["match"])
    return (target is not None and arm_kind(target, p) in {f"{base}+{r}" for r in ROW_SELECTORS}
            and (target.get("split"), target.get("tail")) == (spec.get("split"), spec.get("tail")))


# ------------------------------------------------------------------------------------------ configs

def registered(ledger_path):
    """Hypothesis ids of the ledger (JSON lines with type 'hypothesis')."""
    ids = set()
    for line in Path(ledger_path).read_text().splitlines():
        if line.strip():
            rec = json.loads(line)
            if rec.get("type") == "hypothesis":
                ids.add(rec["id"])
    return ids


def validate(cfg, p=None, ledger_path=None, archive=None, env=os.environ, set_name=None):
    """Check a config against its era's protocol for one evaluation set; return the provenance stamp or raise
    ProtocolError listing every problem."""
    cur = p or load()
    archive = archive or protocol_file().parent / "protocol-archive"
    version = cfg.get("protocol")
    if not str(version or "").strip():
        raise ProtocolError(f"config has no 'protocol' version (current {cur['version']})")
    errors = []
    p = era(version, cur, archive)
    if p is None:
        errors.append(f"config protocol {version!r} is neither the current {cur['version']} nor archived")
        p = cur
    model_path = str(cfg.get("model", ""))
    model = Path(model_path).name
    if any(b in model_path.lower() for b in p.get("banned_model_substrings", ())):
        errors.append(f"banned model {model_path}")
    elif model not in p["models"]:
        errors.append(f"model {model!r} is not in the protocol's models ({p['version']})")
    regs = cfg.get("registration") or []
    if not regs:
        errors.append("no 'registration': list the ledger hypothesis ids this run serves")
    else:
        missing = sorted(set(regs) - registered(ledger_path or protocol_file().parent / cur["ledger"]))
        if missing:
            errors.append(f"registration ids not in the ledger: {missing}")
    errors += frozen_gate(regs, cur)
    if set_name in LOCKED_SETS:
        if LOCKED_SETS[set_name] not in p["sets"]["locked"]:
            errors.append(f"set {set_name!r} is not a locked set of the protocol")
        if not any(str(r).startswith(FINAL) for r in regs):
            errors.append(f"set {set_name!r} is locked: finals only, list the final's {FINAL}... id")
        if p is not cur:
            errors.append(f"set {set_name!r} is locked: finals run only under the current protocol {cur['version']}")
        want_caps = p.get("ruler_max_new", {}).get("tasks")
        if "ruler_max_new" in cfg and (set_name != "ruler" or cfg["ruler_max_new"] != want_caps):
            errors.append(f"ruler_max_new {cfg['ruler_max_new']!r}: only the ruler set, only {want_caps!r}")
        cap, got = p["models"].get(model, {}).get("max_len"), cfg.get(CAPS[set_name])
        if cap and not (type(got) is int and 0 < got <= cap):
            errors.append(f"{model} runs at <= {cap} tokens: set {CAPS[set_name]} to at most {cap}, got {got!r}")
    if env.get("RF_DETERMINISTIC", "1") != "1":
        errors.append("RF_DETERMINISTIC must be 1 for every protocol run")
    arms = cfg.get("arms", [])
    by_name = {a.get("name"): a for a in arms}
    off = [a["name"] for a in arms
           if model not in p["models"] or not _row_in_config(a, by_name, model, p) or cfg.get("drop_bos")]
    exploratory = str(cfg.get("exploratory", "")).strip()
    if off and not exploratory:
        errors.append(f"arms outside the protocol {off}: add an 'exploratory' reason or fix them")
    if errors:
        raise ProtocolError("protocol check failed:\n  - " + "\n  - ".join(errors))
    return dict(version=p["version"], sha256=p["sha256"], registration=list(regs), battery=not off and not exploratory,
                exploratory_arms=off, exploratory=cfg.get("exploratory") or None)
