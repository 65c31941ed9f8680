"""Research-protocol gate applied to a run config before any GPU work (the rules of code/kva/protocol.py:1-347).

The protocol file (protocol.json) carries: version, phase, ledger, models {name: layers, kind, splits, pop_split,
baseline_only, max_len, niah_format}, tails, arms {kind: description}, outside_battery, blind_splits, sets,
banned_model_substrings and ruler_max_new. A config names the protocol version it runs under, the ledger
hypotheses it serves and the model. It is judged under that version's era: the current file when the major.minor
matches, else the newest archived protocol-<x.y.z>.json of that major.minor. Every arm must be a protocol row, or
the config gives an "exploratory" reason. A frozen protocol refuses runs that carry no FINAL- registration, and the
locked sets run only as declared finals under the current protocol.

Arm kinds are read off an arm spec's structure; the names are the protocol file's identifiers:
  base        fill identity -> noproj, proj (a sweep map) -> kva, none -> skip, swiftkv -> swiftkv
  +rows       a named question-window selector: qattn5, qblind5, qattn10, qblind10
  +control    select {kind: random | tail_match, match: <a rows arm>} -> +random, +tailmatch
  kva+st, kva+kexact / kva+vexact (exact_part), kva+ktail / kva+vtail (rescale), kvexact (fill oracle, or the
  hybrid's attention oracle + GDN proj), pop-native (identity, tail_from continuation), swiftkv-native,
  skip+tailbudget
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
ARM_KEYS = frozenset({"name", "split", "tail", "fill", "projector", "sets", "select", "st", "reuse_fill",
                      "tail_from", "exact_part", "fill_by_type", "rescale", "rescale_skip_last"})
ROW_SELECTORS = {
    "qattn5": {"kind": "qattn", "budget": 0.05},
    "qblind5": {"kind": "qattn", "budget": 0.05, "window": "prefix"},
    "qattn10": {"kind": "qattn", "budget": 0.1},
    "qblind10": {"kind": "qattn", "budget": 0.1, "window": "prefix"},
}
CONTROLS = {"random": "random", "tail_match": "tailmatch"}
BASE_OF_FILL = {"identity": "noproj", "proj": "kva", "none": "skip", "swiftkv": "swiftkv"}
FILL_OF_BASE = {base: fill for fill, base in BASE_OF_FILL.items()}
SWEEP_MAP = re.compile(r"-sweep-s\d+\.safetensors$")
KVEXACT_HYBRID = {"attention": "oracle", "gdn": "proj"}
TAILLESS = ("pop-native", "swiftkv-native")
LOCKED_SETS = {"ruler": "ruler", "longbench": "longbench", "longppl": "long-prompts"}
CAPS = {"ruler": "ruler_max_len", "longbench": "longbench_max_len", "longppl": "longppl_max_len"}
_VERSION = re.compile(r"protocol-(\d+)\.(\d+)\.(\d+)\.json")


class ProtocolError(SystemExit):
    pass


def protocol_file():
    env = os.environ.get("RF_PROTOCOL")
    return Path(env) if env else REPO / "protocol.json"


def load(path=None):
    """The protocol as a dict, with the sha256 of its bytes added under 'sha256'."""
    raw = Path(path or protocol_file()).read_bytes()
    proto = json.loads(raw)
    proto["sha256"] = hashlib.sha256(raw).hexdigest()
    return proto


def minor(version):
    major, _, rest = str(version).partition(".")
    return f"{major}.{rest.split('.')[0]}" if rest else major


def archived(archive):
    """{major.minor: path} of the highest-patch protocol-<x.y.z>.json per major.minor in `archive`."""
    newest = {}
    for f in Path(archive).glob("protocol-*.json"):
        m = _VERSION.fullmatch(f.name)
        if m is None:
            continue
        key = tuple(int(x) for x in m.groups())
        mm = minor(".".join(m.groups()))
        if mm not in newest or key > newest[mm][0]:
            newest[mm] = (key, f)
    return {mm: f for mm, (_, f) in newest.items()}


def era(version, current, archive):
    """The protocol a config of this version is judged under (None when that era is not on file)."""
    if minor(version) == minor(current["version"]):
        return current
    path = archived(archive).get(minor(version))
    return None if path is None else load(path)


def phase(p):
    """'development' (the default) or 'frozen'."""
    declared = p.get("phase", PHASES[0])
    if declared in PHASES:
        return declared
    raise ProtocolError(f"protocol {p.get('version')}: phase {declared!r} is neither of {PHASES}")


def _has_final(regs):
    return any(str(r).startswith(FINAL) for r in regs or ())


def frozen_gate(regs, p):
    """[error] for a run that lacks a FINAL- registration under a frozen protocol."""
    if phase(p) != "frozen" or _has_final(regs):
        return []
    return [f"protocol {p['version']} is frozen: a run must serve a declared final ({FINAL}... registration)"]


# ------------------------------------------------------------------------------------------ arm kinds
def _only(spec, *keys):
    """The spec uses no keys beyond these (name and sets are always allowed)."""
    return set(spec) <= {"name", "sets", *keys}


def _select_kind(base, sel):
    if base == "skip":
        budget = sel.get("budget")
        tail_budget = (sel.get("kind") == "start_recent" and set(sel) == {"kind", "start", "budget"}
                       and type(sel["start"]) is int and sel["start"] == 0
                       and type(budget) in (int, float) and 0 < budget < 1)
        return "skip+tailbudget" if tail_budget else None
    if base not in ("kva", "noproj"):
        return None
    named = next((suffix for suffix, want in ROW_SELECTORS.items() if sel == want), None)
    if named is not None:
        return f"{base}+{named}"
    if set(sel) == {"kind", "match"} and sel["kind"] in CONTROLS and isinstance(sel["match"], str):
        return f"{base}+{CONTROLS[sel['kind']]}"
    return None


def _part_kind(spec, base):
    """kva+kexact / kva+vexact / kva+ktail / kva+vtail, or None."""
    if base != "kva" or not _only(spec, "split", "tail", "fill", "projector", "exact_part", "rescale",
                                  "rescale_skip_last"):
        return None
    part, rs, skip = spec.get("exact_part"), spec.get("rescale"), spec.get("rescale_skip_last")
    if part in ("k", "v") and rs is None and skip is None:
        return f"kva+{part}exact"
    skip_ok = skip is None or (type(skip) is int and skip >= 0)
    if part is None and rs in ("ktail", "vtail") and skip_ok:
        return f"kva+{rs}"
    return None


def _structural_kind(spec):
    if not set(spec) <= ARM_KEYS:
        return None
    fill = spec.get("fill", "exact")
    sel = spec.get("select")
    on_sweep_map = SWEEP_MAP.search(str(spec.get("projector", ""))) is not None
    if fill == "swiftkv_native":
        return "swiftkv-native" if _only(spec, "split", "fill") else None
    if "tail_from" in spec:
        pop = spec["tail_from"] == "continuation" and fill == "identity" and _only(spec, "split", "fill",
                                                                                   "tail_from")
        return "pop-native" if pop else None
    if fill == "oracle":
        return "kvexact" if _only(spec, "split", "tail", "fill") else None
    if fill == "by_type":
        hybrid = (on_sweep_map and spec.get("fill_by_type") == KVEXACT_HYBRID
                  and _only(spec, "split", "tail", "fill", "fill_by_type", "projector"))
        return "kvexact" if hybrid else None
    base = BASE_OF_FILL.get(fill)
    if base is None or "fill_by_type" in spec or (base == "kva" and not on_sweep_map):
        return None
    if set(spec) & {"exact_part", "rescale", "rescale_skip_last"}:
        return _part_kind(spec, base)
    if spec.get("st"):
        return "kva+st" if (base == "kva" and not sel) else None
    return _select_kind(base, sel) if sel else base


def arm_kind(spec, p=None):
    """The protocol kind of an arm spec, or None (given p, also None for a kind p does not list)."""
    kind = _structural_kind(spec)
    if kind is None or (p is not None and kind not in p["arms"]):
        return None
    return kind


def _suffix_fields(base, extra):
    """The spec fields a kind's +suffix adds."""
    if extra in ROW_SELECTORS:
        return {"select": dict(ROW_SELECTORS[extra])}
    if extra in ("random", "tailmatch"):
        return {"select": {"kind": "random" if extra == "random" else "tail_match", "match": f"{base}+qattn10"}}
    if extra == "st":
        return {"st": "st.pt"}
    if extra in ("kexact", "vexact"):
        return {"exact_part": extra[0]}
    if extra in ("ktail", "vtail"):
        return {"rescale": extra}
    if extra == "tailbudget":
        return {"select": {"kind": "start_recent", "start": 0, "budget": 0.1}}
    return {}


def template(kind, model, split, tail, p):
    """An arm spec of `kind` at (split, tail), the inverse of arm_kind."""
    name = f"{kind}-s{split}" if tail is None else f"{kind}-s{split}-t{tail}"
    sweep_map = f"{model}-sweep-s{split}.safetensors"
    if kind == "pop-native":
        return {"name": name, "split": split, "fill": "identity", "tail_from": "continuation"}
    if kind == "swiftkv-native":
        return {"name": name, "split": split, "fill": "swiftkv_native"}
    if kind == "kvexact":
        spec = {"name": name, "split": split, "tail": tail}
        if p["models"][model]["kind"] == "dense":
            return {**spec, "fill": "oracle"}
        return {**spec, "fill": "by_type", "fill_by_type": dict(KVEXACT_HYBRID), "projector": sweep_map}
    base, _, extra = kind.partition("+")
    spec = {"name": name, "split": split, "tail": tail, "fill": FILL_OF_BASE[base]}
    if base == "kva":
        spec["projector"] = sweep_map
    spec.update(_suffix_fields(base, extra))
    return spec


def protocol_row(spec, model, p):
    """The spec is a kind of p at one of the model's cells (its split x tail grid, with each kind's own rules)."""
    kind = arm_kind(spec, p)
    m = p["models"].get(model)
    if kind is None or m is None:
        return False
    split, baseline = spec.get("split"), bool(m.get("baseline_only"))
    if kind == "swiftkv":
        return baseline
    if kind == "swiftkv-native":
        return baseline and split in m["splits"]
    if baseline:
        return False
    if kind == "pop-native":
        return split == m.get("pop_split")
    dense = m["kind"] == "dense"
    refused = (split not in m["splits"]
               or (kind == "kva+st" and dense)
               or ("+qblind" in kind and split != p.get("blind_splits", {}).get(model))
               or (kind == "kvexact" and (spec.get("fill") == "oracle") != dense))
    return not refused and spec.get("tail") in p["tails"]


def battery_row(spec, model, p):
    """A protocol row that the battery tables include (kinds listed under outside_battery are rows, not battery)."""
    if not protocol_row(spec, model, p):
        return False
    return arm_kind(spec, p) not in set(p.get("outside_battery", ()))


def battery_cells(model, p):
    """(split, tail, kind) of every battery row of a model, in table order: the split x tail grid of the tailed
    kinds, then the model's pop-native cell, then swiftkv-native at each split."""
    entry = p["models"][model]
    listed = [k for k in p["arms"] if k != "exact"]
    candidates = [(s, t, k) for s in entry["splits"] for t in p["tails"] for k in listed if k not in TAILLESS]
    candidates.append((entry.get("pop_split"), None, "pop-native"))
    candidates.extend((s, None, "swiftkv-native") for s in entry["splits"])
    keep = []
    for s, t, k in candidates:
        if s is None or k not in p["arms"]:
            continue
        if battery_row(template(k, model, s, t, p), model, p):
            keep.append((s, t, k))
    return keep


def _row_in_config(spec, by_name, model, p):
    """protocol_row; a matched control must also point at a rows arm of the same config, fill, split and tail."""
    if not protocol_row(spec, model, p):
        return False
    kind = arm_kind(spec, p)
    if not (kind.endswith("+random") or kind.endswith("+tailmatch")):
        return True
    base = kind.split("+")[0]
    target = by_name.get(spec["select"]["match"])
    if target is None:
        return False
    rows_kinds = {f"{base}+{suffix}" for suffix in ROW_SELECTORS}
    same_cell = (target.get("split"), target.get("tail")) == (spec.get("split"), spec.get("tail"))
    return arm_kind(target, p) in rows_kinds and same_cell


# ------------------------------------------------------------------------------------------ configs
def registered(ledger_path):
    """Hypothesis ids of a ledger (JSON lines; records of type 'hypothesis')."""
    records = (json.loads(line) for line in Path(ledger_path).read_text().splitlines() if line.strip())
    return {r["id"] for r in records if r.get("type") == "hypothesis"}


def _locked_set_errors(cfg, set_name, p, cur, regs, model):
    errs = []
    if LOCKED_SETS[set_name] not in p["sets"]["locked"]:
        errs.append(f"set {set_name!r} is not among the protocol's locked sets")
    if not _has_final(regs):
        errs.append(f"set {set_name!r} is locked: it runs for declared finals only (give the {FINAL}... id)")
    if p is not cur:
        errs.append(f"set {set_name!r} is locked: finals run under the current protocol {cur['version']} only")
    caps = p.get("ruler_max_new", {}).get("tasks")
    if "ruler_max_new" in cfg and (set_name != "ruler" or cfg["ruler_max_new"] != caps):
        errs.append(f"ruler_max_new {cfg['ruler_max_new']!r} is allowed on the ruler set only, as {caps!r}")
    cap, got = p["models"].get(model, {}).get("max_len"), cfg.get(CAPS[set_name])
    if cap and not (type(got) is int and 0 < got <= cap):
        errs.append(f"{model} is capped at {cap} tokens: {CAPS[set_name]} must be an int in (0, {cap}], "
                    f"not {got!r}")
    return errs


def validate(cfg, p=None, ledger_path=None, archive=None, env=os.environ, set_name=None):
    """Check a config against its era's protocol for one evaluation set. Returns the provenance stamp, or raises
    ProtocolError listing every problem found."""
    cur = p or load()
    archive = archive or protocol_file().parent / "protocol-archive"
    version = cfg.get("protocol")
    if not str(version or "").strip():
        raise ProtocolError(f"the config names no 'protocol' version (the current one is {cur['version']})")
    errors = []
    p = era(version, cur, archive)
    if p is None:
        errors.append(f"protocol {version!r} is neither the current {cur['version']} nor an archived version")
        p = cur
    model_path = str(cfg.get("model", ""))
    model = Path(model_path).name
    if any(bad in model_path.lower() for bad in p.get("banned_model_substrings", ())):
        errors.append(f"the model {model_path} is banned by the protocol")
    elif model not in p["models"]:
        errors.append(f"the model {model!r} is not one of the protocol's models ({p['version']})")
    regs = cfg.get("registration") or []
    if regs:
        known = registered(ledger_path or protocol_file().parent / cur["ledger"])
        unknown = sorted(set(regs) - known)
        if unknown:
            errors.append(f"registrations not in the ledger: {unknown}")
    else:
        errors.append("no 'registration' given: list the ledger hypotheses this run serves")
    errors += frozen_gate(regs, cur)
    if set_name in LOCKED_SETS:
        errors += _locked_set_errors(cfg, set_name, p, cur, regs, model)
    if env.get("RF_DETERMINISTIC", "1") != "1":
        errors.append("protocol runs need RF_DETERMINISTIC=1")
    arms = cfg.get("arms", [])
    by_name = {a.get("name"): a for a in arms}
    off = [a["name"] for a in arms
           if cfg.get("drop_bos") or model not in p["models"] or not _row_in_config(a, by_name, model, p)]
    reason = str(cfg.get("exploratory", "")).strip()
    if off and not reason:
        errors.append(f"arms {off} lie outside the protocol: fix them or give an 'exploratory' reason")
    if errors:
        raise ProtocolError("protocol check failed:\n  - " + "\n  - ".join(errors))
    return {"version": p["version"], "sha256": p["sha256"], "registration": list(regs),
            "battery": not off and not reason, "exploratory_arms": off, "exploratory": cfg.get("exploratory") or None}
