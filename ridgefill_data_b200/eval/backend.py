"""Cells to harness runs on this engine (code/finals/lib/kvabackend.py:1-259 role).

harness_configs(cell, protocol) builds one harness config (eval/harness.py, the evaluate CLI's config format) per
(set, variant, model, tasks, lengths) group of a cell's runs, so one prompt's record holds every arm of every split
of those runs and their one exact (the pairing unit). Arms are engine.protocol.template() specs for the arm's
protocol kind, renamed <paper name>-s<layer>, map files under $RF_PROJ_DIR, matched controls pointing at the rows arm
of the same run, nofill+tailbudget taking the cell's budget. Splits are fractions of the model's layers on the
boundary below (floor(num x layers / den)); pop-native runs at the model's pop split, SwiftKV at 16.

run_cell(cell, cell_dir) refuses by name before any model is loaded (HarnessGap / StaleProjector): a missing
environment variable, a map file that is missing, not the bytes the cell pins, or fitted on another calibration list;
a derived-set manifest that is not the cell's. Then per config: the config is written (canonical bytes, whose sha256
a registration pins), the harness runs, and every record gets a sha256 sidecar.

The `ttft` set (the speed cells), which the reference marks as having no engine path, runs here on the engine itself:
per prompt length, each arm's prefill (run_lower + finish) timed on the device with CUDA events after a warm-up,
`repeats` times, recorded per length with the median.
"""
from __future__ import annotations

import dataclasses
import json
import os
import statistics
import time
from pathlib import Path

from ..utils import atomic

PAPER = {"nofill": "skip", "identity": "noproj", "ridgefill": "kva", "pop-native": "pop-native",
         "identity+rows": "noproj+qattn10", "ridgefill+rows": "kva+qattn10",
         "identity+qblind": "noproj+qblind10", "ridgefill+qblind": "kva+qblind10",
         "identity+random": "noproj+random", "ridgefill+random": "kva+random",
         "identity+tailmatch": "noproj+tailmatch", "ridgefill+tailmatch": "kva+tailmatch",
         "nofill+tailbudget": "skip+tailbudget",
         "ridgefill+kexact": "kva+kexact", "ridgefill+vexact": "kva+vexact", "kvexact": "kvexact",
         "ridgefill+ktail": "kva+ktail", "ridgefill+vtail": "kva+vtail",
         "swiftkv": "swiftkv", "swiftkv-native": "swiftkv-native"}
ROWS_OF = {"noproj": "identity+rows", "kva": "ridgefill+rows"}
TTFT_LENGTHS = (8192, 16384, 32768, 65536)


class HarnessGap(NotImplementedError):
    """A named missing piece: the cell can not run until it exists."""


class StaleProjector(RuntimeError):
    """A map file that is not the refit the cell declares."""


def layer_of(model_entry, frac):
    """The layer a split fraction 'a/b' names: floor(a * layers / b)."""
    num, _, den = frac.partition("/")
    return int(num) * model_entry["layers"] // int(den)


def _model_of(cell, run):
    source = cell["swiftkv_model"] if run.get("model") == "swiftkv" else cell["model"]
    return source["name"]


def _declared_maps(cell):
    return {f["layer"]: f["file"] for f in cell.get("projector", {}).get("files", [])}


def arm_spec(p, cell, run, paper, layer):
    """The harness arm spec of a paper arm name at a layer (the protocol template, renamed <paper>-s<layer>, with
    the map under $RF_PROJ_DIR and a control's match pointing at its rows arm)."""
    from ..engine import protocol as PR
    if paper not in PAPER:
        raise HarnessGap(f"unknown arm {paper!r}")
    kind = PAPER[paper]
    model = _model_of(cell, run)
    split = p["models"][model]["pop_split"] if kind == "pop-native" else layer
    spec = PR.template(kind, model, split, None if kind in PR.TAILLESS else cell["tail"], p)
    spec["name"] = f"{paper}-s{split}"
    if "projector" in spec:
        declared = _declared_maps(cell).get(split)
        if declared != spec["projector"]:
            raise HarnessGap(f"cell {cell['name']}: arm {paper} at layer {split} reads {spec['projector']}, which "
                             f"the cell's projector.files does not declare ({declared})")
        spec["projector"] = "$RF_PROJ_DIR/" + spec["projector"]
    select = spec.get("select", {})
    if "match" in select:
        select["match"] = f"{ROWS_OF[kind.partition('+')[0]]}-s{split}"
    if kind == "skip+tailbudget":
        select["budget"] = cell["tailbudget"]["b"]
    return spec


def _group_key(run):
    selection = (tuple(run.get("tasks", ())), tuple(run.get("lengths", ())))
    return (run["set"], run.get("variant"), run.get("model")) + selection


def _set_fields(cell, run):
    """Config keys a run's set (and its row selection) adds."""
    kind = run["set"]
    out = {}
    if kind == "longppl":
        out["keytoken_tail"] = cell["keytoken"]["tail"]
    elif kind == "decode":
        dec = cell["decode"]
        out.update(decode_from=dec["from"], decode_steps=dec["steps"], only=",".join(dec["only"]))
    elif kind == "multiturn":
        out.update(multiturn_from=cell["secondq"]["from"], multiturn_turns=cell["secondq"]["turns"])
    elif kind == "ttft":
        out["ttft_lengths"] = list(cell.get("ttft_lengths", TTFT_LENGTHS))
    if "dataset" in cell:
        out.update(dataset=cell["dataset"], dataset_manifest_sha256=cell["dataset_manifest_sha256"])
    for key, field in (("variant", "ruler_variant"), ("tasks", "ruler_tasks"), ("lengths", "ruler_lengths")):
        if run.get(key):
            out[field] = run[key] if key == "variant" else list(run[key])
    return out


def harness_config(cell, runs, p):
    """(config, set) of the runs that share a set, variant, model and row selection."""
    first = runs[0]
    model = _model_of(cell, first)
    entry = p["models"][model]
    arms, described = [], []
    for r in runs:
        layer = 16 if r.get("model") == "swiftkv" else layer_of(entry, r["split"])
        if layer not in entry["splits"]:
            raise HarnessGap(f"split {r['split']} of {model} is layer {layer}, not one of the protocol's "
                             f"{entry['splits']}")
        arms.extend(arm_spec(p, cell, r, a, layer) for a in r["arms"] if a != "exact")
        described.append(f"{r['id']} ({r['role']}, split {r['split']} = layer {layer})")
    names = [a["name"] for a in arms]
    cfg = dict(cell.get("caps", {}))
    cfg.update(name=f"{cell['model']['name']}-{first['id']}", protocol=cell["code_tag"].removeprefix("protocol-v"),
               registration=[cell["registration"]], model=f"$RF_MODEL_DIR/{model}",
               tokenizer=f"$RF_MODEL_DIR/{cell['model']['name']}", niah_format=entry.get("niah_format"),
               note=f"cell {cell['name']}, set {first['set']}, runs {', '.join(described)}; generated from the cell",
               arms=arms)
    cfg.update(_set_fields(cell, first))
    if len(names) != len(set(names)):
        raise HarnessGap(f"cell {cell['name']}: an arm appears twice in {cfg['name']}: {names}")
    return cfg, first["set"]


def harness_configs(cell, p):
    if cell["kind"] == "flashnext":
        raise HarnessGap("the flashnext cell runs on the engine driver (bench / serve), not through harness configs")
    groups = {}
    for r in cell["runs"]:
        groups.setdefault(_group_key(r), []).append(r)
    return [harness_config(cell, members, p) for members in groups.values()]


def config_bytes(cfg):
    """The bytes a run writes for a config (the pinned form): sorted keys, indent 1, trailing newline."""
    return json.dumps(cfg, indent=1, sort_keys=True).encode() + b"\n"


# ------------------------------------------------------------------------------------------ preflight
def check_projector(path, provenance, sha256=None):
    from ..ridge.projector import meta_of
    name = Path(path).name
    if not Path(path).is_file():
        raise StaleProjector(f"map file {path} does not exist ($RF_PROJ_DIR)")
    if sha256 is not None and atomic.sha256_file(path) != sha256:
        raise StaleProjector(f"StaleProjector: {name} is not the file the cell pins (sha256 {sha256[:16]})")
    meta = meta_of(path)
    if "docs" in meta and meta["docs"] != str(provenance["calib_docs"]):
        raise StaleProjector(f"StaleProjector: {name} was fitted on {meta['docs']} documents, the cell declares "
                             f"{provenance['calib_docs']}")
    if meta.get("rows") != str(provenance["calib_rows"]):
        raise StaleProjector(f"StaleProjector: {name} was fitted on {meta.get('rows')} rows, the cell declares "
                             f"{provenance['calib_rows']}")
    got = meta.get("calib_exclude_sha256")
    if got and got != provenance["calib_exclude_sha256"]:
        raise StaleProjector(f"StaleProjector: {name} was fitted with exclusion list {got[:12]}, the cell declares "
                             f"{provenance['calib_exclude_sha256'][:12]}")


def check_derived(cell, derived_dir):
    for name, want in cell.get("derived", {}).items():
        path = Path(derived_dir) / f"{name}.json"
        got = atomic.sha256_file(path) if path.is_file() else None
        if got != want:
            raise HarnessGap(f"DerivedManifestMismatch: {path} hashes to {got}, the cell pins {want}")


def preflight(cell, configs, env=os.environ, derived_dir=None):
    for v in ("RF_MODEL_DIR", "RF_PROJ_DIR"):
        if not env.get(v):
            raise HarnessGap(f"{v} is not set: the configs read models and map files from it")
    if derived_dir is not None:
        check_derived(cell, derived_dir)
    pinned = {f["file"]: f.get("sha256") for f in cell.get("projector", {}).get("files", [])}
    for cfg, _ in configs:
        for f in sorted({a["projector"] for a in cfg["arms"] if "projector" in a}):
            name = Path(f).name
            if not pinned.get(name):
                raise StaleProjector(f"UnpinnedProjector: cell {cell['name']} declares no sha256 for {name}")
            check_projector(f.replace("$RF_PROJ_DIR", env["RF_PROJ_DIR"]), cell["projector"]["provenance"],
                            pinned[name])


def expand_env(cfg, env=os.environ):
    """The config with $RF_MODEL_DIR / $RF_PROJ_DIR replaced (the harness reads plain paths)."""
    text = json.dumps(cfg)
    for v in ("RF_MODEL_DIR", "RF_PROJ_DIR"):
        if v in env:
            text = text.replace("$" + v, env[v])
    return json.loads(text)


# ------------------------------------------------------------------------------------------ runs
def run_ttft(cfg, out_dir, model=None, repeats=3, lengths=None, log=print):
    """The speed set on this engine: for each length a seeded prompt, every arm's TTFT (device time of run_lower +
    finish to the first-token logits; wall time on the CPU), `repeats` times after one warm-up."""
    import torch
    from ..engine.prefill import finish, run_lower
    from ..eval.data import uniform_prompt
    from .harness import Files, build_arm
    if model is None:
        from ..models.base import load
        model = load(cfg["model"], device="cuda" if torch.cuda.is_available() else "cpu")
    files = Files(model.device)
    arms = [build_arm(s, files) for s in cfg["arms"]]
    from ..engine.arm import Arm
    split0 = max(a.split for a in arms if a.split is not None)
    arms = [Arm("exact", split=split0)] + arms
    out_dir = Path(out_dir)
    out_dir.mkdir(parents=True, exist_ok=True)
    cuda = model.device.type == "cuda"
    n_done = 0
    for L in lengths or cfg.get("ttft_lengths", TTFT_LENGTHS):
        ids = uniform_prompt(L, model.cfg.vocab, seed=L).to(model.device)
        rec = dict(name=f"ttft-{L}", n=L, runs={})
        for a in arms:
            a = a if not a.tail_from else dataclasses.replace(a, tail=1)      # pop-native: the last token
            times = []
            for rep in range(repeats + 1):
                with torch.no_grad():
                    if cuda:
                        torch.cuda.synchronize()
                        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                        e0.record()
                    t0 = time.perf_counter()
                    hs, lower = run_lower(model, ids, [a.split])
                    _, _, P = finish(model, ids, hs[a.split], lower, a, 1, keep_cache=False)
                    if cuda:
                        e1.record()
                        torch.cuda.synchronize()
                        ms = e0.elapsed_time(e1)
                    else:
                        ms = 1e3 * (time.perf_counter() - t0)
                del hs, lower
                if rep:
                    times.append(round(ms, 3))
            rec["runs"][a.name] = dict(ttft_ms=times, median_ms=statistics.median(times), P=P, split=a.split,
                                       tail=L - P, clock="device" if cuda else "wall")
        ex = rec["runs"]["exact"]["median_ms"]
        for r in rec["runs"].values():
            r["speedup_vs_exact"] = round(ex / r["median_ms"], 4) if r["median_ms"] else None
        from ..utils.prov import write_json
        write_json(out_dir / f"{rec['name']}.json", rec)
        log(f"ttft {L}: " + " ".join(f"{k}:{r['median_ms']:.1f}ms" for k, r in rec["runs"].items()))
        n_done += 1
    return n_done


def run_cell(cell, cell_dir, p, env=os.environ, derived_dir=None, model=None, log=print):
    """Preflight, then every config: write it, run it through the harness (or the TTFT runner), sidecar every record
    it wrote. Returns the record count."""
    configs = harness_configs(cell, p)
    preflight(cell, configs, env, derived_dir)
    cell_dir = Path(cell_dir)
    n = 0
    for cfg, set_name in configs:
        cfg_path = cell_dir / f"harness-{cfg['name']}.json"
        atomic.write_bytes(cfg_path, config_bytes(cfg))
        plain = dict(expand_env(cfg, env), out=str(cell_dir / "work" / "results"))
        out_dir = cell_dir / "work" / "results" / f"{set_name}-{cfg['name']}"
        if set_name == "ttft":
            run_ttft(plain, out_dir, model=model, log=log)
        else:
            from .. import evaluate as E
            run_path = cell_dir / f"run-{cfg['name']}.json"
            run_path.write_text(json.dumps(plain, indent=1))
            rc = E.main([str(run_path), set_name])
            if rc:
                raise HarnessGap(f"the harness failed (exit {rc}) for {cfg['name']}")
        records = sorted(p_ for p_ in out_dir.glob("*.json"))
        if not records:
            raise HarnessGap(f"the harness wrote no records in {out_dir}")
        for r in records:
            atomic.refresh_sidecar(r)
        n += len(records)
    return n


# ------------------------------------------------------------------------------------------ registration pins
def canonical(obj):
    return json.dumps(obj, indent=1, sort_keys=True).encode() + b"\n"


def pins(cell, p):
    """{'cell': {name: sha256 of the cell's canonical bytes}, 'config': {name: sha256 of each generated config's
    bytes}}: what a FINAL- registration pins."""
    import hashlib
    return {"cell": {cell["name"]: hashlib.sha256(canonical(cell)).hexdigest()},
            "config": {cfg["name"]: hashlib.sha256(config_bytes(cfg)).hexdigest()
                       for cfg, _ in harness_configs(cell, p)}}


def pins_text(pn):
    """The pins as registration text: 'pins: cell NAME sha256=HEX; config NAME sha256=HEX; ...'."""
    return "pins: " + "; ".join(f"{k} {n} sha256={h}" for k in ("cell", "config") for n, h in pn[k].items())


def pins_of(text):
    import re
    got = {"cell": {}, "config": {}}
    for k, name, h in re.findall(r"\b(cell|config) (\S+) sha256=([0-9a-f]{64})", text or ""):
        got[k][name] = h
    return got


def superseded_label(rid):
    return f"superseded-{rid}"


def _ledger_records(ledger):
    path = Path(ledger)
    if not path.is_file():
        return []
    return [json.loads(s) for s in path.read_text().splitlines() if s.strip()]


def check_record(cell, p, ledger):
    """[] if the ledger's record for the cell's registration pins exactly this cell and the configs it generates and
    the id is not superseded; else the problems, by name."""
    want = pins(cell, p)
    recs = _ledger_records(ledger)
    rid = cell["registration"]
    if any(r.get("id") == superseded_label(rid) or r.get("label") == superseded_label(rid) for r in recs):
        return [f"Superseded: {rid} is superseded ({superseded_label(rid)} in {ledger})"]
    rec = next((r for r in recs if r.get("type") == "hypothesis" and r.get("id") == rid), None)
    if rec is None:
        return [f"registration {rid} is not a hypothesis id in {ledger}: register the cell first"]
    got = pins_of(rec.get("claim") or rec.get("text"))
    problems = [f"ConfigNotRegistered: {k} {n} sha256 {h[:16]} is not what {rid} pins ({got[k].get(n, 'nothing')[:16]})"
                for k in ("cell", "config") for n, h in want[k].items() if got[k].get(n) != h]
    problems += [f"ConfigNotRegistered: {rid} pins {k} {n}, which this cell does not generate"
                 for k in ("cell", "config") for n in got[k] if n not in want[k]]
    return problems
