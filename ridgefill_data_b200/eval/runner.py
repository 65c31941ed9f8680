"""Unattended runner for one declared evaluation cell (code/finals/lib/runner.py): every step fails closed and
names the reason.

  1. the cell's registration must not be FINAL-TBD and must be a ledger record (JSON lines, type 'hypothesis')
  2. the locked set on disk must be the cell's (MANIFEST.tsv sha256 == dataset_manifest_sha256 == FROZEN.json)
  3. host fingerprint (host name, GPU name, driver): a cell never resumes on another host unless new_host, which
     moves the old results to <cell>.abandoned-<utc> and restarts
  4. the cell declaration is frozen with its first results (cell.json must stay identical)
  5. samples: one sample with all its arms at a time (the pairing unit), each written atomically with a sha256
     sidecar; finished samples are skipped, so a rerun resumes
  6. .done with the results tree hash
The harness is a callable harness(cell, sample_id) -> dict; mock_harness is a deterministic stand-in whose
results are never evidence. Battery cells (a "runs" list: eval/cells.py) run instead through eval/backend.py on
this engine, after their registration's pins (the sha256 of the cell and of every config it expands to) are checked.

    python -m ridgefill_data_b200.eval.runner CELL.json --harness package.module:function [--new-host]
"""
from __future__ import annotations

import argparse
import hashlib
import importlib
import json
import os
import shutil
import socket
import time
from pathlib import Path

from ..utils import atomic
from . import locked as LK


class RunnerRefusal(SystemExit):
    pass


def log(msg):
    print(f"[{time.strftime('%H:%M:%S')}] {msg}", flush=True)


def host_info():
    from ..utils.prov import gpu_info
    g = gpu_info() or {}
    return dict(host=os.environ.get("RF_HOST") or socket.gethostname(), gpu_name=g.get("name", "cpu"),
                driver=g.get("driver", "none"))


def fingerprint(info):
    return hashlib.sha256(json.dumps(info, sort_keys=True).encode()).hexdigest()


def check_registration(cell, ledger):
    reg = cell.get("registration")
    if not reg or reg == "FINAL-TBD":
        raise RunnerRefusal(f"cell {cell['name']}: registration {reg!r} is not a declared FINAL- record")
    ids = set()
    if Path(ledger).exists():
        for line in Path(ledger).read_text().splitlines():
            if line.strip():
                rec = json.loads(line)
                if rec.get("type") == "hypothesis":
                    ids.add(rec["id"])
    if reg not in ids:
        raise RunnerRefusal(f"cell {cell['name']}: registration {reg} is not in the ledger {ledger}")


def check_locked(cell, root=None):
    man = LK.manifest(root, pin=cell.get("dataset_manifest_sha256"))
    for rel in cell.get("sources", []):
        LK.source(rel, man, root)
    return man


def sample_ids(cell, manifest=None):
    return list(cell["samples"])


def mock_harness(cell, sid):
    h = hashlib.sha256(f"{cell['name']}:{sid}".encode()).hexdigest()
    return dict(sample=sid, mock=True, arms={a: int(h[i:i + 4], 16) / 65535.0
                                             for i, a in enumerate(cell.get("arms", ["exact"]))})


def _claim_host(cell, cell_dir, info, new_host):
    """Steps 3-4: host fingerprint (restart elsewhere only with new_host) and the frozen cell declaration."""
    fp = fingerprint(info)
    host_file = cell_dir / "host.json"
    if host_file.exists():
        stored = json.loads(host_file.read_text())
        if stored.get("fingerprint") != fp:
            if not new_host:
                raise RunnerRefusal(f"cell {cell['name']} was started on {stored['host']} and this is {info}: a "
                                    "cell does not resume on another host (new_host restarts it)")
            gone = cell_dir.with_name(f"{cell_dir.name}.abandoned-{time.strftime('%Y%m%dT%H%M%SZ', time.gmtime())}")
            shutil.move(str(cell_dir), str(gone))
            log(f"new host: previous results moved to {gone}")
    cell_dir.mkdir(parents=True, exist_ok=True)
    if not host_file.exists():
        atomic.write_result(host_file, dict(fingerprint=fp, host=info))
    decl = cell_dir / "cell.json"
    if decl.exists():
        if json.loads(decl.read_text()) != cell:
            raise RunnerRefusal(f"cell.json in {cell_dir} differs from the declared cell: declare a new cell instead")
    else:
        atomic.write_result(decl, cell)


def run_battery_cell(cell, results_root, ledger, protocol, new_host=False, locked_root=None, info=None, env=None,
                     derived_dir=None, model=None):
    """A battery cell (a list of harness runs, eval/cells.py format): registration and its pins (the cell's and
    every generated config's sha256 must be what the FINAL- record pins), the locked set, host and declaration
    checks, then eval/backend.run_cell (preflight, harness, sidecars) and .done with the results tree hash."""
    from . import backend as BK
    check_registration(cell, ledger)
    problems = BK.check_record(cell, protocol, ledger)
    if problems:
        raise RunnerRefusal(f"cell {cell['name']}: " + "; ".join(problems))
    if cell.get("dataset_manifest_sha256") and any(r["set"] in LK.SETS for r in cell["runs"]):
        check_locked(cell, locked_root)
    cell_dir = Path(results_root) / cell["name"]
    _claim_host(cell, cell_dir, info or host_info(), new_host)
    n = BK.run_cell(cell, cell_dir, protocol, env=env if env is not None else os.environ, derived_dir=derived_dir,
                    model=model, log=log)
    tree = atomic.treehash(cell_dir)
    atomic.write_bytes(cell_dir / ".done", json.dumps(dict(cell=cell["name"], registration=cell["registration"],
                                                            records=n, tree_sha256=tree)).encode())
    log(f"cell {cell['name']} done: {n} records, tree {tree}")
    return tree


def run_cell(cell, results_root, harness, ledger, new_host=False, locked_root=None, info=None):
    check_registration(cell, ledger)
    manifest = check_locked(cell, locked_root) if cell.get("dataset_manifest_sha256") else None
    cell_dir = Path(results_root) / cell["name"]
    _claim_host(cell, cell_dir, info or host_info(), new_host)
    ids = sample_ids(cell, manifest)
    todo = [(s, cell_dir / "samples" / (s.replace("/", "__") + ".json")) for s in ids]
    todo = [(s, p) for s, p in todo if not atomic.finished(p)]
    log(f"{len(ids)} samples, {len(ids) - len(todo)} finished, {len(todo)} to run")
    for sid, path in todo:
        atomic.write_result(path, harness(cell, sid))
    tree = atomic.treehash(cell_dir)
    atomic.write_bytes(cell_dir / ".done", json.dumps(dict(cell=cell["name"], registration=cell["registration"],
                                                            tree_sha256=tree)).encode())
    log(f"cell {cell['name']} done: {len(ids)} samples, tree {tree}")
    return tree


def _load_harness(spec):
    mod, _, fn = spec.partition(":")
    return getattr(importlib.import_module(mod), fn)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("cell")
    ap.add_argument("--harness", default="ridgefill_data_b200.eval.runner:mock_harness")
    ap.add_argument("--results", default=os.environ.get("RF_RESULTS", "results/cells"))
    ap.add_argument("--ledger", default=os.environ.get("RF_LEDGER", "ledger.jsonl"))
    ap.add_argument("--new-host", action="store_true")
    ap.add_argument("--protocol", help="protocol.json for battery cells (default $RF_PROTOCOL)")
    a = ap.parse_args(argv)
    cell = json.loads(Path(a.cell).read_text())
    if "runs" in cell:                                     # a battery cell: harness runs on this engine
        from ..engine import protocol as PR
        run_battery_cell(cell, a.results, a.ledger, PR.load(a.protocol), a.new_host)
        return
    run_cell(cell, a.results, _load_harness(a.harness), a.ledger, a.new_host)


if __name__ == "__main__":
    main()
