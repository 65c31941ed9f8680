"""Evaluation cells: one model x one battery part, declared as JSON and checked before anything runs
(code/finals/lib/cellcheck.py:1-194 role).

`validate(schema, value)` is a fail-closed validator for the JSON-Schema subset cell schemas use (type, enum,
const, pattern, required, properties, additionalProperties false, items, minItems, uniqueItems; $comment, $schema,
title and $semantic are metadata). A keyword outside that subset is a SchemaError: nothing unimplemented passes.
`semantic(cell)` checks the cross-field rules of a cell: (errors, warnings), each string led by the rule's name.

    python -m ridgefill_data_b200.eval.cells --schema cell.schema.json CELL.json   # 0 valid, 2 invalid, 3 schema error
"""
from __future__ import annotations

import json
import re
import sys
from pathlib import Path

META = frozenset(("$comment", "$schema", "title", "$semantic"))
KEYWORDS = frozenset(("type", "enum", "const", "pattern", "required", "properties", "additionalProperties", "items",
                      "minItems", "uniqueItems"))
PY_TYPES = {"object": dict, "array": list, "string": str, "boolean": bool, "integer": int, "number": (int, float)}


class SchemaError(RuntimeError):
    """The schema uses a keyword this validator does not implement."""


def _type_ok(t, value, where):
    if t not in PY_TYPES:
        raise SchemaError(f"unknown type {t!r} at {where}")
    numeric_bool = t in ("integer", "number") and isinstance(value, bool)
    return isinstance(value, PY_TYPES[t]) and not numeric_bool


def _object_errors(schema, value, where):
    props = schema.get("properties", {})
    out = [f"{where}: missing required field {k!r}" for k in schema.get("required", []) if k not in value]
    unknown = [k for k in value if k not in props]
    if unknown and schema.get("additionalProperties") is False:
        out.append(f"{where}: unknown field(s) {unknown}")
    for k, v in value.items():
        if k in props:
            out.extend(validate(props[k], v, f"{where}.{k}"))
    return out


def _array_errors(schema, value, where):
    out = []
    least = schema.get("minItems", 0)
    if len(value) < least:
        out.append(f"{where}: needs >= {least} items, has {len(value)}")
    if schema.get("uniqueItems"):
        canon = [json.dumps(v, sort_keys=True) for v in value]
        if len(set(canon)) != len(canon):
            out.append(f"{where}: duplicate items")
    if "items" in schema:
        for j, v in enumerate(value):
            out.extend(validate(schema["items"], v, f"{where}[{j}]"))
    return out


def validate(schema, value, where="$"):
    """Every problem of value against schema (an empty list: valid)."""
    unsupported = [k for k in schema if k not in META | KEYWORDS]
    if unsupported:
        raise SchemaError(f"schema keyword(s) {unsupported} at {where} are not implemented")
    if "type" in schema and not _type_ok(schema["type"], value, where):
        return [f"{where}: expected {schema['type']}, got {type(value).__name__}"]
    errs = []
    if "enum" in schema and value not in schema["enum"]:
        errs.append(f"{where}: {value!r} not in {schema['enum']}")
    if "const" in schema and value != schema["const"]:
        errs.append(f"{where}: must be {schema['const']!r}, got {value!r}")
    if "pattern" in schema and isinstance(value, str) and re.match(schema["pattern"], value) is None:
        errs.append(f"{where}: {value!r} does not match {schema['pattern']!r}")
    if isinstance(value, dict):
        errs += _object_errors(schema, value, where)
    if isinstance(value, list):
        errs += _array_errors(schema, value, where)
    return errs


# ------------------------------------------------------------------------------------------ cross-field rules
CONTROLS = {"identity+random": "identity+rows", "identity+tailmatch": "identity+rows",
            "ridgefill+random": "ridgefill+rows", "ridgefill+tailmatch": "ridgefill+rows"}
SWIFTKV_ARMS = ("swiftkv", "swiftkv-native")
QBLIND_ARMS = ("identity+qblind", "ridgefill+qblind")
ENGINE_ONLY = ("arms", "sets", "declared_share", "positive_control", "split_layer")
PRIMARY_SPLIT = {"ruler-deep": "5/8", "nll-fresh": "1/2"}         # every other kind: 3/8
SET_BLOCKS = {"longppl": ("keytoken",), "decode": ("decode",), "multiturn": ("secondq",)}


def _uses_maps(arm):
    return arm == "kvexact" or arm.startswith("ridgefill")


def _flashnext(cell):
    missing = [k for k in ENGINE_ONLY if k not in cell]
    missing += [k for k in ("ttft_min_speedup", "ttft_length") if k not in cell.get("margins", {})]
    if missing or "runs" in cell or cell.get("split") != "-":
        return [f"flashnext_cell: needs {missing or 'split -'} and no runs (it runs on the engine's own driver)"]
    return []


# per-run rules, applied to every run in this order: each returns its messages
def _exact_listed(cell, run, rid, arms):
    return [] if "exact" in arms else [f"exact_in_every_run: run {rid} does not list 'exact'"]


def _swiftkv(cell, run, rid, arms):
    swift = [a for a in arms if a in SWIFTKV_ARMS]
    if run.get("model") != "swiftkv":
        return [f"swiftkv_runs: run {rid} lists {swift} off the SwiftKV model"] if swift else []
    out = []
    if not swift or set(arms) - {"exact", *SWIFTKV_ARMS}:
        out.append(f"swiftkv_runs: run {rid} on the SwiftKV model lists {arms}")
    llama = str(cell.get("model", {}).get("name", "")).startswith("llama")
    if "swiftkv_model" not in cell or not llama:
        out.append(f"swiftkv_runs: run {rid} needs 'swiftkv_model' and a llama model")
    return out


def _controls(cell, run, rid, arms):
    return [f"controls_need_their_rows_arm: run {rid}: {c} needs {rows} in the same run"
            for c, rows in CONTROLS.items() if c in arms and rows not in arms]


def _qblind(cell, run, rid, arms):
    if run.get("split") != "3/8" and any(a in QBLIND_ARMS for a in arms):
        return [f"qblind_at_the_blind_split: run {rid} has a qblind arm at {run.get('split')}"]
    return []


def _tailbudget(cell, run, rid, arms):
    if "nofill+tailbudget" in arms and "tailbudget" not in cell:
        return [f"tailbudget_declared: run {rid} has nofill+tailbudget without the cell's 'tailbudget'"]
    return []


def _projector(cell, run, rid, arms):
    if "projector" not in cell and any(map(_uses_maps, arms)):
        return [f"ridgefill_requires_projector: run {rid} needs the cell's 'projector'"]
    return []


def _set_blocks(cell, run, rid, arms):
    s, derived = run.get("set"), cell.get("derived", {})
    out = [f"set_blocks: run {rid} (set {s}) needs the cell's '{k}'" for k in SET_BLOCKS.get(s, ()) if k not in cell]
    if s == "multiturn" and "ruler-twokey" not in derived:
        out.append(f"set_blocks: run {rid} (set multiturn) needs derived 'ruler-twokey'")
    if run.get("variant") == "qfirst" and not (s == "ruler" and "ruler-qfirst" in derived):
        out.append(f"set_blocks: run {rid} (variant qfirst) runs on ruler with derived 'ruler-qfirst'")
    return out


def _row_selection(cell, run, rid, arms):
    s = run.get("set")
    out = []
    if ("tasks" in run and s != "ruler") or ("lengths" in run and s not in ("ruler", "multiturn")):
        out.append(f"row_selection: run {rid}: tasks on ruler runs only, lengths on ruler and multiturn runs")
    cap = cell.get("max_len")
    if cap and any(L > cap for L in run.get("lengths", [])):
        out.append(f"row_selection: run {rid} selects lengths over max_len {cap}")
    return out


RUN_RULES = (_exact_listed, _swiftkv, _controls, _qblind, _tailbudget, _projector, _set_blocks, _row_selection)


def semantic(cell):
    """(errors, warnings) of the cross-field rules, each message led by its rule's name."""
    if cell.get("kind") == "flashnext":
        return _flashnext(cell), []
    errs, warns = [], []
    if "runs" not in cell:
        errs.append("primary_run: a reference cell needs 'runs'")
    want = PRIMARY_SPLIT.get(cell.get("kind"), "3/8")
    if (cell.get("split"), cell.get("tail")) != (want, 4096):
        errs.append(f"primary_run: a {cell.get('kind')} cell declares split {want} and tail 4096, not "
                    f"{cell.get('split')} / {cell.get('tail')}")
    engine_keys = [k for k in ENGINE_ONLY if k in cell]
    if engine_keys:
        errs.append(f"flashnext_cell: {engine_keys} belong to the engine-tier cell")
    warns += [f"projector_unpinned: {f['file']} declares no sha256: the cell can not be registered or run"
              for f in cell.get("projector", {}).get("files", []) if "sha256" not in f]
    runs = cell.get("runs", [])
    ids = [r.get("id") for r in runs]
    repeated = sorted({i for i in ids if ids.count(i) > 1})
    if repeated:
        errs.append(f"run_ids_unique: duplicate run ids {repeated}")
    if runs and not any(r.get("role") == "primary" and r.get("split") == cell.get("split") for r in runs):
        errs.append(f"primary_run: no run with role 'primary' at the primary split {cell.get('split')}")
    for run in runs:
        for rule in RUN_RULES:
            errs += rule(cell, run, run.get("id"), run.get("arms", []))
    longppl_only = cell.get("kind") in ("nll", "nll-causal", "nll-fresh") and all(r.get("set") == "longppl"
                                                                                   for r in runs)
    if "dataset" in cell and not longppl_only:
        errs.append(f"dataset_longppl_only: dataset {cell['dataset']!r} serves nll cells whose runs are all longppl")
    if cell.get("registration") == "FINAL-TBD":
        warns.append("final_tbd_flagged: registration 'FINAL-TBD': the cell does not run until it is registered")
    return errs, warns


def check(cell, schema):
    """(errors, warnings): the schema first; the cross-field rules only for a schema-valid cell."""
    errs = validate(schema, cell, cell.get("name", "cell") if isinstance(cell, dict) else "cell")
    if errs:
        return errs, []
    return semantic(cell)


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="validate an evaluation cell")
    ap.add_argument("--schema", required=True)
    ap.add_argument("cell")
    a = ap.parse_args(argv)
    try:
        errs, warns = check(json.loads(Path(a.cell).read_text()), json.loads(Path(a.schema).read_text()))
    except SchemaError as e:
        print(f"SCHEMA ERROR: {e}", file=sys.stderr)
        return 3
    for w in warns:
        print(f"WARNING {Path(a.cell).name}: {w}", file=sys.stderr)
    for e in errs:
        print(f"INVALID {Path(a.cell).name}: {e}", file=sys.stderr)
    return 2 if errs else 0


if __name__ == "__main__":
    sys.exit(main())
