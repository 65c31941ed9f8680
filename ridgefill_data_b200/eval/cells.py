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


def validate(schema, value, where="$"):
    """Every problem of value against schema (empty list: valid)."""
    unknown = [k for k in schema if k not in META and k not in KEYWORDS]
    if unknown:
        raise SchemaError(f"schema keyword(s) {unknown} at {where} are not implemented")
    errs = []
    t = schema.get("type")
    if t is not None:
        if t not in PY_TYPES:
            raise SchemaError(f"unknown type {t!r} at {where}")
        if not isinstance(value, PY_TYPES[t]) or (t in ("integer", "number") and isinstance(value, bool)):
            return [f"{where}: expected {t}, got {type(value).__name__}"]
    if "enum" in schema and value not in schema["enum"]:
        errs.append(f"{where}: {value!r} not in {schema['enum']}")
    if "const" in schema and value != schema["const"]:
        errs.append(f"{where}: must be {schema['const']!r}, got {value!r}")
    if isinstance(value, str) and "pattern" in schema and not re.match(schema["pattern"], value):
        errs.append(f"{where}: {value!r} does not match {schema['pattern']!r}")
    if isinstance(value, dict):
        props = schema.get("properties", {})
        errs += [f"{where}: missing required field {k!r}" for k in schema.get("required", []) if k not in value]
        extra = [k for k in value if k not in props]
        if schema.get("additionalProperties") is False and extra:
            errs.append(f"{where}: unknown field(s) {extra}")
        for k, v in value.items():
            if k in props:
                errs += validate(props[k], v, f"{where}.{k}")
    if isinstance(value, list):
        if len(value) < schema.get("minItems", 0):
            errs.append(f"{where}: needs >= {schema['minItems']} items, has {len(value)}")
        if schema.get("uniqueItems") and len({json.dumps(v, sort_keys=True) for v in value}) != len(value):
            errs.append(f"{where}: duplicate items")
        if "items" in schema:
            for j, v in enumerate(value):
                errs += validate(schema["items"], v, f"{where}[{j}]")
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
    return arm.startswith("ridgefill") or arm == "kvexact"


def semantic(cell):
    """(errors, warnings) of the cross-field rules."""
    errs, warns = [], []
    if cell.get("kind") == "flashnext":
        need = [k for k in ENGINE_ONLY if k not in cell] + [k for k in ("ttft_min_speedup", "ttft_length")
                                                            if k not in cell.get("margins", {})]
        if need or "runs" in cell or cell.get("split") != "-":
            errs.append(f"flashnext_cell: needs {need or 'split -'} and no runs (it runs on the engine's own driver)")
        return errs, warns
    if "runs" not in cell:
        errs.append("primary_run: a reference cell needs 'runs'")
    want = PRIMARY_SPLIT.get(cell.get("kind"), "3/8")
    if cell.get("split") != want or cell.get("tail") != 4096:
        errs.append(f"primary_run: a {cell.get('kind')} cell declares split {want} and tail 4096, not "
                    f"{cell.get('split')} / {cell.get('tail')}")
    present = [k for k in ENGINE_ONLY if k in cell]
    if present:
        errs.append(f"flashnext_cell: {present} belong to the engine-tier cell")
    for f in cell.get("projector", {}).get("files", []):
        if "sha256" not in f:
            warns.append(f"projector_unpinned: {f['file']} declares no sha256: the cell can not be registered or run")
    runs = cell.get("runs", [])
    ids = [r.get("id") for r in runs]
    dup = sorted({i for i in ids if ids.count(i) > 1})
    if dup:
        errs.append(f"run_ids_unique: duplicate run ids {dup}")
    if runs and not any(r.get("role") == "primary" and r.get("split") == cell.get("split") for r in runs):
        errs.append(f"primary_run: no run with role 'primary' at the primary split {cell.get('split')}")
    derived = cell.get("derived", {})
    for r in runs:
        arms, rid, s = r.get("arms", []), r.get("id"), r.get("set")
        if "exact" not in arms:
            errs.append(f"exact_in_every_run: run {rid} does not list 'exact'")
        swift = [a for a in arms if a in SWIFTKV_ARMS]
        if r.get("model") == "swiftkv":
            if set(arms) - {"exact", *SWIFTKV_ARMS} or not swift:
                errs.append(f"swiftkv_runs: run {rid} on the SwiftKV model lists {arms}")
            if "swiftkv_model" not in cell or not str(cell.get("model", {}).get("name", "")).startswith("llama"):
                errs.append(f"swiftkv_runs: run {rid} needs 'swiftkv_model' and a llama model")
        elif swift:
            errs.append(f"swiftkv_runs: run {rid} lists {swift} off the SwiftKV model")
        for c, rows in CONTROLS.items():
            if c in arms and rows not in arms:
                errs.append(f"controls_need_their_rows_arm: run {rid}: {c} needs {rows} in the same run")
        if any(a in QBLIND_ARMS for a in arms) and r.get("split") != "3/8":
            errs.append(f"qblind_at_the_blind_split: run {rid} has a qblind arm at {r.get('split')}")
        if "nofill+tailbudget" in arms and "tailbudget" not in cell:
            errs.append(f"tailbudget_declared: run {rid} has nofill+tailbudget without the cell's 'tailbudget'")
        if any(_uses_maps(a) for a in arms) and "projector" not in cell:
            errs.append(f"ridgefill_requires_projector: run {rid} needs the cell's 'projector'")
        for k in SET_BLOCKS.get(s, ()):
            if k not in cell:
                errs.append(f"set_blocks: run {rid} (set {s}) needs the cell's '{k}'")
        if s == "multiturn" and "ruler-twokey" not in derived:
            errs.append(f"set_blocks: run {rid} (set multiturn) needs derived 'ruler-twokey'")
        if r.get("variant") == "qfirst" and (s != "ruler" or "ruler-qfirst" not in derived):
            errs.append(f"set_blocks: run {rid} (variant qfirst) runs on ruler with derived 'ruler-qfirst'")
        if ("tasks" in r and s != "ruler") or ("lengths" in r and s not in ("ruler", "multiturn")):
            errs.append(f"row_selection: run {rid}: tasks on ruler runs only, lengths on ruler and multiturn runs")
        cap = cell.get("max_len")
        if cap and any(L > cap for L in r.get("lengths", [])):
            errs.append(f"row_selection: run {rid} selects lengths over max_len {cap}")
    if "dataset" in cell and (cell.get("kind") not in ("nll", "nll-causal", "nll-fresh")
                              or any(r.get("set") != "longppl" for r in runs)):
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
