"""Typed run configuration: arm specs (the reference's JSON arm keys) and their validation before any GPU
work (code/kva/protocol.py:182-284 role: refuse a bad config by name, early).

A config JSON: {"model": preset name or checkpoint dir, "arms": [spec, ...], "prompts": {...}, "out": dir}.
An arm spec: {"name", "split", "tail", "fill", "projector" (map file), "st" (correction file), "select",
"fill_by_type", "context", "refresh", "refresh_projector", "tail_bias_from", "tail_bias_skip_last",
"exact_part", "rescale", "rescale_skip_last", "tail_from", "f1", "kvfold", "repair", "repair_by", "sets",
"reuse_fill", "tail_round"}.
"""
from __future__ import annotations

import json
from pathlib import Path

from ..utils.paths import expand
from .arm import FILLS, ORACLE_RESCALE, TAIL_RESCALE, Arm
from .select import KINDS

SPEC_KEYS = {"name", "split", "tail", "fill", "projector", "st", "select", "fill_by_type", "context", "refresh",
             "refresh_projector", "tail_bias_from", "tail_bias_skip_last", "exact_part", "rescale",
             "rescale_skip_last", "tail_from", "f1", "kvfold", "repair", "repair_by", "sets", "reuse_fill",
             "tail_round"}


class ConfigError(ValueError):
    pass


def validate_spec(spec, n_layers):
    """Raise ConfigError naming the first problem of one arm spec."""
    name = spec.get("name", "?")
    unknown = set(spec) - SPEC_KEYS
    if unknown:
        raise ConfigError(f"arm {name}: unknown keys {sorted(unknown)}")
    fill = spec.get("fill", "exact")
    if fill not in FILLS:
        raise ConfigError(f"arm {name}: fill {fill!r} not in {FILLS}")
    if fill != "exact":
        s = spec.get("split")
        if not isinstance(s, int) or not 0 < s < n_layers:
            raise ConfigError(f"arm {name}: split {s!r} must be an int in (0, {n_layers})")
        if spec.get("tail_from") is not None:
            if spec["tail_from"] != "continuation" or "tail" in spec:
                raise ConfigError(f"arm {name}: tail_from 'continuation' sets the tail per prompt (no 'tail')")
        elif fill != "swiftkv_native" and (not isinstance(spec.get("tail"), int) or spec["tail"] < 1):
            raise ConfigError(f"arm {name}: tail must be a positive int")
    if fill == "proj" and "projector" not in spec:
        raise ConfigError(f"arm {name}: fill 'proj' needs a projector file")
    sel = spec.get("select")
    if sel is not None and sel.get("kind") not in KINDS:
        raise ConfigError(f"arm {name}: select kind {sel.get('kind')!r} not in {KINDS}")
    rs = spec.get("rescale")
    if rs is not None and rs not in ORACLE_RESCALE + TAIL_RESCALE:
        raise ConfigError(f"arm {name}: rescale {rs!r}")
    if spec.get("exact_part") not in (None, "k", "v"):
        raise ConfigError(f"arm {name}: exact_part must be 'k' or 'v'")


def validate(cfg, n_layers):
    if not cfg.get("arms"):
        raise ConfigError("config has no arms")
    names = [a.get("name") for a in cfg["arms"]]
    if len(set(names)) != len(names) or None in names:
        raise ConfigError(f"arm names must be present and unique: {names}")
    for a in cfg["arms"]:
        validate_spec(a, n_layers)
        sel = a.get("select") or {}
        if "match" in sel and sel["match"] not in names:
            raise ConfigError(f"arm {a['name']}: select.match {sel['match']!r} is not an arm")


def load(path):
    return expand(json.loads(Path(path).read_text()))


def arm_of(spec, device="cpu", projector_cache=None):
    """An Arm from a validated spec (map files loaded once per path)."""
    from ..ridge.projector import Projector, load_st
    cache = {} if projector_cache is None else projector_cache

    def proj(path):
        if path not in cache:
            cache[path] = Projector.load(path, device)
        return cache[path]

    kw = {k: spec[k] for k in ("split", "tail", "fill", "fill_by_type", "context", "refresh", "tail_bias_from",
                              "tail_bias_skip_last", "exact_part", "rescale", "rescale_skip_last", "tail_from", "f1")
          if k in spec}
    if "projector" in spec:
        kw["projector"] = proj(spec["projector"])
    if "refresh_projector" in spec:
        kw["refresh_projector"] = proj(spec["refresh_projector"])
    if "st" in spec:
        kw["st"] = load_st(spec["st"], device)
    meta = {k: spec[k] for k in ("select", "repair", "repair_by") if k in spec}
    return Arm(spec["name"], meta=meta, **kw)
