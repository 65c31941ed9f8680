"""Job-start canary (code/kva/canary.py:145-219 role): a fixed synthetic prompt through the exact arm and an
identity-fill arm; the logits' sha256 (and values) must match a stored variant for this host key (GPU name, driver,
CUDA and torch versions, model) bitwise, or within `tol` (max abs logit difference) when given (models with known
numeric variants). The file keeps a list of accepted variants: the first run on a new host key records the first
one; mode 'accept' appends the current result as another variant after a reviewed mismatch, 'reset' replaces the
list. A result that matches no variant raises CanaryMismatch before any result is produced."""
from __future__ import annotations

import hashlib
import json
from pathlib import Path

import torch

from . import prov

PROMPT_LEN = 512
TAIL = 128


class CanaryMismatch(RuntimeError):
    pass


def host_key(model_name):
    g = prov.gpu_info() or {}
    facts = dict(gpu=g.get("name", "cpu"), cuda=torch.version.cuda, torch=torch.__version__, model=model_name)
    return hashlib.sha256(json.dumps(facts, sort_keys=True).encode()).hexdigest()[:16], facts


@torch.no_grad()
def run(model, split):
    from ..engine.arm import Arm
    from ..engine.prefill import prefill
    from ..eval.data import uniform_prompt
    ids = uniform_prompt(PROMPT_LEN, model.cfg.vocab, seed=20260930).to(model.device)
    out = {}
    for arm in (Arm("exact"), Arm("noproj", split=split, tail=TAIL, fill="identity")):
        logits, _, _ = prefill(model, ids, arm, keep=1)
        lg = logits.float().cpu()
        out[arm.name] = dict(sha256=hashlib.sha256(lg.numpy().tobytes()).hexdigest(), values=lg[0, :64].tolist(),
                             argmax=int(lg[-1].argmax()))
    return out


def _matches(got, variant, tol):
    for arm, r in variant.items():
        g = got[arm]
        if g["sha256"] == r["sha256"]:
            continue
        if tol is not None and g["argmax"] == r["argmax"] and \
                max(abs(a - b) for a, b in zip(g["values"], r["values"])) <= tol:
            continue
        return False
    return True


def check(model, results_dir, split, mode="check", tol=None):
    """'recorded' | 'ok (variant k)' | 'accepted (variant k)' | 'reset'; raises CanaryMismatch in mode check."""
    if mode not in ("check", "record", "accept", "reset"):
        raise ValueError(f"canary mode {mode!r}")
    key, facts = host_key(model.cfg.name)
    path = Path(results_dir) / f"canary-{key}.json"
    got = run(model, split)
    if not path.exists() or mode in ("record", "reset"):
        prov.write_json(path, dict(facts=facts, variants=[got]))
        return "reset" if mode == "reset" else "recorded"
    stored = json.loads(path.read_text())
    variants = stored.get("variants") or [stored["arms"]]
    for k, v in enumerate(variants):
        if _matches(got, v, tol):
            return f"ok (variant {k})"
    if mode == "accept":
        prov.write_json(path, dict(facts=facts, variants=variants + [got]))
        return f"accepted (variant {len(variants)})"
    raise CanaryMismatch(f"canary: logits match none of the {len(variants)} stored variant(s) in {path} "
                         f"(exact sha {got['exact']['sha256'][:12]}); after review, mode 'accept' adds this one")
