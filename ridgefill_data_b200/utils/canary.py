"""Job-start canary (code/kva/canary.py:145-219 role): a fixed synthetic prompt through the exact arm and an
identity-fill arm; the logits' sha256 (and values) must match the reference stored for this host key (GPU name,
driver, CUDA and torch versions, model) bitwise, or within `tol` (max abs logit difference) when given. The first
run on a new host key writes the reference (mode 'record'); a mismatch raises CanaryMismatch before any result
is produced."""
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


def check(model, results_dir, split, mode="check", tol=None):
    key, facts = host_key(model.cfg.name)
    path = Path(results_dir) / f"canary-{key}.json"
    got = run(model, split)
    if mode == "record" or not path.exists():
        prov.write_json(path, dict(facts=facts, arms=got))
        return "recorded"
    ref = json.loads(path.read_text())["arms"]
    for arm, r in ref.items():
        g = got[arm]
        if g["sha256"] == r["sha256"]:
            continue
        if tol is not None:
            diff = max(abs(a - b) for a, b in zip(g["values"], r["values"]))
            if diff <= tol and g["argmax"] == r["argmax"]:
                continue
        raise CanaryMismatch(f"canary {arm}: logits differ from the reference {path} (sha {g['sha256'][:12]} vs "
                             f"{r['sha256'][:12]})")
    return "ok"
