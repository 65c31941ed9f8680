"""Evaluation CLI: arms x prompts, one atomic JSON record per prompt (resumable).

  python -m ridgefill_data_b200.evaluate CONFIG.json SET [--only a,b] [--limit k] [--canary check|accept|reset|off]

Configs in the research harness's format (no "prompts" block; its arm keys, $KVA_DATA / $RF_DATA paths) run the
harness's evaluation sets: SET = grade | niah | niahg | multiturn | ruler | longbench | longppl | decode
(eval/harness.py: protocol validation, canary, shared lower layers, selectors, reuse_fill, tail_round, tail_from,
oracle / context / refresh arms, key-token tails, per-prompt records with the harness's field names).

Configs with a "prompts" block run this framework's synthetic-set tasks (TASK below):

CONFIG: {"model": preset or checkpoint dir, "seed": 0, "backend": "b200"|"torch", "arms": [arm specs]
(engine/spec.py), "prompts": {"kind": ..., "lengths": [...], "count": k, "seed": s}, "out": results dir, "keep":
scored rows, "tokenizer": dir or "char" (text sets; default the model dir), "format": "raw"|"chat",
"protocol": version (optional: the research-protocol checks of engine/protocol.py run first)}.
Prompt kinds: token-id synthetic sets "uniform" | "zipf" | "niah" (no tokenizer), and the text sets "grade",
"k20" (K20 NIAH; "variant": "mk4"), "niahg", "ruler", "longbench", "longppl", "twokey", "qfirst" (eval/text.py,
eval/locked.py, eval/derived.py, eval/niahg.py; config keys of those modules: ruler_tasks, ruler_lengths,
ruler_max_len, longbench_max_len, longppl_max_len, ...).
TASK:
  quality   per arm: filled late-layer K/V (and GDN state) relative error vs exact prefill, next-token KL and
            top-1 agreement of the last `keep` rows
  ppl       per arm: mean NLL of the last `keep` prompt tokens (graded prompts: the last 512, also over novel
            tokens; long-prompt documents: the continuation)
  niah      greedy decode after each arm's prefill; correct iff the needle's value is reproduced
  generate  greedy decode up to the row's budget, decoded and scored by the set's metric (RULER, LongBench,
            non-numeric NIAH, K20)
  decode    decode agreement vs exact (teacher-forced KL, top-1, first divergence)
  speed     per arm: device-timed TTFT (CUDA events) and tokens/s
Validation happens before any model is built (engine/spec.py, engine/protocol.py); results carry a provenance
block and are written atomically, one per prompt (a rerun skips finished prompts).
"""
import argparse
import json
import sys
import time
from pathlib import Path

import torch


TEXT_KINDS = ("grade", "k20", "niahg", "ruler", "longbench", "longppl", "twokey", "qfirst")


def text_prompts(cfg, tok):
    """Prompts of a text set for this tokenizer (ids as tensors)."""
    from .eval import derived, locked, niahg
    from .eval import text as TX
    p = cfg.get("prompts", {})
    kind, fmt = p["kind"], cfg.get("format", "raw")
    if kind == "grade":
        out = TX.grade_prompts(tok, fmt)
    elif kind == "k20":
        out = TX.niah_prompts(tok, fmt, variant=p.get("variant"))
    elif kind == "niahg":
        out = niahg.prompts(tok, fmt)
    elif kind in ("twokey", "qfirst"):
        man = locked.manifest()
        out, _ = derived.prompts(kind, tok, fmt, man, cfg.get("ruler_max_len"), cfg.get("ruler_tasks"),
                                 cfg.get("ruler_lengths"), cfg.get("ruler_max_new"))
    else:
        protocol = {"models": {Path(str(cfg["model"])).name: {"niah_format": fmt}}}
        out, _ = locked.prompts(kind, tok, dict(cfg, niah_format=fmt), Path(str(cfg["model"])).name, protocol)
    for q in out:
        q["ids"] = torch.as_tensor(q["ids"], dtype=torch.long)
    return out


def prompts_of(cfg, vocab, tok=None):
    from .eval.data import uniform_prompt, zipf_ids
    from .eval.niah import DEPTHS, niah_prompt
    p = cfg.get("prompts", {})
    kind, seed = p.get("kind", "uniform"), p.get("seed", 2)
    if kind in TEXT_KINDS:
        return text_prompts(cfg, tok)
    out = []
    for n in p.get("lengths", [2048]):
        for j in range(p.get("count", 1)):
            if kind == "uniform":
                out.append(dict(name=f"uniform-{n}-{j}", ids=uniform_prompt(n, vocab, seed=seed + j)))
            elif kind == "zipf":
                out.append(dict(name=f"zipf-{n}-{j}", ids=zipf_ids(n, vocab, seed=seed + j)))
            elif kind == "niah":
                d = DEPTHS[j % len(DEPTHS)]
                rec = niah_prompt(n, vocab, d, seed=seed + j)
                out.append(dict(name=f"niah-{n}-{d}-{j}", **rec))
            else:
                raise ValueError(f"prompt kind {kind!r}")
    return out


def _rel(a, b):
    return float((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30))


def score_generation(prm, text):
    """The row's own metric on a decoded continuation."""
    from .eval import locked, niahg
    from .eval import text as TX
    if prm.get("set") in ("ruler", "longbench"):
        return locked.score(prm, text)
    if "type" in prm:                                   # non-numeric NIAH
        return niahg.score(text, prm["value"], prm["type"], prm.get("format", "raw"))
    return dict(pred=text, score=float(TX.niah_correct(text, prm["value"])))


@torch.no_grad()
def run_prompt(model, arms, prm, task, keep, tok=None):
    from .engine.decode import greedy
    from .engine.prefill import finish, run_lower
    from .engine import agree as AG
    from .engine.arm import Arm
    from .engine.decode import fork_cache
    from .engine.scoring import kl, score_tokens, top1_agree
    ids = prm["ids"].to(model.device)
    n = ids.shape[0]
    rec = dict(name=prm["name"], n=n, runs={})
    exact_logits, exact_cache = model.forward_exact(ids, keep=torch.arange(n - keep, n, device=model.device))
    splits = sorted({a.split for a in arms if a.split is not None})
    lower = {S: run_lower(model, ids, [S]) for S in splits}
    for arm in arms:
        t0 = time.time()
        if arm.fill == "exact":
            logits, cache = exact_logits, exact_cache
        else:
            hs, lc = lower[arm.split]
            logits, cache, _ = finish(model, ids, hs[arm.split], lc, arm, keep)
        r = dict(wall_s=round(time.time() - t0, 4))
        if task == "quality":
            errs = {}
            for i in range(arm.split or model.n_layers, model.n_layers):
                c, e = cache[i], exact_cache[i]
                if model.layer_types[i] == "attn":
                    errs[i] = dict(k=_rel(c["k"], e["k"]), v=_rel(c["v"], e["v"]))
                else:
                    errs[i] = dict(state=_rel(c["rec"], e["rec"]))
            r.update(kv_rel_err=errs, kl=float(kl(exact_logits, logits).mean()),
                     top1=float(top1_agree(exact_logits, logits).mean()))
        elif task == "ppl":
            lp = score_tokens(logits, ids, keep - 1).double()
            r["nll"] = float(-lp.mean())
            novel = prm.get("novel")
            if novel is not None and len(novel) == keep - 1:
                m = torch.tensor(novel, dtype=torch.bool)
                r["nll_novel"] = float(-lp[m].mean()) if bool(m.any()) else None
        elif task == "generate":
            steps = int(prm.get("max_new", 32))
            gen, reason = greedy(model, ids, cache, logits, steps, arm, eos=tuple(getattr(model, "eos_ids", ()) or ()))
            text = tok.decode(gen, skip_special_tokens=False) if tok is not None else ""
            r.update(gen=gen, finish_reason=reason, **score_generation(prm, text))
        elif task == "niah":
            from .eval.niah import niah_correct
            gen, reason = greedy(model, ids, cache, logits, len(prm["value"]) + 4, arm)
            r.update(gen=gen, finish_reason=reason, correct=niah_correct(gen, prm["value"]))
        elif task == "decode":
            fields, ref = AG.exact_record(model, n, fork_cache(exact_cache), exact_logits, 8, Arm("exact"))
            r.update(AG.compare(model, n, cache, logits, 8, arm, *ref), exact_gen=fields["gen"])
        rec["runs"][arm.name] = r
    return rec


TASKS = ("quality", "ppl", "niah", "generate", "decode", "speed")


def harness_main(cfg, a):
    """The research harness's sets (eval/harness.py) for a config in its format."""
    import os

    from .engine import protocol as PR
    from .eval import harness as H
    from .eval import text as TX
    from .models.base import from_config, load
    from .models.config import PRESETS
    from .utils import canary, gpu, prov
    if a.set not in H.SETS:
        raise SystemExit(f"set {a.set!r}: one of {H.SETS} (configs without a 'prompts' block)")
    source = a.set
    if a.set == "decode":
        source = cfg.get("decode_from")
    if a.set == "multiturn" and cfg.get("multiturn_from", "mk4") == "ruler":
        source = "ruler"
    dry = os.environ.get("RF_CPU_DRYRUN") == "1"
    stamp = None if (dry and "protocol" not in cfg) else PR.validate(cfg, set_name=source)
    device, gpu_info = gpu.setup()
    backend = cfg.get("backend", "b200" if device.type == "cuda" else "torch")
    dtype = torch.float32 if cfg.get("dtype") == "fp32" else torch.bfloat16
    tok_path = cfg.get("tokenizer", cfg["model"])
    tok = TX.tokenizer(tok_path)
    name = Path(str(cfg["model"])).name
    if cfg["model"] in PRESETS:
        model = from_config(PRESETS[cfg["model"]], seed=cfg.get("seed", 0), device=device, backend=backend,
                            dtype=dtype)
    else:
        model = load(cfg["model"], device=device, backend=backend, dtype=dtype)
    root = Path(cfg.get("out", "results"))
    out = root / f"{a.set}-{cfg['name']}"
    out.mkdir(parents=True, exist_ok=True)
    eos = TX.eos_ids(tok_path, tok) if tok_path != "char" else (tok.eos_token_id,)
    try:
        h = H.Harness(model, tok, cfg, a.set, out, eos=eos)
    except H.EvalError as e:
        raise SystemExit(f"refusing: {e}")
    if a.canary != "off":
        split = min(x.split for x in h.arms if x.split is not None) if any(x.split for x in h.arms) else \
            model.n_layers // 2
        tol = cfg.get("canary_tolerance")
        print(f"canary: {canary.check(model, root, split, a.canary, tol)}")
    try:
        protocol = PR.load()
    except OSError:
        protocol = {"models": {name: {"niah_format": cfg.get("niah_format", "raw")}}}
    prompts, extra = H.set_prompts(a.set, cfg, tok, name, protocol)
    if a.set == "niahg":
        trim = cfg.get("niahg_tail", max(x.tail for x in h.arms if x.split is not None))
        prompts = [q for q in prompts if q["needle_end"] <= len(q["ids"]) - trim]
        extra["niahg_tail"] = trim
    only = a.only or cfg.get("only", "")
    if only:
        prompts = [q for q in prompts if q["name"] in only.split(",")]
    if a.limit:
        prompts = prompts[:a.limit]
    run_cfg = dict(config=cfg, protocol=stamp, set=a.set, keep=H.KEEP, niah_steps=H.NIAH_STEPS,
                   file_sha256=h.files.hashes, **extra)
    try:
        n = h.run(prompts, prov.provenance(cfg["model"], run_cfg, gpu_info))
    except H.EvalError as e:
        raise SystemExit(f"refusing: {e}")
    print(f"done: {n} prompts run, {len(prompts) - n} already complete")
    return 0


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("config")
    ap.add_argument("set", help="harness set (grade niah niahg multiturn ruler longbench longppl decode) or, for "
                                "configs with a 'prompts' block, a task (quality ppl niah generate decode speed)")
    ap.add_argument("--only", default="")
    ap.add_argument("--limit", type=int, default=0)
    ap.add_argument("--canary", choices=("check", "accept", "reset", "off"), default="check")
    a = ap.parse_args(argv)
    from .engine import spec
    from .models.base import from_config, load
    from .models.config import PRESETS, ModelConfig
    from .utils import prov
    cfg = spec.load(a.config)
    if "prompts" not in cfg:
        return harness_main(cfg, a)
    a.task = a.set
    if a.task not in TASKS:
        raise SystemExit(f"task {a.task!r}: one of {TASKS} (configs with a 'prompts' block)")
    mcfg = PRESETS[cfg["model"]] if cfg["model"] in PRESETS else ModelConfig.from_dir(cfg["model"])
    spec.validate(cfg, mcfg.n_layers)
    stamp = None
    if cfg.get("protocol"):
        from .engine import protocol
        stamp = protocol.validate(cfg, set_name=cfg.get("prompts", {}).get("kind"))
    tok = None
    if cfg.get("prompts", {}).get("kind") in TEXT_KINDS or a.task == "generate":
        from .eval.text import tokenizer
        tok = tokenizer(cfg.get("tokenizer", cfg["model"]))
    dev = cfg.get("device", "cuda" if torch.cuda.is_available() else "cpu")
    backend = cfg.get("backend", "b200" if dev.startswith("cuda") else "torch")
    dtype = torch.float32 if cfg.get("dtype") == "fp32" else torch.bfloat16
    if cfg["model"] in PRESETS:
        model = from_config(mcfg, seed=cfg.get("seed", 0), device=dev, backend=backend, dtype=dtype)
    else:
        model = load(cfg["model"], device=dev, backend=backend, dtype=dtype)
    cache = {}
    arms = [spec.arm_of(s, dev, cache) for s in cfg["arms"]]
    out = Path(cfg.get("out", "results")) / a.task
    keep = cfg.get("keep", 16)
    prompts = prompts_of(cfg, mcfg.vocab, tok)
    if cfg.get("prompts", {}).get("kind") == "longppl":        # every scored row inside every arm's exact tail
        from .eval.locked import check_tails

        def tail_of(arm):
            return lambda q: len(q["ids"]) - (arm.prefix_len(len(q["ids"])) if arm.split is not None else 0)
        check_tails(prompts, {arm.name: tail_of(arm) for arm in arms})
    for prm in prompts:
        path = out / f"{prm['name']}.json"
        if path.exists():
            continue
        if a.task == "speed":
            rec = dict(name=prm["name"], runs={})
            from .engine.prefill import prefill
            ids = prm["ids"].to(dev)
            for arm in arms:
                prefill(model, ids, arm)
                if dev.startswith("cuda"):
                    torch.cuda.synchronize()
                    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    e0.record()
                    prefill(model, ids, arm)
                    e1.record()
                    torch.cuda.synchronize()
                    ms = e0.elapsed_time(e1)
                else:
                    t0 = time.time()
                    prefill(model, ids, arm)
                    ms = (time.time() - t0) * 1e3
                rec["runs"][arm.name] = dict(ttft_ms=ms, tok_s=ids.shape[0] / ms * 1e3)
        else:
            k = keep
            if a.task == "ppl" and "cont_len" in prm:
                k = prm["cont_len"] + 1                   # long-prompt documents: the whole continuation
            elif a.task == "ppl" and "novel" in prm:
                k = len(prm["novel"]) + 1                 # graded prompts: the scored window
            rec = run_prompt(model, arms, prm, a.task, k, tok)
        rec["provenance"] = prov.provenance(cfg["model"], dict(task=a.task, protocol=stamp))
        prov.write_json(path, rec)
        print(json.dumps({k: v for k, v in rec.items() if k != "provenance"})[:400])
    return 0


if __name__ == "__main__":
    sys.exit(main())
