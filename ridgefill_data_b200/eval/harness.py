"""The evaluation sets of the research harness, run through this engine (semantics of code/scripts/evaluate.py:
1-649; the same config files, set names, arm keys and per-prompt record fields, so configs and results move between
the two).

  grade      log-probs of the last 512 prompt tokens per arm (inside every arm's exact tail), the novel-token mask
             and the short-context reference; grade_format raw | chat
  niah       K20 needle-in-a-haystack: greedy up to 48 tokens, the first standalone 7-digit number must be the value
  niahg      the non-numeric NIAH set (names, phrases, hex ids, identifiers, sentences), needles inside every arm's
             approximated prefix only (niahg_tail)
  multiturn  mk4 prompts as k-turn chats over one carried cache, with deferred repair arms (eval/multiturn.py)
  ruler, longbench, longppl   the locked test set (eval/locked.py): greedy to the task's output length and the
             official metric; longppl the continuation's NLL
  decode     exact vs every arm over decode_steps tokens (engine/agree.py), prompts from decode_from (grade | longppl)
             without their scored tokens
Per prompt: the lower layers run once and are shared; every arm runs finish() over them (largest split first),
optionally with exact rows chosen by its selector (engine/select.py: digits, regex, verbatim, qattn, pred, freq,
frag, blend, band, start_recent, keydiff, deviation, qfp, random, tail_match), a reused fill (reuse_fill), a
block-rounded tail (tail_round), the continuation as the tail (tail_from), oracle inputs, context inputs,
refresh, K/V rescale or tail bias. One JSON record per prompt, rewritten after every prompt; a rerun skips the
prompts whose ids and arms are complete. keytoken_tail adds the exact model's log-probs given only the last T ids.
"""
from __future__ import annotations

import dataclasses
import hashlib
import json
import time
from pathlib import Path

import torch

from ..engine import agree as AG
from ..engine import select as SEL
from ..engine.arm import ENGINE_MIN_TAIL, Arm, exclude_scored, rounded_tail
from ..engine.prefill import finish, oracle_tap, run_lower
from ..engine.scoring import check_finite, score_tokens
from . import text as TX

SETS = ("grade", "niah", "niahg", "multiturn", "ruler", "longbench", "longppl", "decode")
DECODE_FROM = ("grade", "longppl")
MULTITURN_FROM = ("mk4", "ruler")
KEEP = TX.SCORED + 1
NIAH_STEPS = 48
DECODE_STEPS = 512
TURN_ROWS = 64               # rows a later multiturn question adds at most (position guard)


class EvalError(ValueError):
    """A config, arm or prompt refused before (or instead of) running."""


# ---------------------------------------------------------------------------------------------- arm checks
def check_reuse(specs):
    """reuse_fill: the named arm must come earlier, with the same split, tail, fill, maps and selection."""
    by_name = {}
    for s in specs:
        src = by_name.get(s.get("reuse_fill"))
        if "reuse_fill" in s and src is None:
            raise EvalError(f"arm {s['name']}: reuse_fill {s['reuse_fill']!r} is not an earlier arm")
        if src is not None:
            diff = [k for k in ("split", "tail", "tail_round", "tail_from", "fill", "fill_by_type", "projector",
                                "kvfold", "select", "context", "refresh", "refresh_projector", "tail_bias_from",
                                "tail_bias_skip_last", "exact_part", "rescale", "rescale_skip_last")
                    if s.get(k) != src.get(k) or (k == "select" and s.get(k))
                    or (k in ("tail_bias_from", "rescale") and s.get(k) is not None)]
            if diff:
                raise EvalError(f"arm {s['name']} reuses the fill of {src['name']} but its P or fill can differ "
                                f"({', '.join(diff)})")
        by_name[s["name"]] = s


def check_tail_round(specs):
    for s in specs:
        tr = s.get("tail_round")
        if tr is None:
            continue
        bad = []
        if not (isinstance(tr, dict) and set(tr) == {"base", "block"} and type(tr["base"]) is int
                and type(tr["block"]) is int):
            bad.append(f"{tr!r} is not {{'base': int, 'block': int}}")
        else:
            if tr["base"] != s.get("tail") or tr["base"] < ENGINE_MIN_TAIL:
                bad.append(f"base {tr['base']} must equal the arm's tail ({s.get('tail')}) and be at least "
                           f"{ENGINE_MIN_TAIL}")
            if tr["block"] < 1:
                bad.append(f"block {tr['block']} must be positive")
        if s.get("select"):
            bad.append("with a select the rows would be picked against the unrounded boundary")
        if s.get("tail_from") is not None:
            bad.append("tail_from sets the tail per prompt")
        if bad:
            raise EvalError(f"arm {s['name']}: tail_round refused: " + "; ".join(bad))


def check_tail_from(spec):
    tf = spec.get("tail_from")
    if tf is not None and (tf != "continuation" or "tail" in spec or spec.get("select") or spec.get("tail_round")
                           or spec.get("reuse_fill")):
        raise EvalError(f"arm {spec['name']}: tail_from 'continuation' sets the tail per prompt: no 'tail', select, "
                        "tail_round or reuse_fill")


class Files:
    """Map files, corrections, predictors and frequency tables, each loaded once; their sha256 recorded. A map file
    is checked against the sha256 that the fit records give for it (the JSON files under `records`, default the map
    file's own directory, where the fit writes them) when they name it, else against its disk copy."""

    def __init__(self, device, records=None):
        self.device = device
        self.records = records
        self.maps, self.st, self.pred, self.freq, self.hashes = {}, {}, {}, {}, {}

    def projector(self, path, kind="proj"):
        from ..ridge.projector import KVFold, Projector
        from ..utils.integrity import recorded_sha256
        if path not in self.maps:
            cls = KVFold if kind == "kvfold" else Projector
            recs = self.records or Path(path).parent        # fit records sit beside the maps they describe
            ref = None if Path(path).is_dir() else recorded_sha256(path, recs)
            self.maps[path] = cls.load(path, "cpu", sha256=ref)
            self.hashes[path] = self.maps[path].sha256
        return self.maps[path]

    def correction(self, path):
        from ..ridge.projector import load_st
        from ..utils.prov import sha256
        if path not in self.st:
            self.st[path] = load_st(path, self.device)
            self.hashes[path] = sha256(path)
        return self.st[path]

    def predictor(self, path):
        from ..engine.pred import Predictor
        from ..utils.prov import sha256
        if path not in self.pred:
            self.pred[path] = Predictor.load(path)
            self.hashes[path] = sha256(path)
        return self.pred[path]

    def table(self, path):
        from ..engine.pred import load_freq
        from ..utils.prov import sha256
        if path not in self.freq:
            self.freq[path] = load_freq(path)
            self.hashes[path] = sha256(path)
        return self.freq[path]


def build_arm(spec, files):
    check_tail_from(spec)
    a = Arm(spec["name"], split=spec.get("split"), tail=spec.get("tail", 0), fill=spec.get("fill", "exact"),
            tail_from=spec.get("tail_from"), f1=spec.get("f1", False), fill_by_type=spec.get("fill_by_type"),
            tail_bias_from=spec.get("tail_bias_from"), tail_bias_skip_last=spec.get("tail_bias_skip_last", 0),
            exact_part=spec.get("exact_part"), rescale=spec.get("rescale"),
            rescale_skip_last=spec.get("rescale_skip_last", 0), meta=dict(spec))
    if spec.get("projector"):
        a.projector = files.projector(spec["projector"])
        if a.projector.split != a.split:
            raise EvalError(f"arm {a.name}: {spec['projector']} is for split {a.projector.split}, not {a.split}")
        a.context = spec.get("context", 0)
        if int(a.projector.meta.get("context", 0)) != a.context:
            raise EvalError(f"arm {a.name}: context {a.context}, but {spec['projector']} reads context "
                            f"{a.projector.meta.get('context', 0)}")
    if spec.get("refresh") is not None:
        a.refresh, a.refresh_projector = spec["refresh"], files.projector(spec["refresh_projector"])
        if a.refresh_projector.split != a.refresh + 1 or int(a.refresh_projector.meta.get("context", 0)):
            raise EvalError(f"arm {a.name}: refresh {a.refresh} needs a plain projector of split {a.refresh + 1}")
    if spec.get("kvfold"):
        a.kvfold = files.projector(spec["kvfold"], "kvfold")
        if a.kvfold.split != a.split:
            raise EvalError(f"arm {a.name}: {spec['kvfold']} is for split {a.kvfold.split}, not {a.split}")
    if spec.get("st"):
        a.st = files.correction(spec["st"])
    return a


def check_selects(arms, files):
    by_name = {a.name: a for a in arms}
    for a in arms:
        sel = a.meta.get("select")
        if not sel:
            continue
        sig = SEL.signals(sel)
        if (sel["kind"] not in SEL.KINDS or (sel.get("match") in by_name) != (sel["kind"] in ("random", "tail_match"))
                or bool(sel.get("predictor")) != ("pred" in sig) or bool(sel.get("table")) != bool(sig & {"freq", "frag"})):
            raise EvalError(f"arm {a.name}: bad select spec {sel}")
        if sel.get("table"):
            files.table(sel["table"])
        if sel.get("predictor") and files.predictor(sel["predictor"]).split != a.split:
            raise EvalError(f"arm {a.name}: predictor {sel['predictor']} is not for split {a.split}")
        if "deviation" in sig:
            q = sel.get("projector")
            proj = files.projector(q) if q else a.projector
            if proj is None or proj.split != a.split:
                raise EvalError(f"arm {a.name}: deviation needs a projector of split {a.split}")


# ---------------------------------------------------------------------------------------------- prompts
def set_prompts(set_name, cfg, tok, model_name, protocol):
    """(prompts, run_cfg additions) of one set."""
    from . import locked, niahg
    run_cfg = {}
    fmt = cfg.get("niah_format", "raw")
    if set_name == "decode":
        source = cfg.get("decode_from")
        if source == "grade":
            src = TX.grade_prompts(tok, cfg.get("grade_format", "raw"))
        else:
            src, run_cfg["skipped"] = locked.prompts(source, tok, cfg, model_name, protocol)
            run_cfg["longppl_max_len"] = cfg.get("longppl_max_len")
        out = []
        for q in src:
            cut = TX.SCORED if source == "grade" else q["cont_len"]
            out.append(dict(name=q["name"], ids=list(q["ids"][:len(q["ids"]) - cut]), decode_from=source, cut=cut,
                            **{k: q[k] for k in ("kind", "task", "length", "source", "source_sha256", "format")
                               if k in q}))
        run_cfg.update(decode_from=source, decode_steps=cfg.get("decode_steps", DECODE_STEPS))
        return out, run_cfg
    if set_name == "grade":
        return TX.grade_prompts(tok, cfg.get("grade_format", "raw"), drop_bos=bool(cfg.get("drop_bos"))), run_cfg
    if set_name == "niah":
        return TX.niah_prompts(tok, fmt, cfg.get("niah_variant")), run_cfg
    if set_name == "multiturn":
        if cfg.get("multiturn_from", "mk4") == "ruler":
            from . import derived
            if cfg.get("multiturn_turns", 4) != 2:
                raise EvalError("the two-key RULER set has 2 turns: multiturn_turns 2")
            fmt = locked.fmt_of(cfg, model_name, protocol)
            out, run_cfg["skipped"] = derived.prompts("twokey", tok, fmt, locked.manifest(), cfg.get("ruler_max_len"))
            run_cfg.update(multiturn_from="ruler", ruler_max_len=cfg.get("ruler_max_len"))
            return out, run_cfg
        if cfg.get("niah_variant") != "mk4":
            raise EvalError("the multiturn set needs niah_variant mk4 (the distractor keys are the later turns)")
        return TX.niah_prompts(tok, fmt, "mk4"), run_cfg
    if set_name in locked.SETS:
        out, run_cfg["skipped"] = locked.prompts(set_name, tok, cfg, model_name, protocol)
        for k in ("ruler_max_len", "longbench_max_len", "longppl_max_len", "ruler_max_new", "ruler_variant", "dataset",
                  "dataset_manifest_sha256"):
            if cfg.get(k) is not None:
                run_cfg[k] = cfg.get(k)
        return out, run_cfg
    if set_name == "niahg":
        return niahg.prompts(tok, fmt, cfg.get("niahg_types", niahg.TYPES)), run_cfg
    raise EvalError(f"set {set_name!r}: one of {SETS}")


def _complete(run, set_name):
    if set_name in ("grade", "longppl"):
        return "logprobs" in run
    if set_name == "decode":
        return "gen" in run
    if set_name == "multiturn":
        return "turns" in run
    return "gen" in run


def gen_budget(set_name, q, steps_dec, turns):
    steps_q = q.get("max_new", NIAH_STEPS)
    if set_name in ("grade", "longppl"):
        return 0
    if set_name == "decode":
        return steps_dec
    if set_name == "multiturn":
        return (turns - 1) * (TURN_ROWS - NIAH_STEPS + steps_q) + steps_q
    return steps_q


# ---------------------------------------------------------------------------------------------- runner
class Harness:
    def __init__(self, model, tok, cfg, set_name, out_dir, files=None, eos=(), log=print):
        if set_name not in SETS:
            raise EvalError(f"set {set_name!r}: one of {SETS}")
        self.m, self.tok, self.cfg, self.set = model, tok, cfg, set_name
        self.out = Path(out_dir)
        self.files = files or Files(model.device, cfg.get("fit_records"))
        self.eos = tuple(eos)
        self.log = log
        self.fmt = cfg.get("niah_format", "raw")
        kt = cfg.get("keytoken_tail")
        if kt is not None and not isinstance(kt, int):
            raise EvalError(f"keytoken_tail {kt!r}: an integer (grade and longppl)")
        self.key_tail = kt if set_name in ("grade", "longppl") else None
        self.turns = cfg.get("multiturn_turns", 4)
        if self.turns not in (2, 3, 4):
            raise EvalError(f"multiturn_turns {self.turns!r}: 2, 3 or 4")
        self.steps_dec = cfg.get("decode_steps", DECODE_STEPS)
        if not isinstance(self.steps_dec, int) or self.steps_dec < 1:
            raise EvalError(f"decode_steps {self.steps_dec!r}: a positive integer")
        if set_name == "decode" and cfg.get("decode_from") not in DECODE_FROM:
            raise EvalError(f"the decode set needs 'decode_from' in {DECODE_FROM}, got {cfg.get('decode_from')!r}")
        if cfg.get("multiturn_from", "mk4") not in MULTITURN_FROM:
            raise EvalError(f"multiturn_from {cfg.get('multiturn_from')!r}: one of {MULTITURN_FROM}")
        if cfg.get("drop_bos") and set_name != "grade":
            raise EvalError("drop_bos runs on the grade set only")
        if cfg.get("dataset") is not None and set_name != "longppl":
            raise EvalError(f"dataset {cfg['dataset']!r} replaces the locked set for longppl only, not {set_name!r}")
        from . import multiturn as MT
        specs = [s for s in cfg["arms"] if set_name in s.get("sets", SETS)]
        check_reuse(specs)
        check_tail_round(specs)
        try:
            MT.check_arms(specs, set_name)
        except MT.MultiturnError as e:
            raise EvalError(str(e))
        self.arms = [build_arm(s, self.files) for s in specs]
        if not self.arms:
            raise EvalError(f"no arm of the config runs on the {set_name} set")
        self.by_name = {a.name: a for a in self.arms}
        check_selects(self.arms, self.files)
        sels = [a.meta["select"] for a in self.arms if a.meta.get("select")]
        self.lexical = any(SEL.signals(s) & {"freq", "frag", "regex", "verbatim"} for s in sels)
        need_digits = self.lexical or any(s["kind"] == "digits" for s in sels)
        self.digit_set = SEL.digit_ids(tok) if need_digits else None
        self.breaks = SEL.word_breaks(tok) if any("frag" in SEL.signals(s) for s in sels) else None
        self.tbytes = SEL.token_bytes(tok) if any(SEL.signals(s) & {"regex", "verbatim"} for s in sels) else None
        self.exact_split = max(a.split for a in self.arms if a.split is not None) if any(
            a.split is not None for a in self.arms) else model.n_layers

    # -- checks before the run
    def check_prompts(self, prompts):
        from . import locked
        from .keytok import check_tail
        if self.set == "longppl":
            locked.check_tails(prompts, {a.name: (lambda q, a=a: len(q["ids"]) - a.prefix_len(len(q["ids"]))
                                                  if not a.tail_from else q["cont_len"] + 1) for a in self.arms})
        mp = getattr(self.m, "max_positions", None)
        for q in prompts:
            g = gen_budget(self.set, q, self.steps_dec, self.turns)
            if mp and len(q["ids"]) + g > mp:
                raise EvalError(f"PositionsExceeded: {q['name']}: {len(q['ids'])} prompt ids + up to {g} more exceed "
                                f"max_position_embeddings {mp}")
        if self.key_tail is not None:
            for q in prompts:
                scored = TX.SCORED if self.set == "grade" else q["cont_len"]
                try:
                    check_tail(len(q["ids"]), scored, self.key_tail, self._bos_of(q["ids"]))
                except ValueError as e:
                    raise EvalError(f"{q['name']}: {e}")

    def _bos_of(self, ids):
        b = TX.bos_ids(self.tok)
        return list(ids[:1]) if b and ids[0] == b[0] else []

    # -- one prompt
    def run(self, prompts, provenance=None):
        self.check_prompts(prompts)
        done = 0
        for p in prompts:
            path = self.out / f"{p['name']}.json"
            rec = json.loads(path.read_text()) if path.exists() else None
            want = ["exact"] + [a.name for a in self.arms]
            ids_sha = hashlib.sha256(json.dumps(list(p["ids"])).encode()).hexdigest()
            if (rec and rec.get("ids_sha256") == ids_sha and all(
                    n in rec["runs"] and _complete(rec["runs"][n], self.set) for n in want)
                    and (self.key_tail is None or rec.get("tail_only", {}).get("T") == self.key_tail)):
                continue
            if rec is None or rec.get("ids_sha256") != ids_sha:
                rec = dict(name=p["name"], n=len(p["ids"]), ids_sha256=ids_sha, runs={}, provenance=[],
                           **{k: v for k, v in p.items() if k not in ("ids", "short_ids", "name", "asks")})
            if provenance is not None:
                rec["provenance"].append(provenance)
            t0 = time.time()
            msg = self.run_prompt(p, rec)
            self._write(path, rec)
            self.log(f"{p['name']} n={len(p['ids'])} {time.time() - t0:.1f}s | {msg}")
            done += 1
        return done

    def _write(self, path, rec):
        from ..utils.prov import write_json
        write_json(path, rec)

    @torch.no_grad()
    def run_prompt(self, p, rec):
        m, tok = self.m, self.tok
        if self.set == "multiturn":
            from . import multiturn as MT
            return MT.run_prompt(m, tok, p, self.arms, rec, self.fmt, self.eos, p.get("max_new", NIAH_STEPS),
                                 self.digit_set, self.turns)
        ids = torch.tensor(list(p["ids"]))
        n = ids.shape[0]
        keep = KEEP if self.set == "grade" else p["cont_len"] + 1 if self.set == "longppl" else 1
        scored = keep - 1 if self.set in ("grade", "longppl") else 0
        known = n - scored
        todo = [Arm("exact", split=self.exact_split)] + sorted(self.arms, key=lambda x: -(x.split or 0))
        todo = [a for a in todo if not (a.name in rec["runs"] and _complete(rec["runs"][a.name], self.set))]
        todo = [dataclasses.replace(a, tail=keep) if a.tail_from else a for a in todo]
        todo = [exclude_scored(a, scored) for a in todo]
        if self.set == "decode" and todo and todo[0].name != "exact":
            todo.insert(0, Arm("exact", split=self.exact_split))
        refs = [self.by_name[a.meta["select"]["match"]] for a in todo if "match" in a.meta.get("select", {})]
        oracle, tap = None, None
        if any(a.uses_oracle() for a in todo):
            if todo[0].name != "exact":
                todo.insert(0, Arm("exact", split=self.exact_split))
            oracle = {}
            tap = oracle_tap(oracle, min(a.split for a in todo if a.uses_oracle()),
                             max(a.prefix_len(n) for a in todo if a.uses_oracle()))
        need = sorted({a.split for a in todo + refs if a.split is not None})
        ends = {known}
        for b in todo + refs:
            sel = b.meta.get("select", {})
            if sel and "qattn" in SEL.signals(sel) and sel.get("window") == "prefix":
                ends.add(b.prefix_len(n))
        wins = {e: {} for e in ends}
        want_win = any("qattn" in SEL.signals(b.meta["select"]) for b in todo + refs if b.meta.get("select"))
        recv_P = sorted({b.prefix_len(n) for b in todo + refs if b.meta.get("select")
                         and "qfp" in SEL.signals(b.meta["select"])})
        recv = {}
        pos_all = torch.arange(n, device=m.device)

        def lower_hook(i, h):
            if tap is not None:
                tap(i, h)
            if want_win:
                for end, win in wins.items():
                    win[i] = h[max(0, end - SEL.WINDOW):end].clone()
            if recv_P and isinstance(i, int) and m.layer_types[i] == "attn":
                from ..engine import impact as IM
                x = m.in_norm(h, m.W[i]["ln1"])
                q, k = m.queries(i, x, pos_all), IM.attn_kv(m, i, x, pos_all)[0]
                for P_ in recv_P:
                    recv[(P_, i)] = IM.received_mass(q, k, m.scale, rows_below=P_,
                                                     stride=int(self.cfg.get("qfp_stride", 1)))[1]
        mixes = {}
        mix_layers = {a.split - k for a in todo for k in range(1, a.context + 1)}
        hs, lower = run_lower(m, ids, set(need) if need else {self.exact_split},
                              hook=lower_hook if (tap is not None or want_win or recv_P) else None,
                              mix=(lambda i, x: mixes.__setitem__(i, x) if i in mix_layers else None)
                              if mix_layers else None)
        masses, scores, emb = {}, {}, []

        def mass_of(split, layers, end):
            key = (tuple(SEL.qattn_layers(m, split, layers)), end)
            if key not in masses:
                masses[key] = SEL.window_mass(m, wins[end], lower, key[0], end)
            return masses[key]

        def pred_of(split, path, P):
            from ..engine.pred import prefix_scores
            if not emb:
                emb.append(m.embed(ids.to(m.device)))
            if (split, path, P) not in scores:
                scores[split, path, P] = prefix_scores(self.files.predictor(path), hs[split], emb[0], P)
            return scores[split, path, P]

        def keys_of(split, layers, P):
            key = ("keydiff", tuple(SEL.qattn_layers(m, split, layers)), P)
            if key not in scores:
                scores[key] = SEL.key_diff(lower, key[1], P)
            return scores[key]

        def dev_of(a, P):
            q = a.meta["select"].get("projector")
            proj = self.files.projector(q) if q else a.projector
            key = ("deviation", id(proj), a.split, P)
            if key not in scores:
                scores[key] = SEL.fill_deviation(m, proj, hs[a.split], a.split, P)
            return scores[key]

        def recv_of(split, P_):
            low = sum(v for (pp, i), v in recv.items() if pp == P_ and i < split)
            return SEL.per_later_token(low, P_)
        picks = SEL.choose(todo + refs, n, list(p["ids"]), p["name"], self.digit_set, mass_of, pred_of, keys_of,
                           dev_of, self.files.freq.get, self.breaks, recv_of, self.tbytes, known=known)
        fills, ref_dec = {}, None
        for j, a in enumerate(todo):
            t1 = time.time()
            if m.device.type == "cuda":
                torch.cuda.reset_peak_memory_stats()
            store = {} if any(b.meta.get("reuse_fill") == a.name for b in todo[j + 1:]) else None
            reuse = fills.pop(a.meta.get("reuse_fill"), None)
            pick = picks.get(a.name)
            run_arm = dataclasses.replace(a, tail=a.tail + pick["extra_tail"]) if pick else a
            if a.meta.get("tail_round"):
                tr = a.meta["tail_round"]
                run_arm = dataclasses.replace(run_arm, tail=rounded_tail(n, tr["base"], tr["block"]))
            logits, cache, P = finish(m, ids, hs[a.split], lower, run_arm, keep, keep_cache=keep == 1,
                                      fill_store=store, fill_reuse=reuse, oracle=oracle,
                                      exact_rows=pick["rows"] if pick else None,
                                      hook=tap if a.name == "exact" else None, mix=mixes or None)
            check_finite(logits, f"{p['name']} {a.name}")
            if store is not None:
                fills[a.name] = store
            run = self._run_fields(a, P, n, pick, p)
            self._score(run, a, p, ids, n, keep, logits, cache, P, rec, ref_dec)
            if self.set == "decode" and a.name == "exact":
                ref_dec = run.pop("_ref")
            run["wall_s"] = round(time.time() - t1, 3)
            if m.device.type == "cuda":
                run["mem_gib"] = dict(alloc_peak=round(torch.cuda.max_memory_allocated() / 2**30, 2),
                                      reserved_peak=round(torch.cuda.max_memory_reserved() / 2**30, 2))
            rec["runs"][a.name] = run
            del logits, cache
            rest = {b.split for b in todo[j + 1:]}
            top = max(rest) if rest else 0
            for i in range(top, len(lower)):
                lower[i] = {}
        if self.key_tail is not None and rec.get("tail_only", {}).get("T") != self.key_tail:
            from .keytok import exact_tail_only
            sc = KEEP - 1 if self.set == "grade" else p["cont_len"]
            bos = self._bos_of(p["ids"])
            rec["tail_only"] = dict(T=self.key_tail, bos=bos, logprobs=[
                round(float(x), 6) for x in exact_tail_only(m, list(p["ids"]), self.key_tail, bos, sc)])
        if self.set == "grade" and "short" not in rec and "short_ids" in p:
            s = torch.tensor(p["short_ids"])
            lg, _ = m.forward_exact(s.to(m.device), keep=torch.arange(s.shape[0] - KEEP, s.shape[0], device=m.device))
            rec["short"] = dict(n=s.shape[0], tail_match=p.get("short_tail_match"),
                                logprobs=[round(float(x), 6) for x in score_tokens(lg, s, KEEP - 1)])
        return self._summary(rec)

    def _run_fields(self, a, P, n, pick, p):
        run = dict(P=P, split=a.split, tail=n - P, fill=a.fill, st=bool(a.st), f1=a.f1)
        if a.tail_from:
            run["tail_from"] = a.tail_from
        if a.context or a.refresh is not None:
            run.update(context=a.context, refresh=a.refresh)
        if a.tail_bias_from is not None:
            run.update(tail_bias_from=a.tail_bias_from, tail_bias_skip_last=a.tail_bias_skip_last)
        if a.exact_part is not None:
            run["exact_part"] = a.exact_part
        if a.rescale is not None:
            run.update(rescale=a.rescale, rescale_skip_last=a.rescale_skip_last)
        if a.fill_by_type:
            run["fill_by_type"] = a.fill_by_type
        if pick:
            rows = pick["rows"]
            run.update(select=pick["kind"], n_rows=len(rows), tail_extra=pick["extra_tail"], rows=SEL.ranges(rows))
            for k in ("overlap", "window_end"):
                if k in pick:
                    run[k] = pick[k]
            ids = list(p["ids"])
            if self.lexical:
                run["digit_rows"] = sum(int(ids[r]) in self.digit_set for r in rows)
                run["digit_share"] = round(run["digit_rows"] / len(rows), 4) if rows else None
            if "needle_start" in p:
                run["needle_rows_exact"] = sum(p["needle_start"] <= r < p["needle_end"] for r in rows)
            if self.set == "niahg" and "value_start" in p:
                run["value_rows_exact"] = sum(p["value_start"] <= r < p["value_end"] for r in rows)
        return run

    def _score(self, run, a, p, ids, n, keep, logits, cache, P, rec, ref_dec):
        from . import locked, niahg
        m, tok = self.m, self.tok
        if self.set in ("grade", "longppl"):
            run["logprobs"] = [round(float(x), 6) for x in score_tokens(logits, ids, keep - 1)]
            if self.set == "grade":
                run["argmax"] = logits[:-1].argmax(-1).tolist()
            else:
                run.update(score=locked.nll(run["logprobs"]), metric="nll")
            old = rec["runs"].get(a.name)
            if old is not None and "logprobs" in old:
                run["rescore_max_abs_logprob_diff"] = max(abs(x - y) for x, y in zip(run["logprobs"], old["logprobs"]))
                run["first_run"] = {k: v for k, v in old.items() if k in ("logprobs", "wall_s")}
        elif self.set == "decode":
            if a.name == "exact":
                fields, ref = AG.exact_record(m, n, cache, logits, self.steps_dec, a, self.eos)
                run.update(fields)
                run["_ref"] = ref
            else:
                run.update(AG.compare(m, n, cache, logits, self.steps_dec, a, *ref_dec))
        else:
            from ..engine.decode import greedy
            gen, reason = greedy(m, ids.to(m.device), cache, logits, p.get("max_new", NIAH_STEPS), a, self.eos)
            text = tok.decode(gen, skip_special_tokens=False)
            run.update(gen=gen, text=text, finish_reason=reason)
            if self.set in locked.GEN_SETS:
                run.update(locked.score(p, tok.decode(gen, skip_special_tokens=True)))
            elif self.set == "niah":
                run["needle_projected"] = p["needle_end"] <= P
                run["correct"] = TX.niah_correct(text, p["value"])
            else:
                run["needle_projected"] = p["needle_end"] <= P
                run.update(niahg.score(text, p["value"], p["type"], self.fmt))

    def _summary(self, rec):
        runs = rec["runs"]
        if self.set == "grade" and "novel" in rec:
            nov = rec["novel"]

            def nll(lp):
                xs = [-x for x, k in zip(lp, nov) if k]
                return sum(xs) / max(1, len(xs))
            ex = nll(runs["exact"]["logprobs"])
            return " ".join(f"{k}:{nll(r['logprobs']) - ex:+.4f}" for k, r in runs.items() if k != "exact")
        if self.set == "longppl":
            ex = runs["exact"]["score"]
            return " ".join(f"{k}:{r['score'] - ex:+.4f}" for k, r in runs.items() if k != "exact")
        if self.set in ("ruler", "longbench"):
            return " ".join(f"{k}:{r['score']:.2f}" for k, r in runs.items())
        if self.set == "decode":
            return " ".join(f"{k}: same {r['frac_identical']:.3f} div@{r['first_divergence']} kl {r['kl_mean']:.4g}"
                            for k, r in runs.items() if k != "exact")
        return " ".join(f"{k}:{'ok' if r.get('correct') else 'MISS'}{'*' if r.get('needle_projected') else ''}"
                        for k, r in runs.items())
