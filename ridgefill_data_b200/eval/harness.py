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
# keys whose equality makes two arms' prefix fills (and P) identical
_FILL_KEYS = ("split", "tail", "tail_round", "tail_from", "fill", "fill_by_type", "projector", "kvfold", "select",
              "context", "refresh", "refresh_projector", "tail_bias_from", "tail_bias_skip_last", "exact_part",
              "rescale", "rescale_skip_last")
_PER_PROMPT_KEYS = ("select", "tail_bias_from", "rescale")       # set at all, they make the fill prompt-specific


def check_reuse(specs):
    """reuse_fill names an earlier arm whose fill this arm may take over: same P, same maps, same fill, and
    nothing that computes the fill from the prompt's tail or selection."""
    earlier = {}
    for spec in specs:
        name = spec.get("reuse_fill")
        if "reuse_fill" in spec and name not in earlier:
            raise EvalError(f"arm {spec['name']}: reuse_fill {name!r} is not an earlier arm")
        if name in earlier:
            src = earlier[name]
            differs = [k for k in _FILL_KEYS if spec.get(k) != src.get(k)
                       or (k in _PER_PROMPT_KEYS and (spec.get(k) if k == "select" else spec.get(k) is not None))]
            if differs:
                raise EvalError(f"arm {spec['name']} reuses the fill of {src['name']} but its P or fill can differ "
                                f"({', '.join(differs)})")
        earlier[spec["name"]] = spec


def _tail_round_problems(spec, tr):
    if not isinstance(tr, dict) or set(tr) != {"base", "block"} or type(tr["base"]) is not int \
            or type(tr["block"]) is not int:
        yield f"{tr!r} is not {{'base': int, 'block': int}}"
    else:
        if tr["base"] != spec.get("tail") or tr["base"] < ENGINE_MIN_TAIL:
            yield (f"base {tr['base']} must equal the arm's tail ({spec.get('tail')}) and be at least "
                   f"{ENGINE_MIN_TAIL}")
        if tr["block"] < 1:
            yield f"block {tr['block']} must be positive"
    if spec.get("select"):
        yield "with a select the rows would be picked against the unrounded boundary"
    if spec.get("tail_from") is not None:
        yield "tail_from sets the tail per prompt"


def check_tail_round(specs):
    """tail_round {base, block}: the tail grows so the prefix ends on a block multiple (as a block engine runs)."""
    for spec in specs:
        if spec.get("tail_round") is None:
            continue
        problems = list(_tail_round_problems(spec, spec["tail_round"]))
        if problems:
            raise EvalError(f"arm {spec['name']}: tail_round refused: " + "; ".join(problems))


def check_tail_from(spec):
    """tail_from 'continuation' makes every prompt's tail its scored continuation: nothing else may set it."""
    tf = spec.get("tail_from")
    if tf is None:
        return
    clashes = "tail" in spec or any(spec.get(k) for k in ("select", "tail_round", "reuse_fill"))
    if tf != "continuation" or clashes:
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


_ARM_FIELDS = {"split": None, "tail": 0, "fill": "exact", "tail_from": None, "f1": False, "fill_by_type": None,
               "tail_bias_from": None, "tail_bias_skip_last": 0, "exact_part": None, "rescale": None,
               "rescale_skip_last": 0}


def _same_split(arm, maps, path):
    if maps.split != arm.split:
        raise EvalError(f"arm {arm.name}: {path} is for split {maps.split}, not {arm.split}")


def build_arm(spec, files):
    """An Arm from a JSON arm spec, its map files loaded (once) through `files` and checked against the arm."""
    check_tail_from(spec)
    a = Arm(spec["name"], meta=dict(spec), **{k: spec.get(k, default) for k, default in _ARM_FIELDS.items()})
    if spec.get("projector"):
        a.projector = files.projector(spec["projector"])
        _same_split(a, a.projector, spec["projector"])
        a.context = spec.get("context", 0)
        fitted = int(a.projector.meta.get("context", 0))
        if fitted != a.context:
            raise EvalError(f"arm {a.name}: context {a.context}, but {spec['projector']} reads context {fitted}")
    if spec.get("refresh") is not None:
        a.refresh = spec["refresh"]
        a.refresh_projector = files.projector(spec["refresh_projector"])
        plain = int(a.refresh_projector.meta.get("context", 0)) == 0
        if a.refresh_projector.split != a.refresh + 1 or not plain:
            raise EvalError(f"arm {a.name}: refresh {a.refresh} needs a plain projector of split {a.refresh + 1}")
    if spec.get("kvfold"):
        a.kvfold = files.projector(spec["kvfold"], "kvfold")
        _same_split(a, a.kvfold, spec["kvfold"])
    if spec.get("st"):
        a.st = files.correction(spec["st"])
    return a


def _select_ok(sel, sig, by_name):
    matched = sel["kind"] in ("random", "tail_match")
    return (sel["kind"] in SEL.KINDS
            and (sel.get("match") in by_name) == matched
            and bool(sel.get("predictor")) == ("pred" in sig)
            and bool(sel.get("table")) == bool(sig & {"freq", "frag"}))


def check_selects(arms, files):
    """Every select spec is well formed and its predictor, table or deviation maps exist for the arm's split."""
    by_name = {a.name: a for a in arms}
    for a in (x for x in arms if x.meta.get("select")):
        sel = a.meta["select"]
        sig = SEL.signals(sel)
        if not _select_ok(sel, sig, by_name):
            raise EvalError(f"arm {a.name}: bad select spec {sel}")
        if sel.get("table"):
            files.table(sel["table"])
        if sel.get("predictor") and files.predictor(sel["predictor"]).split != a.split:
            raise EvalError(f"arm {a.name}: predictor {sel['predictor']} is not for split {a.split}")
        if "deviation" in sig:
            path = sel.get("projector")
            maps = files.projector(path) if path else a.projector
            if maps is None or maps.split != a.split:
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
class _Signals:
    """One prompt's exact lower layers, shared by every arm, and the selection signals read from them (each
    computed once, on first use): window attention mass, predicted surprisal, key diversity, fill deviation and
    the attention a row receives from later prefix rows."""

    def __init__(self, h, ids, todo, refs, known):
        self.m, self.files = h.m, h.files
        m = h.m
        n = ids.shape[0]
        self.ids = ids
        every = todo + refs
        selects = [b.meta["select"] for b in every if b.meta.get("select")]
        self.oracle, self.tap = None, None
        readers = [a for a in todo if a.uses_oracle()]
        if readers:
            self.oracle = {}
            self.tap = oracle_tap(self.oracle, min(a.split for a in readers), max(a.prefix_len(n) for a in readers))
        ends = {known} | {b.prefix_len(n) for b in every if b.meta.get("select")
                          and "qattn" in SEL.signals(b.meta["select"]) and b.meta["select"].get("window") == "prefix"}
        self.windows = {e: {} for e in ends}
        self.want_windows = any("qattn" in SEL.signals(s) for s in selects)
        self.recv_P = sorted({b.prefix_len(n) for b in every if b.meta.get("select")
                              and "qfp" in SEL.signals(b.meta["select"])})
        self.recv = {}
        self.qfp_stride = int(h.cfg.get("qfp_stride", 1))
        self.pos = torch.arange(n, device=m.device)
        self.mixes = {}
        mix_layers = {a.split - k for a in todo for k in range(1, a.context + 1)}

        def keep_mix(i, x):
            if i in mix_layers:
                self.mixes[i] = x
        splits = {a.split for a in every if a.split is not None} or {h.exact_split}
        hooked = self.tap is not None or self.want_windows or bool(self.recv_P)
        self.hs, self.lower = run_lower(m, ids, splits, hook=self._lower_hook if hooked else None,
                                        mix=keep_mix if mix_layers else None)
        self.cached = {}
        self.emb = None

    def _lower_hook(self, i, h):
        m = self.m
        if self.tap is not None:
            self.tap(i, h)
        if self.want_windows:
            for end, rows in self.windows.items():
                rows[i] = h[max(0, end - SEL.WINDOW):end].clone()
        if self.recv_P and isinstance(i, int) and m.layer_types[i] == "attn":
            from ..engine import impact as IM
            x = m.in_norm(h, m.W[i]["ln1"])
            q, k = m.queries(i, x, self.pos), IM.attn_kv(m, i, x, self.pos)[0]
            for P_ in self.recv_P:
                self.recv[P_, i] = IM.received_mass(q, k, m.scale, rows_below=P_, stride=self.qfp_stride)[1]

    def _once(self, key, make):
        if key not in self.cached:
            self.cached[key] = make()
        return self.cached[key]

    def mass(self, split, layers, end):
        used = tuple(SEL.qattn_layers(self.m, split, layers))
        return self._once(("mass", used, end),
                          lambda: SEL.window_mass(self.m, self.windows[end], self.lower, used, end))

    def pred(self, split, path, P):
        from ..engine.pred import prefix_scores
        if self.emb is None:
            self.emb = self.m.embed(self.ids.to(self.m.device))
        return self._once(("pred", split, path, P),
                          lambda: prefix_scores(self.files.predictor(path), self.hs[split], self.emb, P))

    def keydiff(self, split, layers, P):
        used = tuple(SEL.qattn_layers(self.m, split, layers))
        return self._once(("keydiff", used, P), lambda: SEL.key_diff(self.lower, used, P))

    def deviation(self, a, P):
        path = a.meta["select"].get("projector")
        proj = self.files.projector(path) if path else a.projector
        return self._once(("deviation", id(proj), a.split, P),
                          lambda: SEL.fill_deviation(self.m, proj, self.hs[a.split], a.split, P))

    def received(self, split, P_):
        below = sum(v for (pp, i), v in self.recv.items() if pp == P_ and i < split)
        return SEL.per_later_token(below, P_)

    def release_below(self, top):
        """Drop the lower-layer caches from layer `top` up once no remaining arm reads them."""
        for i in range(top, len(self.lower)):
            self.lower[i] = {}


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
    def _plan(self, p, rec, n, keep, scored):
        """The arms still to run on this prompt (exact first where others need it) and the matched arms their
        controls read."""
        exact = Arm("exact", split=self.exact_split)
        todo = [exact] + sorted(self.arms, key=lambda x: -(x.split or 0))
        todo = [a for a in todo if not (a.name in rec["runs"] and _complete(rec["runs"][a.name], self.set))]
        todo = [exclude_scored(dataclasses.replace(a, tail=keep) if a.tail_from else a, scored) for a in todo]
        needs_exact = self.set == "decode" or any(a.uses_oracle() for a in todo)
        if todo and needs_exact and todo[0].name != "exact":
            todo.insert(0, exact)
        refs = [self.by_name[a.meta["select"]["match"]] for a in todo if "match" in a.meta.get("select", {})]
        return todo, refs

    def run_prompt(self, p, rec):
        m = self.m
        if self.set == "multiturn":
            from . import multiturn as MT
            return MT.run_prompt(m, self.tok, p, self.arms, rec, self.fmt, self.eos, p.get("max_new", NIAH_STEPS),
                                 self.digit_set, self.turns)
        ids = torch.tensor(list(p["ids"]))
        n = ids.shape[0]
        if self.set == "grade":
            keep = KEEP
        elif self.set == "longppl":
            keep = p["cont_len"] + 1
        else:
            keep = 1
        scored = keep - 1 if self.set in ("grade", "longppl") else 0
        todo, refs = self._plan(p, rec, n, keep, scored)
        sig = _Signals(self, ids, todo, refs, known=n - scored)
        picks = SEL.choose(todo + refs, n, list(p["ids"]), p["name"], self.digit_set, sig.mass, sig.pred,
                           sig.keydiff, sig.deviation, self.files.freq.get, self.breaks, sig.received, self.tbytes,
                           known=n - scored)
        saved_fills, ref_dec = {}, None
        for j, a in enumerate(todo):
            later = todo[j + 1:]
            started = time.time()
            on_gpu = m.device.type == "cuda"
            if on_gpu:
                torch.cuda.reset_peak_memory_stats()
            pick = picks.get(a.name)
            arm = a if not pick else dataclasses.replace(a, tail=a.tail + pick["extra_tail"])
            rounding = a.meta.get("tail_round")
            if rounding:
                arm = dataclasses.replace(arm, tail=rounded_tail(n, rounding["base"], rounding["block"]))
            store = {} if any(b.meta.get("reuse_fill") == a.name for b in later) else None
            logits, cache, P = finish(m, ids, sig.hs[a.split], sig.lower, arm, keep, keep_cache=keep == 1,
                                      fill_store=store, fill_reuse=saved_fills.pop(a.meta.get("reuse_fill"), None),
                                      oracle=sig.oracle, exact_rows=pick["rows"] if pick else None,
                                      hook=sig.tap if a.name == "exact" else None, mix=sig.mixes or None)
            check_finite(logits, f"{p['name']} {a.name}")
            if store is not None:
                saved_fills[a.name] = store
            run = self._run_fields(a, P, n, pick, p)
            self._score(run, a, p, ids, n, keep, logits, cache, P, rec, ref_dec)
            if self.set == "decode" and a.name == "exact":
                ref_dec = run.pop("_ref")
            run["wall_s"] = round(time.time() - started, 3)
            if on_gpu:
                gib = 2 ** 30
                run["mem_gib"] = {"alloc_peak": round(torch.cuda.max_memory_allocated() / gib, 2),
                                  "reserved_peak": round(torch.cuda.max_memory_reserved() / gib, 2)}
            rec["runs"][a.name] = run
            del logits, cache
            sig.release_below(max((b.split for b in later), default=0))
        self._extra_references(p, rec)
        return self._summary(rec)

    def _extra_references(self, p, rec):
        """The tail-only key-token reference and the graded set's short-context reference, once per record."""
        m = self.m
        if self.key_tail is not None and rec.get("tail_only", {}).get("T") != self.key_tail:
            from .keytok import exact_tail_only
            n_scored = KEEP - 1 if self.set == "grade" else p["cont_len"]
            bos = self._bos_of(p["ids"])
            lps = exact_tail_only(m, list(p["ids"]), self.key_tail, bos, n_scored)
            rec["tail_only"] = {"T": self.key_tail, "bos": bos, "logprobs": [round(float(x), 6) for x in lps]}
        if self.set == "grade" and "short" not in rec and "short_ids" in p:
            short = torch.tensor(p["short_ids"])
            rows = torch.arange(short.shape[0] - KEEP, short.shape[0], device=m.device)
            logits, _ = m.forward_exact(short.to(m.device), keep=rows)
            rec["short"] = {"n": short.shape[0], "tail_match": p.get("short_tail_match"),
                            "logprobs": [round(float(x), 6) for x in score_tokens(logits, short, KEEP - 1)]}

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
