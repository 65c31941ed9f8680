"""The `multiturn` evaluation set: several NIAH questions over one carried cache, with deferred repair (the
semantics of code/kva/multiturn.py:1-393).

The document is prefilled once by the arm and the cache is then kept, as a chat server keeps it:

* turn 1 is the mk4 NIAH prompt asking its target key, prefilled by the arm and answered greedily;
* each later turn asks one distractor key (the prompt's distractor order) as a new user turn, run exactly on top of
  the carried cache (engine.multiturn.extend), answered greedily and scored by eval.text.niah_correct.

An arm's own answers stay in its cache. The last answer token has not been fed when a turn ends, so the next turn
feeds it first unless it is an end-of-sequence id. A chat turn is then the template's turn closer, the question
(leading blank lines trimmed) and the assistant header; a raw turn is the question alone.

Repair arms (spec keys "repair": r in [0, 1] and "repair_by": "position" or "question") share turn 1 with the arm
they extend (the same spec without name / repair / repair_by) and then pay the skipped late-layer work back once:
* by position, right after turn 1: the first round(r P) rows of every late layer are recomputed from their stored
  exact layer-split inputs (r = 1 covers every cached row and makes the cache exact, GDN states included);
* by question, as turn 2 reaches the split: its rows' attention mass (the qattn signal over turn 2's last WINDOW
  rows) picks round(r P) prefix rows, which are recomputed through the late layers over the other rows as filled;
  GDN states stay as they are.

Record layout: rec["turns"] is the plan; rec["runs"][arm] = {P, split, tail, fill, st, f1, turn1_from,
turn1_wall_s, [select, n_rows, rows], [repair], turns: [{turn, key, value, correct, text, gen, finish_reason, ctx,
new, needle_start, needle_end, needle_projected, [needle_rows_exact], [needle_repaired], new_ids}], wall_s}.
"""
from __future__ import annotations

import json
import time

import torch

from ..engine import multiturn as EM
from ..engine import select as SEL
from ..engine.arm import Arm
from ..engine.decode import fork_cache
from ..engine.prefill import finish, run_lower
from . import text as TX
from .cost import CostModel

TURNS = 4
TURN_FILLS = ("proj", "identity", "none")
REPAIR_FILLS = ("proj", "identity")
HS_BYTES = 2                    # a repair keeps its layer-split inputs in bf16
_REPAIR_KEYS = ("name", "repair", "repair_by")


class MultiturnError(ValueError):
    pass


def _fills(spec):
    by_type = spec.get("fill_by_type")
    if by_type or spec.get("fill") == "by_type":
        return list((by_type or {}).values())
    return [spec.get("fill", "exact")]


def _turn1_problem(spec):
    """Why an arm's turn 1 is not a plain finish() the set can carry, or None."""
    if spec.get("fill", "exact") == "exact":
        return None
    kind = (spec.get("select") or {}).get("kind")
    if any(f not in TURN_FILLS for f in _fills(spec)):
        return "its fill"
    for key in ("tail_round", "reuse_fill", "tail_from"):
        if spec.get(key):
            return f"'{key}'"
    if kind in ("tail_match", "digits"):
        return f"the {kind} selector"
    return None


def _repair_problem(spec, r, by):
    if not isinstance(r, (int, float)) or not 0 <= r <= 1 or by not in ("position", "question"):
        return "repair takes a share in [0, 1] and repair_by 'position' or 'question'"
    if any(f not in REPAIR_FILLS for f in _fills(spec)):
        return "a repair recomputes from proj or identity fills only"
    if spec.get("tail_bias_from") is not None or spec.get("rescale") is not None:
        return "a repair arm takes no tail_bias_from or rescale"
    if by == "question" and ((spec.get("select") or {}).get("kind") or spec.get("f1")):
        return "a repair by question takes no select or f1"
    return None


def check_arms(specs, set_name):
    """Refuse repair keys outside the multiturn set, and arms whose turn 1 the set cannot carry."""
    for spec in specs:
        name = spec["name"]
        has_repair = "repair" in spec or "repair_by" in spec
        if set_name != "multiturn":
            if has_repair:
                raise MultiturnError(f"arm {name}: repair keys belong to the multiturn set")
            continue
        why = _turn1_problem(spec)
        if why:
            raise MultiturnError(f"arm {name}: {why} is not supported on the multiturn set")
        r = spec.get("repair")
        if r is None:
            if "repair_by" in spec:
                raise MultiturnError(f"arm {name}: repair_by given without a repair share")
            continue
        why = _repair_problem(spec, r, spec.get("repair_by", "position"))
        if why:
            raise MultiturnError(f"arm {name}: {why}")


def followup_pieces(tok, fmt):
    """(ids closing an assistant reply, ids opening the next reply after a user turn) of the chat template; both
    empty for raw prompts."""
    if fmt != "chat":
        return [], []
    answer, nxt = "<<rf-answer>>", "<<rf-next>>"
    convo = [dict(role="user", content="<<rf-first>>"), dict(role="assistant", content=answer),
             dict(role="user", content=nxt)]
    rendered = tok.apply_chat_template(convo, tokenize=False, add_generation_prompt=True)
    after_answer = rendered[rendered.index(answer) + len(answer):]
    closer, _, opener = after_answer.partition(nxt)
    return TX.encode(tok, closer), TX.encode(tok, opener)


def ask_ids(tok, fmt, key, pieces):
    """A later turn asking `key` in NIAH's question wording."""
    closer, opener = pieces
    question = TX.niah_question(fmt, key)
    if fmt == "chat":
        question = question.lstrip()
    return closer + TX.encode(tok, question) + opener


def ask_text_ids(tok, fmt, ask, pieces):
    """A later turn given as text (the two-key RULER rows: a question and the reply's prefix)."""
    closer, opener = pieces
    if fmt != "chat":
        return TX.encode(tok, f"\n{ask['question']}{ask['reply']}")
    return closer + TX.encode(tok, ask["question"]) + opener + TX.encode(tok, ask["reply"])


def needle_span(tok, ids, key, value):
    """[start, end) of a needle sentence inside the prompt ids (needles are encoded on their own and spliced in)."""
    sentence = TX.encode(tok, TX.niah_needle(key, value))
    width = len(sentence)
    for s in (i for i, t in enumerate(ids[:len(ids) - width + 1]) if t == sentence[0]):
        if ids[s:s + width] == sentence:
            return s, s + width
    raise MultiturnError(f"the prompt holds no needle for {key}")


def _spec(key, value, start, end):
    return dict(key=key, value=value, needle_start=start, needle_end=end)


def plan(tok, p, turns=TURNS):
    """The first `turns` turns of a prompt: its target key, then the distractors, each with its needle span."""
    if turns < 2 or turns > TURNS:
        raise MultiturnError(f"between 2 and {TURNS} turns, not {turns}")
    if "turn_plan" in p:
        have = p["turn_plan"]
        if turns > len(have):
            raise MultiturnError(f"{p['name']} plans {len(have)} turns, {turns} asked")
        return [dict(t) for t in have[:turns]]
    if p.get("variant") != "mk4":
        raise MultiturnError("multiturn prompts are mk4 NIAH prompts (their distractors give the later keys)")
    out = [_spec(p["key"], p["value"], p["needle_start"], p["needle_end"])]
    out += [_spec(d["key"], d["value"], *needle_span(tok, p["ids"], d["key"], d["value"])) for d in p["distractors"]]
    return out[:turns]


def _turn(tok, t, spec, gen, reason, ctx, new, P, rows=None):
    text = tok.decode(gen, skip_special_tokens=False)
    rec = dict(turn=t, key=spec["key"], value=spec["value"], correct=TX.niah_correct(text, spec["value"]),
               text=text, gen=gen, finish_reason=reason, ctx=ctx, new=new)
    rec.update(needle_start=spec["needle_start"], needle_end=spec["needle_end"],
               needle_projected=spec["needle_end"] <= P)
    if rows is not None:
        lo, hi = spec["needle_start"], spec["needle_end"]
        rec["needle_rows_exact"] = sum(1 for r in rows if lo <= r < hi)
    return rec


def repair_by_question(model, cache, arm, r, b, cost, info):
    """The extend() hook of turn 2 for a repair by question: turn 2's lower-layer rows rank the prefix rows by the
    attention they receive, the top round(r P) are recomputed (engine.multiturn.repair_selected), and `info`
    records what was done and what it cost."""
    P = b.shape[0]

    def hook(low):
        start = time.time()
        layers = SEL.qattn_layers(model, arm.split)
        end = EM.cached_rows(cache, 0)
        window = {i: low[i][-SEL.WINDOW:] for i in layers}
        mass = SEL.window_mass(model, window, cache, layers, end)
        picked = SEL.top_rows(mass, P, round(r * P))
        EM.repair_selected(model, cache, arm, b, picked)
        centre = (sum(picked) / len(picked) / P) if picked else 0.5
        w = window[layers[0]].shape[0] if layers else 0
        macs = cost.repair_selected(arm.split, len(picked), P, centre) + cost.qattn_select(end, arm.split, window=w)
        info.update(rows=len(picked), macs=macs, hs_bytes=model.hidden * P * HS_BYTES, picked=SEL.ranges(picked),
                    fixed=set(picked), wall_s=round(time.time() - start, 3))
    return hook


def later_turns(model, tok, cache, H, last, asks, turns, steps, eos, P, rows=None, split=None, before=None):
    """Turns 2, 3, ... on `cache` (H rows cached; `last` is the previous answer's unfed token). The cache grows."""
    done = []
    for number, ask, spec in zip(range(2, 2 + len(turns)), asks, turns):
        feed = ask if last in eos else [last] + ask
        hook = before if number == 2 else None
        logits, _ = EM.extend(model, cache, feed, H, split if hook is not None else None, hook)
        ctx = H
        H += len(feed)
        gen, reason, _ = EM.decode(model, cache, logits, H, steps, eos)
        H += len(gen) - 1
        done.append({**_turn(tok, number, spec, gen, reason, ctx, len(feed), P, rows), "new_ids": feed})
        last = gen[-1]
    return done


def base_key(arm):
    """Arms with the same key share turn 1 (a repair arm and the arm it extends)."""
    if arm.fill == "exact":
        return "exact"
    kept = {k: v for k, v in arm.meta.items() if k not in _REPAIR_KEYS}
    return json.dumps(kept, sort_keys=True, default=str)


class _Lower:
    """One prompt's exact lower layers, run once for every arm, with the window rows the qattn signals read."""

    def __init__(self, model, ids, arms):
        n = ids.shape[0]
        self.model = model
        selecting = [a for a in arms if a.meta.get("select")]
        ends = {n}
        ends.update(a.prefix_len(n) for a in selecting if a.meta["select"].get("window") == "prefix")
        self.windows = {e: {} for e in ends}
        self.masses = {}
        hook = self._keep if selecting else None
        self.hs, self.cache = run_lower(model, ids, sorted({a.split for a in arms}), hook=hook)

    def _keep(self, i, h):
        for end, rows in self.windows.items():
            rows[i] = h[max(0, end - SEL.WINDOW):end].clone()

    def mass(self, split, layers, end):
        used = tuple(SEL.qattn_layers(self.model, split, layers))
        if (used, end) not in self.masses:
            self.masses[used, end] = SEL.window_mass(self.model, self.windows[end], self.cache, used, end)
        return self.masses[used, end]


def _repaired(turn, fixed):
    """A later turn's needle lies wholly in the repaired rows."""
    return turn["turn"] > 1 and all(j in fixed for j in range(turn["needle_start"], turn["needle_end"]))


def _repair_position(model, cache, arm, r, P, H, hs_split, fed, cost):
    start = time.time()
    R = EM.repair_rows(r, P, H)
    inputs = hs_split if fed is None else torch.cat((hs_split.to(fed.device), fed))
    EM.repair(model, cache, inputs, arm.split, R)
    return dict(rows=R, macs=cost.repair(arm.split, R), hs_bytes=model.hidden * R * HS_BYTES, fixed=range(R),
                wall_s=round(time.time() - start, 3))


@torch.no_grad()
def run_prompt(model, tok, p, arms, rec, fmt, eos, steps, digit_set=None, n_turns=TURNS):
    """Run exact and every arm on one prompt, filling rec["turns"] and rec["runs"]; returns a one-line summary."""
    ids = torch.tensor(p["ids"])
    n = ids.shape[0]
    turns = rec["turns"] = plan(tok, p, n_turns)
    pieces = followup_pieces(tok, fmt)
    if "asks" in p:
        asks = [ask_text_ids(tok, fmt, a, pieces) for a in p["asks"][:len(turns) - 1]]
    else:
        asks = [ask_ids(tok, fmt, t["key"], pieces) for t in turns[1:]]
    deepest = max(a.split for a in arms if a.split is not None)
    every = [Arm("exact", split=deepest), *arms]
    groups = {}
    for a in every:
        groups.setdefault(base_key(a), []).append(a)
    low = _Lower(model, ids, every)
    picks = SEL.choose(every, n, p["ids"], p["name"], digit_set, low.mass)
    cost = CostModel(model.cfg)
    for members in groups.values():
        lead = members[0]
        start = time.time()
        pick = picks.get(lead.name)
        rows = pick["rows"] if pick else None
        logits, cache, P = finish(model, ids, low.hs[lead.split], low.cache, lead, 1, exact_rows=rows)
        keep_inputs = any(m.meta.get("repair") is not None for m in members)
        gen, reason, fed = EM.decode(model, cache, logits, n, steps, eos, lead.split if keep_inputs else None)
        H = n + len(gen) - 1
        first = _turn(tok, 1, turns[0], gen, reason, 0, n, P, rows)
        turn1_s = round(time.time() - start, 3)
        for m in members:
            start = time.time()
            run = dict(P=P, split=m.split, tail=n - P, fill=m.fill, st=bool(m.st), f1=m.f1, turn1_from=lead.name,
                       turn1_wall_s=turn1_s)
            if pick:
                run.update(select=pick["kind"], n_rows=len(rows), rows=SEL.ranges(rows))
            # the last member carries turn 1's cache itself: keeping it as a fork source would hold every K/V
            # buffer the later turns regrow
            own = cache if m is members[-1] else fork_cache(cache)
            if m is members[-1]:
                cache = None
            r, by = m.meta.get("repair"), m.meta.get("repair_by", "position")
            info, before = {}, None
            if r is not None and by == "position":
                info = _repair_position(model, own, m, r, P, H, low.hs[m.split], fed, cost)
            elif r is not None:
                before = repair_by_question(model, own, m, r, low.hs[m.split][:P], cost, info)
            later = later_turns(model, tok, own, H, gen[-1], asks, turns[1:], steps, eos, P, rows, m.split, before)
            run["turns"] = [first, *later]
            if r is not None:
                fixed = info.pop("fixed")
                depth = model.n_layers - m.split
                run["repair"] = dict(r=r, by=by, layers=depth, row_layers=info["rows"] * depth,
                                     macs_exact_prompt=cost.exact(n), **info)
                run["turns"] = [{**t, "needle_repaired": _repaired(t, fixed)} for t in run["turns"]]
            run["wall_s"] = round(time.time() - start, 3)
            rec["runs"][m.name] = run
    marks = {k: "".join("+" if t["correct"] else "-" for t in r["turns"]) for k, r in rec["runs"].items()}
    return " ".join(f"{k}:{v}" for k, v in marks.items())
