"""Multi-turn NIAH over a carried cache, with deferred repair (the `multiturn` evaluation set; semantics of
code/kva/multiturn.py:1-393).

A pasted document is prefilled once (approximately, by the arm) and its cache carried through several questions:
  turn 1      the mk4 NIAH prompt (the question about its target key), prefilled by the arm;
  turns 2..k  one per distractor key (in the prompt's distractor order), as a new user turn prefilled exactly on
              top of the carried cache, then greedy decode as NIAH, scored by eval.text.niah_correct.
Each arm keeps its own answer tokens in the cache (as a chat server does). An answer's last token has not been fed
yet; the next turn feeds it first unless it is an EOS (the chat template's turn closer follows either way).
  chat: next turn = [last token] + closer + question (leading blank lines trimmed) + assistant header
  raw:  next turn = [last token] + question
Repair arms ("repair": r, "repair_by": "position" | "question") share turn 1 with their base arm (the same spec
without name / repair / repair_by) and pay the skipped late-layer work back once:
  position  after turn 1, rows [0, round(r P)) of every late layer recomputed exactly from their stored exact
            layer-split inputs (every cached row at r = 1, which makes the cache exact: GDN states included)
  question  when turn 2 arrives: its rows run the exact lower layers, their attention mass (the qattn selector over
            turn 2's last WINDOW rows) picks round(r P) prefix rows, which are recomputed through the late layers
            over the other rows as filled (approximately exact); GDN states stay
Records: rec["turns"] (the plan) and per arm runs[arm] = {P, split, tail, fill, st, f1, turn1_from,
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
HS_BYTES = 2                    # bf16 layer-split inputs a repair keeps


class MultiturnError(ValueError):
    pass


def _fills(spec):
    if spec.get("fill") == "by_type" or spec.get("fill_by_type"):
        return list((spec.get("fill_by_type") or {}).values())
    return [spec.get("fill", "exact")]


def check_arms(specs, set_name):
    """Repair keys belong to the multiturn set; that set takes arms whose turn 1 is a plain finish()."""
    for s in specs:
        name, r, by = s["name"], s.get("repair"), s.get("repair_by", "position")
        if set_name != "multiturn":
            if "repair" in s or "repair_by" in s:
                raise MultiturnError(f"arm {name}: 'repair' runs on the multiturn set only")
            continue
        kind = (s.get("select") or {}).get("kind")
        if s.get("fill", "exact") != "exact" and (any(f not in TURN_FILLS for f in _fills(s)) or s.get("tail_round")
                                                  or kind in ("tail_match", "digits") or s.get("reuse_fill")
                                                  or s.get("tail_from")):
            raise MultiturnError(f"arm {name}: not supported on the multiturn set")
        if r is None:
            if "repair_by" in s:
                raise MultiturnError(f"arm {name}: repair_by without repair")
            continue
        if not (isinstance(r, (int, float)) and 0 <= r <= 1) or by not in ("position", "question"):
            raise MultiturnError(f"arm {name}: repair must be a fraction in [0, 1] by position or question")
        if (any(f not in REPAIR_FILLS for f in _fills(s)) or (by == "question" and (kind or s.get("f1")))
                or s.get("tail_bias_from") is not None or s.get("rescale") is not None):
            raise MultiturnError(f"arm {name}: repair needs fill proj or identity, no tail_bias_from or rescale "
                                 "(by question: no select, no f1)")


def followup_pieces(tok, fmt):
    """(closer after an assistant reply, header opening the next reply) of the chat template; raw: nothing."""
    if fmt != "chat":
        return [], []
    u1, a1, u2 = "\x00U1\x00", "\x00A1\x00", "\x00U2\x00"
    r = tok.apply_chat_template([{"role": "user", "content": u1}, {"role": "assistant", "content": a1},
                                 {"role": "user", "content": u2}], tokenize=False, add_generation_prompt=True)
    close, opener = r.split(a1)[1].split(u2)
    return TX.encode(tok, close), TX.encode(tok, opener)


def ask_ids(tok, fmt, key, pieces):
    close, opener = pieces
    q = TX.niah_question(fmt, key)
    return close + TX.encode(tok, q.lstrip() if fmt == "chat" else q) + opener


def ask_text_ids(tok, fmt, ask, pieces):
    """A later turn given as text (two-key RULER rows: question and reply prefix)."""
    close, opener = pieces
    if fmt == "chat":
        return close + TX.encode(tok, ask["question"]) + opener + TX.encode(tok, ask["reply"])
    return TX.encode(tok, "\n" + ask["question"] + ask["reply"])


def needle_span(tok, ids, key, value):
    """[start, end) of a needle sentence's ids inside the prompt (needles are spliced in as encoded alone)."""
    nd = TX.encode(tok, TX.niah_needle(key, value))
    m = len(nd)
    for s in range(len(ids) - m + 1):
        if ids[s] == nd[0] and ids[s:s + m] == nd:
            return s, s + m
    raise MultiturnError(f"the needle for {key} is not in the prompt")


def plan(tok, p, turns=TURNS):
    """The first `turns` turns of a prompt: the target key, then its distractors, each with its needle span."""
    if not 2 <= turns <= TURNS:
        raise MultiturnError(f"{turns} turns: 2..{TURNS}")
    if "turn_plan" in p:
        if turns > len(p["turn_plan"]):
            raise MultiturnError(f"{turns} turns, but {p['name']} has {len(p['turn_plan'])}")
        return [dict(t) for t in p["turn_plan"][:turns]]
    if p.get("variant") != "mk4":
        raise MultiturnError("the multiturn set reads mk4 prompts (the distractors are the later turns' keys)")
    out = [dict(key=p["key"], value=p["value"], needle_start=p["needle_start"], needle_end=p["needle_end"])]
    for d in p["distractors"]:
        s, e = needle_span(tok, p["ids"], d["key"], d["value"])
        out.append(dict(key=d["key"], value=d["value"], needle_start=s, needle_end=e))
    return out[:turns]


def _turn(tok, t, spec, gen, reason, ctx, new, P, rows=None):
    text = tok.decode(gen, skip_special_tokens=False)
    d = dict(turn=t, key=spec["key"], value=spec["value"], correct=TX.niah_correct(text, spec["value"]), text=text,
             gen=gen, finish_reason=reason, ctx=ctx, new=new, needle_start=spec["needle_start"],
             needle_end=spec["needle_end"], needle_projected=spec["needle_end"] <= P)
    if rows is not None:
        d["needle_rows_exact"] = sum(spec["needle_start"] <= r < spec["needle_end"] for r in rows)
    return d


def repair_by_question(model, cache, arm, r, b, cost, info):
    """extend()'s hook on turn 2: the turn's lower-layer inputs pick round(r P) prefix rows by attention mass; those
    are recomputed (engine.multiturn.repair_selected). Fills info."""
    P = b.shape[0]

    def hook(low):
        t0 = time.time()
        layers = SEL.qattn_layers(model, arm.split)
        end = EM.cached_rows(cache, 0)
        win = {i: low[i][-SEL.WINDOW:] for i in layers}
        picked = SEL.top_rows(SEL.window_mass(model, win, cache, layers, end), P, round(r * P))
        EM.repair_selected(model, cache, arm, b, picked)
        pos = sum(picked) / len(picked) / P if picked else 0.5
        window = win[layers[0]].shape[0] if layers else 0
        info.update(rows=len(picked), macs=cost.repair_selected(arm.split, len(picked), P, pos)
                    + cost.qattn_select(end, arm.split, window=window), hs_bytes=model.hidden * P * HS_BYTES,
                    picked=SEL.ranges(picked), fixed=set(picked), wall_s=round(time.time() - t0, 3))
    return hook


def later_turns(model, tok, cache, H, last, asks, turns, steps, eos, P, rows=None, split=None, before=None):
    """Turns 2.. on cache (H cached rows; `last` = the previous answer's unfed token). Appends to cache."""
    out = []
    for t, (ask, spec) in enumerate(zip(asks, turns), 2):
        new = ([] if last in eos else [last]) + ask
        hook = before if t == 2 else None
        lg, _ = EM.extend(model, cache, new, H, split if hook else None, hook)
        ctx, H = H, H + len(new)
        gen, reason, _ = EM.decode(model, cache, lg, H, steps, eos)
        H += len(gen) - 1
        out.append(dict(_turn(tok, t, spec, gen, reason, ctx, len(new), P, rows), new_ids=new))
        last = gen[-1]
    return out


def base_key(arm):
    if arm.fill == "exact":
        return "exact"
    return json.dumps({k: v for k, v in arm.meta.items() if k not in ("name", "repair", "repair_by")},
                      sort_keys=True, default=str)


@torch.no_grad()
def run_prompt(model, tok, p, arms, rec, fmt, eos, steps, digit_set=None, n_turns=TURNS):
    """Every arm (and exact) on one prompt; fills rec['turns'] and rec['runs']. Returns a one-line summary."""
    ids = torch.tensor(p["ids"])
    n = ids.shape[0]
    turns = rec["turns"] = plan(tok, p, n_turns)
    pieces = followup_pieces(tok, fmt)
    asks = ([ask_text_ids(tok, fmt, a, pieces) for a in p["asks"][:len(turns) - 1]] if "asks" in p
            else [ask_ids(tok, fmt, t["key"], pieces) for t in turns[1:]])
    todo = [Arm("exact", split=max(a.split for a in arms if a.split is not None))] + list(arms)
    groups = {}
    for a in todo:
        groups.setdefault(base_key(a), []).append(a)
    sel = [a for a in todo if a.meta.get("select")]
    ends = {n} | {a.prefix_len(n) for a in sel if a.meta["select"].get("window") == "prefix"}
    wins = {e: {} for e in ends}

    def hook(i, h):
        for e, w in wins.items():
            w[i] = h[max(0, e - SEL.WINDOW):e].clone()
    splits = sorted({a.split for a in todo})
    hs, lower = run_lower(model, ids, splits, hook=hook if sel else None)
    masses = {}

    def mass_of(split, layers, end):
        key = (tuple(SEL.qattn_layers(model, split, layers)), end)
        if key not in masses:
            masses[key] = SEL.window_mass(model, wins[end], lower, key[0], end)
        return masses[key]
    picks = SEL.choose(todo, n, p["ids"], p["name"], digit_set, mass_of)
    cost = CostModel(model.cfg)
    for members in groups.values():
        a = members[0]
        t0 = time.time()
        pick = picks.get(a.name)
        rows = pick["rows"] if pick else None
        logits, cache, P = finish(model, ids, hs[a.split], lower, a, 1, exact_rows=rows)
        need_hb = any(b.meta.get("repair") is not None for b in members)
        gen, reason, hb = EM.decode(model, cache, logits, n, steps, eos, a.split if need_hb else None)
        H = n + len(gen) - 1
        first = _turn(tok, 1, turns[0], gen, reason, 0, n, P, rows)
        t1 = round(time.time() - t0, 3)
        for b in members:
            t0 = time.time()
            run = dict(P=P, split=b.split, tail=n - P, fill=b.fill, st=bool(b.st), f1=b.f1, turn1_from=a.name,
                       turn1_wall_s=t1)
            if pick:
                run.update(select=pick["kind"], n_rows=len(rows), rows=SEL.ranges(rows))
            # the group's last arm takes turn 1's cache itself: a fork's source would keep every regrown K/V
            # buffer of the later turns alive
            if b is members[-1]:
                c, cache = cache, None
            else:
                c = fork_cache(cache)
            r, by, before, info = b.meta.get("repair"), b.meta.get("repair_by", "position"), None, {}
            if r is not None and by == "position":
                R = EM.repair_rows(r, P, H)
                hb_all = hs[b.split] if hb is None else torch.cat((hs[b.split].to(hb.device), hb))
                EM.repair(model, c, hb_all, b.split, R)
                info = dict(rows=R, macs=cost.repair(b.split, R), hs_bytes=model.hidden * R * HS_BYTES,
                            fixed=range(R), wall_s=round(time.time() - t0, 3))
            elif r is not None:
                before = repair_by_question(model, c, b, r, hs[b.split][:P], cost, info)
            run["turns"] = [first] + later_turns(model, tok, c, H, gen[-1], asks, turns[1:], steps, eos, P, rows,
                                                 b.split, before)
            if r is not None:
                fixed = info.pop("fixed")
                L = model.n_layers - b.split
                run["repair"] = dict(r=r, by=by, layers=L, row_layers=info["rows"] * L,
                                     macs_exact_prompt=cost.exact(n), **info)
                run["turns"] = [dict(t, needle_repaired=t["turn"] > 1 and all(
                    j in fixed for j in range(t["needle_start"], t["needle_end"]))) for t in run["turns"]]
            run["wall_s"] = round(time.time() - t0, 3)
            rec["runs"][b.name] = run
    return " ".join(f"{k}:" + "".join("+" if t["correct"] else "-" for t in r["turns"])
                    for k, r in rec["runs"].items())
