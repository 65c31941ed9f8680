"""Quality mode: a RidgeFill arm whose prefix keeps some rows exact, chosen per prompt from what the prompt itself says
matters (the serving mode behind the published 27B headline, whose flags are listed in
code/qwen38-27b-kit/common.py:20-27; the bypass semantics are code/kva/kva.py:392-459).

Rows picked, in priority order, up to `share` of the prefix:
  rules    every prefix row whose token is a digit token or a special token (the caller's id sets; the tokenizer's
           when the server has one)
  lexical  spans of the prefix, before the last `lexical_window` prompt tokens, that repeat a run of `lexical_min`
           or more of those tokens (the question quoting its context): each match marks the matched tokens plus up
           to `lexical_span_rows` rows from the match start; only the `lexical_max_occurrences` latest matches of a run
  qattn    the round(qattn_share * N) rows with the highest attention mass from the last `qattn_window` prompt rows
           in the exact lower attention layers (engine/select.py window_mass, the tensor-core kernel on a GPU)
Prompts shorter than `min_prompt` run exact. The tail is the arm's own. The reference release gives this mode's flags
but not its engine source, so the rules above are this framework's reading of them; every number is a field here.
"""
from __future__ import annotations

from dataclasses import dataclass, field

import torch

from . import select as S
from .prefill import finish, run_lower


@dataclass
class QualityMode:
    min_prompt: int = 8192
    share: float = 0.5
    qattn_share: float = 0.2
    qattn_window: int = 64
    digits: bool = True
    specials: bool = True
    lexical: bool = True
    lexical_window: int = 64
    lexical_min: int = 4
    lexical_span_rows: int = 80
    lexical_max_occurrences: int = 2
    digit_ids: frozenset = field(default_factory=frozenset)
    special_ids: frozenset = field(default_factory=frozenset)

    def to_meta(self):
        return {k: (sorted(v) if isinstance(v, frozenset) else v) for k, v in self.__dict__.items()}


def rule_rows(ids, P, mode):
    """Prefix rows whose token is a digit or special token."""
    want = set()
    if mode.digits:
        want |= set(mode.digit_ids)
    if mode.specials:
        want |= set(mode.special_ids)
    if not want or P <= 0:
        return []
    head = ids[:P].tolist()
    return [r for r, t in enumerate(head) if t in want]


def lexical_rows(ids, P, mode):
    """Rows of prefix spans that repeat a run of >= lexical_min tokens of the prompt's last lexical_window tokens."""
    n, m = ids.numel(), mode.lexical_min
    if not mode.lexical or P < m or n < m:
        return []
    ids = ids.to("cpu", torch.long)
    w0 = max(0, n - mode.lexical_window)
    window = ids[w0:]
    stop = min(P, w0)                                 # matches lie before the window (not the window itself)
    if window.numel() < m or stop < m:
        return []
    # every m-gram starting in the prefix, hashed (int64 polynomial, wrapping); hash hits are checked exactly
    powers = torch.tensor([1000003 ** k for k in range(m)], dtype=torch.long)
    keys = (ids[:stop].unfold(0, m, 1) * powers).sum(1)
    wkeys = (window.unfold(0, m, 1) * powers).sum(1)
    cand = torch.nonzero(torch.isin(keys, wkeys)).flatten().tolist()
    grams = {tuple(g) for g in window.unfold(0, m, 1).tolist()}
    seq = ids.tolist()
    hits = {}
    for s in cand:                                    # starts of prefix m-grams that occur in the window
        g = tuple(seq[s:s + m])
        if g in grams:
            hits.setdefault(g, []).append(s)
    rows = set()
    for starts in hits.values():
        for s in starts[-mode.lexical_max_occurrences:]:
            rows.update(range(s, min(stop, s + max(m, mode.lexical_span_rows))))
    return sorted(rows)


def pick_rows(ids, P, mode, mass=None):
    """The exact prefix rows of one prompt (ascending), at most round(share * P)."""
    cap = min(P, round(mode.share * P))
    chosen, seen = [], set()

    def add(rows):
        for r in rows:
            if len(chosen) >= cap:
                return
            if r not in seen:
                seen.add(r)
                chosen.append(r)

    add(rule_rows(ids, P, mode))
    add(lexical_rows(ids, P, mode))
    if mass is not None and mode.qattn_share > 0:
        add(S.top_rows(mass, P, round(mode.qattn_share * ids.numel())))
    return sorted(chosen)


def prefill_quality(model, ids, arm, mode, keep=1, keep_cache=True, reserve=64, tick=None):
    """(logits of the last `keep` rows, cache, P, exact rows) of one prompt under the quality mode: exact below
    min_prompt, else RidgeFill with the picked prefix rows recomputed exactly through every late layer."""
    ids = ids.to(model.device)
    n = ids.numel()
    if n < mode.min_prompt or arm.split is None:
        hs, cache = run_lower(model, ids, [model.n_layers], reserve=reserve, tick=tick)
        return model.logits(hs[model.n_layers][-keep:]), cache, 0, []
    layers = S.qattn_layers(model, arm.split) if mode.qattn_share > 0 else []
    w = min(mode.qattn_window, n)
    win = {}

    def grab(i, h):
        if i in layers:
            win[i] = h[n - w:n].clone()
    hs, lower = run_lower(model, ids, [arm.split], hook=grab if layers else None, reserve=reserve, tick=tick,
                          maps=arm.projector)
    P = arm.prefix_len(n)
    mass = S.window_mass(model, win, lower, layers, end=n) if layers else None
    rows = pick_rows(ids.cpu(), P, mode, mass)
    logits, cache, P = finish(model, ids, hs[arm.split], lower, arm, keep, keep_cache=keep_cache,
                              exact_rows=rows or None, tick=tick)
    return logits, cache, P, rows


def special_ids_of(tokenizer):
    """The tokenizer's special and added-token ids."""
    if tokenizer is None:
        return frozenset()
    ids = set(getattr(tokenizer, "all_special_ids", []) or [])
    ids |= set(getattr(tokenizer, "added_tokens_decoder", {}) or {})
    return frozenset(int(i) for i in ids)


def digit_ids_of(tokenizer):
    if tokenizer is None or not hasattr(tokenizer, "convert_ids_to_tokens"):
        return frozenset()
    return frozenset(S.digit_ids(tokenizer))


