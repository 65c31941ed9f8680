"""Decode-side agreement with the exact model: the `decode` evaluation set (the measures of
code/kva/agree.py:1-85).

Every arm prefills the same prompt, then decodes exactly (SwiftKV-native arms through their own late layers) for a
fixed number of steps, end-of-sequence ignored, so that every prompt contributes the same number of positions:

* exact: the greedy tokens y_0 .. y_{s-1} and the log-probabilities at every step;
* arm, teacher-forced on y: per-step KL(exact || arm) over the vocabulary, and the share of steps whose argmax is
  y_t;
* arm, free-running: greedy from the arm's own cache, with the first position that leaves y and the share of
  positions equal to y.

The forced pass runs on a fork of the arm's cache (engine.decode.fork_cache), so both passes start from the same
filled state. Record fields: exact {gen, first_eos}; arm {gen, first_divergence, frac_identical,
forced_top1_agree, kl_mean, kl}.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from . import decode as D
from .scoring import check_finite


@torch.no_grad()
def run(model, n, cache, first_logits, steps, arm, feed=None, logprobs=False):
    """Decode `steps` positions after a prompt of n rows, starting from its last row's logits. Greedy by default;
    with `feed`, token feed[t] is the input after step t (teacher forcing). Returns (argmax of every step,
    fp32 host log-probabilities [steps, V] or None)."""
    if feed is not None and len(feed) < steps:
        raise ValueError(f"{steps} forced steps need {steps} tokens; {len(feed)} given")
    argmax, rows = [], []
    cur = first_logits[-1]
    for t in range(steps):
        check_finite(cur, f"{arm.name} decode step {t}")
        top = int(cur.argmax())
        argmax.append(top)
        if logprobs:
            rows.append(cur.float().log_softmax(-1).cpu())
        if t + 1 < steps:
            cur = D.step(model, top if feed is None else int(feed[t]), n + t, cache, arm)[-1]
    return argmax, (torch.stack(rows) if logprobs else None)


def kl_steps(lp_exact, lp_arm):
    """KL(exact || arm) of every step [steps] from fp32 log-probabilities [steps, V], in torch's KL reduction (the
    recorded arithmetic, so records compare across harnesses)."""
    return F.kl_div(lp_arm, lp_exact, reduction="none", log_target=True).sum(dim=-1)


def agreement(exact_tokens, arm_tokens):
    """(first position where the sequences differ, or None; share of equal positions)."""
    if not exact_tokens or len(arm_tokens) != len(exact_tokens):
        raise ValueError(f"cannot compare {len(arm_tokens)} arm tokens with {len(exact_tokens)} exact tokens")
    equal = [x == y for x, y in zip(exact_tokens, arm_tokens)]
    first = equal.index(False) if not all(equal) else None
    return first, sum(equal) / len(equal)


def exact_record(model, n, cache, first_logits, steps, arm, eos=()):
    """The exact run: (record fields, (tokens, log-probabilities))."""
    tokens, lp = run(model, n, cache, first_logits, steps, arm, logprobs=True)
    stops = set(eos)
    first_eos = next((t for t, tok in enumerate(tokens) if tok in stops), None)
    return {"gen": tokens, "first_eos": first_eos}, (tokens, lp)


def compare(model, n, cache, first_logits, steps, arm, y_exact, lp_exact):
    """An arm's forced and free passes against the exact run: its record fields."""
    forced, lp_arm = run(model, n, D.fork_cache(cache), first_logits, steps, arm, feed=y_exact, logprobs=True)
    kl = kl_steps(lp_exact, lp_arm)
    free, _ = run(model, n, cache, first_logits, steps, arm)
    first, share = agreement(y_exact, free)
    hits = sum(1 for a, b in zip(forced, y_exact) if a == b)
    return {"gen": free, "first_divergence": first, "frac_identical": round(share, 6),
            "forced_top1_agree": round(hits / steps, 6), "kl_mean": round(float(kl.mean()), 8),
            "kl": [round(float(v), 8) for v in kl]}
