"""Decode-side agreement with the exact model (the `decode` evaluation set; code/kva/agree.py:1-85 semantics).

Every arm prefills the same prompt; decoding is exact for every arm (SwiftKV-native arms through their own late
layers), for a fixed number of steps with EOS ignored, so each prompt contributes the same number of positions.
  exact         greedy tokens y_0..y_{s-1} and the log-probs at every step
  arm, forced   the arm's prefill cache fed the EXACT tokens: per-step KL(exact || arm) over the vocabulary and the
                share of steps whose arm argmax equals y_t
  arm, free     greedy from the arm's own cache: first divergence from y and the share of identical positions
The forced pass runs on a fork of the arm's cache (engine.decode.fork_cache: shared K/V buffers whose appended rows
land past the prompt, where the free pass then overwrites them; cloned recurrent states), so both passes start from
the same filled cache.
Record fields (the results' interface): exact {gen, first_eos}; arm {gen, first_divergence, frac_identical,
forced_top1_agree, kl_mean, kl}.
"""
from __future__ import annotations

import torch

from . import decode as D
from .scoring import check_finite


@torch.no_grad()
def run(model, n, cache, first_logits, steps, arm, feed=None, logprobs=False):
    """`steps` decode steps from the prompt's last-row logits (prompt of n rows). feed None: greedy; feed = tokens:
    teacher-forced (feed[t] enters after step t). Returns (argmax per step, log-probs [steps, V] fp32 on the host or
    None)."""
    if feed is not None and len(feed) < steps:
        raise ValueError(f"teacher forcing needs {steps} tokens, got {len(feed)}")
    tops, lps = [], []
    logits = first_logits[-1]
    for t in range(steps):
        check_finite(logits, f"{arm.name} decode step {t}")
        tops.append(int(logits.argmax()))
        if logprobs:
            lps.append(torch.log_softmax(logits.float(), -1).cpu())
        if t == steps - 1:
            break
        nxt = tops[t] if feed is None else int(feed[t])
        logits = D.step(model, nxt, n + t, cache, arm)[-1]
    return tops, (torch.stack(lps) if logprobs else None)


def kl_steps(lp_exact, lp_arm):
    """KL(exact || arm) per step [steps] from fp32 log-probs [steps, V]: sum_v p_exact (log p_exact - log p_arm)
    (the decode set's recorded arithmetic: fp32 log-softmax, torch's KL reduction, so records compare across
    harnesses)."""
    import torch.nn.functional as F
    return F.kl_div(lp_arm, lp_exact, reduction="none", log_target=True).sum(-1)


def agreement(exact_tokens, arm_tokens):
    """(first position whose tokens differ or None, share of equal positions)."""
    if len(exact_tokens) != len(arm_tokens) or not exact_tokens:
        raise ValueError(f"{len(exact_tokens)} exact vs {len(arm_tokens)} arm tokens")
    same = [a == b for a, b in zip(exact_tokens, arm_tokens)]
    first = next((t for t, s in enumerate(same) if not s), None)
    return first, sum(same) / len(same)


def exact_record(model, n, cache, first_logits, steps, arm, eos=()):
    """The exact run: (record fields, (tokens, log-probs))."""
    y, lp = run(model, n, cache, first_logits, steps, arm, logprobs=True)
    first_eos = next((t for t, x in enumerate(y) if x in set(eos)), None)
    return dict(gen=y, first_eos=first_eos), (y, lp)


def compare(model, n, cache, first_logits, steps, arm, y_exact, lp_exact):
    """The arm's forced and free passes against the exact run; returns the record fields."""
    fork = D.fork_cache(cache)
    forced, lp_arm = run(model, n, fork, first_logits, steps, arm, feed=y_exact, logprobs=True)
    del fork
    kl = kl_steps(lp_exact, lp_arm)
    free, _ = run(model, n, cache, first_logits, steps, arm)
    first, frac = agreement(y_exact, free)
    return dict(gen=free, first_divergence=first, frac_identical=round(frac, 6),
                forced_top1_agree=round(sum(a == b for a, b in zip(forced, y_exact)) / steps, 6),
                kl_mean=round(float(kl.mean()), 8), kl=[round(float(x), 8) for x in kl])
