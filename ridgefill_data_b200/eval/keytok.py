"""Token-level NLL readouts over a scored window: novel tokens and LongPPL-style key tokens
(code/kva/keytok.py:26-78 semantics). Key tokens: the scored tokens whose exact-model log-prob drops by more
than THRESHOLD nats when the prefix is removed (context [BOS] + the last T prompt tokens)."""
from __future__ import annotations

import torch

from ..engine.scoring import score_tokens

THRESHOLD = 2.0


class KeyTokenReferenceMissing(ValueError):
    pass


def _bos_list(bos):
    """The BOS ids kept in front of a tail-only context: a list (possibly empty); None means none."""
    return [] if bos is None else list(bos)


def check_tail(n, scored, tail, bos):
    usable = n - len(_bos_list(bos))
    if not scored + 1 <= tail < usable:
        raise ValueError(f"key-token tail {tail}: needs scored + 1 ({scored + 1}) <= tail < {usable}")


@torch.no_grad()
def exact_tail_only(model, ids, tail, bos, scored):
    """Exact log-probs of the last `scored` tokens given only the prompt's own BOS ids (`bos`, a list, possibly
    empty) + the last `tail` prompt tokens."""
    ids = torch.as_tensor(ids, dtype=torch.long)
    b = _bos_list(bos)
    check_tail(ids.shape[0], scored, tail, b)
    ctx = ids[-tail:]
    if b:
        ctx = torch.cat((torch.tensor(b, dtype=torch.long), ctx))
    logits, _ = model.forward_exact(ctx.to(model.device),
                                    keep=torch.arange(ctx.shape[0] - scored - 1, ctx.shape[0], device=model.device))
    return score_tokens(logits, ctx, scored)


def key_mask(lp_full, lp_tail, threshold=THRESHOLD):
    return (lp_full.double() - lp_tail.double()) > threshold


def nll_delta(lp_arm, lp_exact, mask=None):
    d = (-lp_arm.double()) - (-lp_exact.double())
    if mask is not None:
        if int(mask.sum()) == 0:
            return None, 0
        d = d[mask]
    return float(d.mean()), int(d.numel())


def readout(rec, threshold=THRESHOLD):
    """{arm: {all | novel | key: {delta, n}}} for every non-exact arm of a grade or longppl evaluation record:
    the mean NLL change against exact over all scored tokens, the novel tokens and the key tokens (exact log-prob
    above the tail-only one by more than `threshold` nats). Reads {"runs": {arm: {"logprobs"}}, "tail_only":
    {"logprobs"}} records (also the flat {"lp": {arm: [...]}, "tail_only": [...]} form)."""
    if rec.get("tail_only") is None:
        raise KeyTokenReferenceMissing(f"{rec.get('name')}: no tail_only log-probs (run with keytoken_tail)")
    lp = rec["lp"] if "lp" in rec else {a: r["logprobs"] for a, r in rec["runs"].items() if "logprobs" in r}
    tail = rec["tail_only"]["logprobs"] if isinstance(rec["tail_only"], dict) else rec["tail_only"]
    f64 = dict(dtype=torch.float64)
    exact = torch.as_tensor(lp["exact"], **f64)
    masks = dict(all=None, novel=torch.as_tensor(rec["novel"], dtype=torch.bool) if "novel" in rec else None,
                 key=key_mask(exact, torch.as_tensor(tail, **f64), threshold))
    out = {}
    for arm, values in lp.items():
        if arm == "exact":
            continue
        v = torch.as_tensor(values, **f64)
        out[arm] = {}
        for k, m in masks.items():
            if k == "novel" and m is None:
                continue
            d, n = nll_delta(v, exact, m)
            out[arm][k] = dict(delta=d, n=n)
    return out
