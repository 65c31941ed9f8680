"""Scoring: teacher-forced log-probs, next-token KL, decode agreement, finite checks
(code/kva/kva.py:463-478, code/kva/agree.py:23-85)."""
from __future__ import annotations

import torch


class NonFiniteLogits(RuntimeError):
    """NaN/inf logits: a broken forward stops the run and never becomes a data point."""


def check_finite(logits, where):
    if not bool(torch.isfinite(logits).all()):
        raise NonFiniteLogits(f"non-finite logits ({where})")
    return logits


def _device_scorer(*tensors):
    """The sm_100a vocabulary-reduction kernel applies when every tensor is on a CUDA device."""
    return all(t.is_cuda for t in tensors)


def score_tokens(logits, ids, keep_targets):
    """Log-probs (fp64) of the last keep_targets prompt tokens; logits = the last keep_targets + 1 rows."""
    tgt = ids[-keep_targets:].to(logits.device)
    if _device_scorer(logits):
        from ..ops.kernels import score_rows
        return score_rows(logits[:-1], targets=tgt)["logprob"].cpu()
    lp = torch.log_softmax(logits[:-1].double(), -1)
    return lp.gather(1, tgt[:, None])[:, 0].cpu()


def mean_nll(logits, ids, keep_targets):
    return float(-score_tokens(logits, ids, keep_targets).double().mean())


def kl(p_logits, q_logits):
    """KL(p || q) per row, fp64 log-softmax (the device kernel on CUDA)."""
    if _device_scorer(p_logits, q_logits):
        from ..ops.kernels import score_rows
        return score_rows(q_logits, ref=p_logits)["kl"]
    lp = torch.log_softmax(p_logits.double(), -1)
    lq = torch.log_softmax(q_logits.double(), -1)
    return (lp.exp() * (lp - lq)).sum(-1)


def top1_agree(p_logits, q_logits):
    return (p_logits.argmax(-1) == q_logits.argmax(-1)).double()


@torch.no_grad()
def decode_agreement(model, ids, exact_cache, exact_first, arm_cache, arm_first, steps, eos=()):
    """Exact greedy tokens; the arm teacher-forced on them (per-step KL(exact || arm), top-1 agreement) and
    free-running (first divergence, identical share)."""
    from .decode import fork_cache
    n = ids.shape[0]
    ref_tokens, logits_ex, logits_arm = [], [exact_first[-1]], [arm_first[-1]]
    ce, ca = fork_cache(exact_cache), fork_cache(arm_cache)
    tok = int(exact_first[-1].argmax())
    for t in range(steps):
        ref_tokens.append(tok)
        if tok in eos or t == steps - 1:
            break
        pos = torch.tensor([n + t], device=model.device)
        he = model.embed(torch.tensor([tok], device=model.device))
        ha = he.clone()
        for i in range(model.n_layers):
            he = model.layer(i, he, pos, ce)
            ha = model.layer(i, ha, pos, ca)
        le, la = model.logits(he)[-1], model.logits(ha)[-1]
        logits_ex.append(le)
        logits_arm.append(la)
        tok = int(le.argmax())
    le, la = torch.stack(logits_ex), torch.stack(logits_arm)
    kls = kl(le, la)
    agree = top1_agree(le, la)
    # free pass
    cf = fork_cache(arm_cache)
    free = []
    tok = int(arm_first[-1].argmax())
    for t in range(len(ref_tokens)):
        free.append(tok)
        if t == len(ref_tokens) - 1:
            break
        pos = torch.tensor([n + t], device=model.device)
        h = model.embed(torch.tensor([tok], device=model.device))
        for i in range(model.n_layers):
            h = model.layer(i, h, pos, cf)
        tok = int(model.logits(h)[-1].argmax())
    diverge = next((t for t, (a, b) in enumerate(zip(ref_tokens, free)) if a != b), None)
    same = sum(a == b for a, b in zip(ref_tokens, free)) / max(1, len(ref_tokens))
    return dict(tokens=ref_tokens, kl=kls.tolist(), mean_kl=float(kls.mean()), top1=float(agree.mean()),
                first_divergence=diverge, identical_share=same)
