"""Scoring: teacher-forced log-probs, next-token KL, top-1 agreement, finite checks (code/kva/kva.py:463-478);
decode agreement is engine/agree.py."""
from __future__ import annotations

import torch


class NonFiniteLogits(RuntimeError):
    """NaN/inf logits: a broken forward stops the run and never becomes a data point."""


def check_finite(logits, where):
    """logits, after checking that every value is finite."""
    if torch.isfinite(logits).all().item():
        return logits
    raise NonFiniteLogits(f"{where}: the logits hold NaN or inf")


def _device_scorer(*tensors):
    """The sm_100a vocabulary-reduction kernel applies when every tensor is on a CUDA device."""
    return all(t.is_cuda for t in tensors)


def score_tokens(logits, ids, keep_targets):
    """Log-probs (fp64) of the last keep_targets prompt tokens; logits = the last keep_targets + 1 rows."""
    tgt = ids[-keep_targets:].to(logits.device)
    if _device_scorer(logits):
        from ..ops.kernels import score_rows
        return score_rows(logits[:-1], targets=tgt)["logprob"].cpu()
    logp = logits[:-1].double().log_softmax(-1)
    return logp[torch.arange(tgt.shape[0], device=logp.device), tgt].cpu()


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
