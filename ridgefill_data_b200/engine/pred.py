"""Predictability scores for the pred / blend selectors (code/kva/pred.py semantics).

A ridge from f(t) = [h_S(t-1) ; embed(ids[t])] to log1p of the exact model's surprisal of token t: a token the
model cannot predict from its context can only be copied later, so it should stay exact. The ridge runs on
standardised columns and is folded back to the raw features: s_hat(t) = f(t) . w + c. File: safetensors w [2H],
c [1] (fp32) with metadata split, hidden, features, target. Free baselines: unigram log-frequency tables
(add-one smoothed), logfreq [V] fp32.
"""
from __future__ import annotations

import torch

FEATURES = "[h_S(t-1) ; embed(ids[t])]"
TARGET = "log1p(exact surprisal of t)"


class Predictor:
    def __init__(self, split, w, c, meta=None):
        self.split, self.w, self.c = int(split), w.float(), float(c)
        self.meta = meta or {}

    @torch.no_grad()
    def score(self, h, e, block=8192):
        H = h.shape[1]
        w = self.w.to(h.device)
        out = torch.empty(h.shape[0], dtype=torch.float64)
        for r in range(0, h.shape[0], block):
            s = h[r:r + block].float() @ w[:H] + e[r:r + block].to(h.device).float() @ w[H:]
            out[r:r + block] = s.double().cpu()
        return out + self.c

    @classmethod
    def load(cls, path):
        from safetensors import safe_open
        with safe_open(str(path), "pt", device="cpu") as f:
            meta = f.metadata() or {}
            w, c = f.get_tensor("w"), f.get_tensor("c")
        return cls(int(meta["split"]), w, float(c[0]), meta)

    def save(self, path, meta):
        from safetensors.torch import save_file
        save_file({"w": self.w.float().contiguous(), "c": torch.tensor([self.c], dtype=torch.float32)}, str(path),
                  metadata={k: str(v) for k, v in dict(meta, split=self.split, hidden=self.w.numel() // 2,
                                                       features=FEATURES, target=TARGET).items()})


def log_freq(counts):
    c = counts.double() + 1
    return (c / c.sum()).log().float()


def save_freq(path, logfreq, meta):
    from safetensors.torch import save_file
    save_file({"logfreq": logfreq.float().contiguous()}, str(path), metadata={k: str(v) for k, v in meta.items()})


def load_freq(path):
    from safetensors import safe_open
    with safe_open(str(path), "pt", device="cpu") as f:
        return f.get_tensor("logfreq")


def prefix_scores(pred, h_split, emb, P):
    """Predicted surprisal [P] of prefix rows from h_split[j - 1] and emb[j]; row 0 ranks last (-inf)."""
    out = torch.full((P,), float("-inf"), dtype=torch.float64)
    if P > 1:
        out[1:] = pred.score(h_split[:P - 1], emb[1:P])
    return out


def standardise(state):
    n, sx = state["n"], state["sx"].double()
    sd = ((state["sxx"].diagonal().double() - sx * sx / n) / n).clamp_min(1e-12).sqrt()
    return dict(state, cx=state["cx"].double() / sd, sx=sx / sd, sxx=state["sxx"].double() / torch.outer(sd, sd),
                sxy={i: v.double() / sd[:, None] for i, v in state["sxy"].items()}), sd


def solve(state, alphas, layer=0):
    """{alpha: (w [d] fp64, c)}: ridge on standardised columns (penalty alpha * n), folded back to raw x."""
    from ..ridge.fit import EigenFit
    st, sd = standardise(state)
    return {a: (w[0].double() / sd, float(b[0])) for a, (w, b) in EigenFit(st).layer(layer, alphas).items()}


@torch.no_grad()
def fit_predictor(model, docs, split, alphas=(0.1, 1.0, 10.0)):
    """Fit the surprisal predictor on documents: features [h_S(t-1); embed(t)], target log1p surprisal."""
    from ..ridge.stats import RidgeStats
    st = RidgeStats(split, [0], 2 * model.hidden, "cpu", out_dim=1)
    for d in docs:
        ids = torch.as_tensor(d["ids"]).to(model.device)
        got = {}
        logits, _ = model.forward_exact(ids, hook=lambda i, h: got.__setitem__(i, h) if i == split else None,
                                        keep=torch.arange(ids.shape[0], device=model.device))
        lp = torch.log_softmax(logits[:-1].float(), -1)
        surprisal = -lp.gather(1, ids[1:, None])[:, 0]
        x = torch.cat((got[split][:-1].float(), model.embed(ids[1:]).float()), 1).cpu()
        st.add(x, {0: torch.log1p(surprisal).cpu()[:, None]})
    sols = solve(st.state(), alphas)
    a = alphas[len(alphas) // 2]
    return Predictor(split, sols[a][0].float(), sols[a][1])


def ranks(x):
    x = x.double()
    order = torch.argsort(x, stable=True)
    _, inv, counts = torch.unique_consecutive(x[order], return_inverse=True, return_counts=True)
    mean_rank = counts.cumsum(0).double() - (counts.double() - 1) / 2
    r = torch.empty_like(x)
    r[order] = mean_rank[inv]
    return r


def spearman(a, b):
    ra, rb = ranks(a), ranks(b)
    ra, rb = ra - ra.mean(), rb - rb.mean()
    return float((ra * rb).sum() / (ra.norm() * rb.norm()).clamp_min(1e-300))


def topk_recall(pred, true, frac):
    k = max(1, round(frac * true.numel()))
    return len(set(pred.topk(k).indices.tolist()) & set(true.topk(k).indices.tolist())) / k
