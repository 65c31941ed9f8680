"""Surprisal predictor and unigram-frequency tables behind the pred / freq / frag selectors
(code/kva/pred.py semantics).

A token that the model could not have guessed from what came before (a number, a name, an identifier) can only be
copied later, so it is worth keeping exact. The predictor estimates that surprisal before any question is seen:

    s_hat(t) = h_S(t-1) . w_h + embed(ids[t]) . w_e + c       (w = [w_h ; w_e], length 2H)

fitted by ridge to log1p(-log p(ids[t] | ids[<t])) of the exact model, on standardised feature columns (the
residual stream has a few very large dimensions) and stored with the scaling folded back into w.

On-disk layout, kept alike with the reference so its files load: a safetensors file with tensors "w" [2H] and
"c" [1] (fp32) and string metadata split / hidden / features / target plus provenance; a frequency table is a
safetensors file with "logfreq" [V] fp32 = log((count + 1) / (total + V)).
"""
from __future__ import annotations

import numpy as np
import torch

FEATURES = "[h_S(t-1) ; embed(ids[t])]"
TARGET = "log1p(exact surprisal of t)"


def _str_meta(d):
    return {str(k): str(v) for k, v in d.items()}


class Predictor:
    """Linear surprisal predictor of one split layer."""

    def __init__(self, split, w, c, meta=None):
        self.split = int(split)
        self.w = w.detach().float().reshape(-1)
        self.c = float(c)
        self.meta = dict(meta or {})

    @property
    def hidden(self):
        return self.w.numel() // 2

    @torch.no_grad()
    def score(self, h, e, block=8192):
        """s_hat [m] (fp64, host) for rows whose split-layer input of the previous token is h [m, H] and whose
        embedding is e [m, H]; evaluated in blocks of `block` rows on h's device."""
        dev = h.device
        w_h, w_e = self.w[:self.hidden].to(dev), self.w[self.hidden:].to(dev)
        parts = [torch.mv(h[a:a + block].float(), w_h).add_(torch.mv(e[a:a + block].to(dev).float(), w_e))
                 for a in range(0, h.shape[0], block)]
        flat = torch.cat(parts) if parts else torch.zeros(0, device=dev)
        return flat.double().cpu() + self.c

    @classmethod
    def load(cls, path):
        from safetensors import safe_open
        with safe_open(str(path), "pt", device="cpu") as f:
            meta = dict(f.metadata() or {})
            w, c = f.get_tensor("w"), f.get_tensor("c")
        return cls(meta["split"], w, c.reshape(-1)[0].item(), meta)

    def save(self, path, meta):
        from safetensors.torch import save_file
        info = dict(meta)
        info.update(split=self.split, hidden=self.hidden, features=FEATURES, target=TARGET)
        tensors = {"w": self.w.contiguous(), "c": torch.full((1,), self.c, dtype=torch.float32)}
        save_file(tensors, str(path), metadata=_str_meta(info))


def log_freq(counts):
    """Add-one smoothed log unigram frequency [V] (fp32) of a token-count vector."""
    smoothed = counts.to(torch.float64) + 1.0
    return (smoothed.log() - smoothed.sum().log()).float()


def save_freq(path, logfreq, meta):
    from safetensors.torch import save_file
    save_file({"logfreq": logfreq.float().contiguous()}, str(path), metadata=_str_meta(meta))


def load_freq(path):
    from safetensors.torch import load_file
    return load_file(str(path))["logfreq"]


def prefix_scores(pred, h_split, emb, P):
    """Predicted surprisal [P] of prefix rows 1..P-1 (read from h_split rows 0..P-2 and emb rows 1..P-1, so it
    depends on the prefix alone); row 0, with nothing to be predicted from, gets -inf and ranks last."""
    scores = [torch.full((1,), float("-inf"), dtype=torch.float64)] if P > 0 else []
    if P > 1:
        scores.append(pred.score(h_split[:P - 1], emb[1:P]))
    return torch.cat(scores) if scores else torch.zeros(0, dtype=torch.float64)


def standardise(state):
    """Sufficient statistics (a RidgeStats.state()) of the columns rescaled to unit standard deviation, and the
    per-column standard deviations used."""
    n = state["n"]
    mean = state["sx"].double() / n
    var = state["sxx"].diagonal().double() / n - mean * mean
    sd = var.clamp_min(1e-12).sqrt()
    inv = 1.0 / sd
    scaled = dict(state)
    scaled["cx"] = state["cx"].double() * inv
    scaled["sx"] = state["sx"].double() * inv
    scaled["sxx"] = state["sxx"].double() * inv[:, None] * inv[None, :]
    scaled["sxy"] = {k: v.double() * inv[:, None] for k, v in state["sxy"].items()}
    return scaled, sd


def solve(state, alphas, layer=0):
    """{alpha: (w [d] fp64, intercept)} of the ridge on standardised columns with penalty alpha * n, mapped back to
    the raw features."""
    from ..ridge.fit import EigenFit
    scaled, sd = standardise(state)
    fits = EigenFit(scaled).layer(layer, alphas)
    return {a: (wb[0][0].double() / sd, float(wb[1][0])) for a, wb in fits.items()}


@torch.no_grad()
def fit_predictor(model, docs, split, alphas=(0.1, 1.0, 10.0)):
    """Fit the predictor on calibration documents ({"ids": [...]}) and return the middle alpha's solution."""
    from ..ridge.stats import RidgeStats
    acc = RidgeStats(split, [0], 2 * model.hidden, "cpu", out_dim=1)
    for doc in docs:
        ids = torch.as_tensor(doc["ids"]).to(model.device)
        seen = {}

        def grab(i, h):
            if i == split:
                seen["h"] = h

        logits, _ = model.forward_exact(ids, hook=grab, keep=torch.arange(ids.shape[0], device=model.device))
        nll = torch.nn.functional.cross_entropy(logits[:-1].float(), ids[1:], reduction="none")
        feats = torch.cat((seen["h"][:-1].float(), model.embed(ids[1:]).float()), 1).cpu()
        acc.add(feats, {0: nll.log1p().cpu()[:, None]})
    chosen = alphas[len(alphas) // 2]
    w, c = solve(acc.state(), alphas)[chosen]
    return Predictor(split, w.float(), c)


def ranks(x):
    """1-based ranks of x (fp64), tied values sharing the mean of their ranks."""
    from scipy.stats import rankdata
    return torch.from_numpy(rankdata(x.double().cpu().numpy(), method="average")).to(torch.float64)


def spearman(a, b):
    """Spearman rank correlation (0 when either side is constant)."""
    ra, rb = ranks(a).numpy(), ranks(b).numpy()
    ra, rb = ra - ra.mean(), rb - rb.mean()
    den = float(np.sqrt((ra * ra).sum() * (rb * rb).sum()))
    return float((ra * rb).sum()) / den if den > 0 else 0.0


def topk_recall(pred, true, frac):
    """Share of the k = round(frac * n) (at least 1) highest true rows that are among the k highest predicted."""
    k = max(1, round(frac * true.numel()))
    hit = set(torch.topk(pred, k).indices.tolist())
    return sum(int(i in hit) for i in torch.topk(true, k).indices.tolist()) / k
