"""Ridge fits from sufficient statistics.

Centred form (the reference's, code/kva/ridge.py:77-131): C = S - s s^T / n,
    W(lam) = (Cxx + lam * mean(diag Cxx) * I)^-1 Cxy,    bias b = mean_y - mean_x W  (unpenalised).
mean(diag Cxx) is trace(Cxx) / d of the centred scatter.
Plain form (the benchmark plan's tiny configuration): no centring, no bias,
    W(lam) = (X^T X + lam * trace(X^T X) / d * I)^-1 X^T Y.

Two solvers:
  EigenFit     one fp64 eigendecomposition of Cxx shared by every layer and lambda (CPU; the oracle);
               also reduced-rank ridge and per-output sums of squares.
  CholeskyFit  one Cholesky factorisation of (Cxx + lam s I) per lambda, then triangular solves for every
               late layer's Cxy at once; runs on the device (sm_100a fp64 kernels when the tensors are on
               CUDA, torch.linalg on the CPU).
Both return {lam: (weight [d_out, d_in] fp32, bias [d_out] fp32)} in F.linear layout.
"""
from __future__ import annotations

import torch

from .stats import raw_moments


def centred(state):
    """(n, mean_x, Cxx, scale = mean(diag Cxx)) fp64 from a state dict."""
    n = state["n"]
    sx = state["sx"].double()
    mean_x = state["cx"].double() + sx / n
    cxx = state["sxx"].double() - torch.outer(sx, sx) / n
    return n, mean_x, cxx, cxx.diagonal().mean().item()


def centred_cross(state, i):
    """(Cxy, mean_y) fp64 of layer i."""
    n = state["n"]
    sx, sy = state["sx"].double(), state["sy"][i].double()
    cxy = state["sxy"][i].double() - torch.outer(sx, sy) / n
    return cxy, state["cy"][i].double() + sy / n


class EigenFit:
    """Eigendecomposition of the centred input scatter, shared by every layer and lambda."""

    def __init__(self, state, center=True):
        self.state = state
        self.center = center
        if center:
            self.n, self.mean_x, cxx, self.scale = centred(state)
        else:
            self.n = state["n"]
            self.mean_x = None
            cxx, _ = raw_moments(state, state["layers"][0])
            self.scale = (cxx.diagonal().sum() / cxx.shape[0]).item()
        self.evals, self.evecs = torch.linalg.eigh(cxx)

    def _cross(self, i):
        if self.center:
            cxy, mean_y = centred_cross(self.state, i)
        else:
            _, cxy = raw_moments(self.state, i)
            mean_y = None
        return self.evecs.T @ cxy, mean_y

    def layer(self, i, lams):
        a, mean_y = self._cross(i)
        out = {}
        for lam in lams:
            w = self.evecs @ (a / (self.evals + lam * self.scale)[:, None])         # [d_in, d_out]
            bias = mean_y - self.mean_x @ w if self.center else torch.zeros(w.shape[1], dtype=w.dtype)
            out[lam] = (w.T.float().contiguous(), bias.float())
        return out

    def sq(self, i, weight):
        """Per output over the training rows: (sum of squares of the fitted values, sum of squares of the
        targets) fp64; needs state['sq'][i] = per-output sum of (y - cy)^2 (code/kva/ridge.py:107-115)."""
        st = self.state
        cy, sy = st["cy"][i].double(), st["sy"][i].double()
        z = self.evecs.T @ weight.double().T
        fitted = (z * z * self.evals[:, None]).sum(0) + self.n * (cy + sy / self.n) ** 2
        return fitted, st["sq"][i] + 2 * cy * sy + self.n * cy * cy

    def reduced_rank(self, i, lam, ranks):
        """Reduced-rank ridge: the rank-r minimiser of |Y - XW|^2 + lam s |W|^2 is W(lam) V_r V_r^T, V_r the top
        r eigenvectors of a^T diag(1 / (e + lam s)) a (code/kva/ridge.py:117-131). Returns ({r: (weight,
        bias)}, cumulative share of the fitted energy kept by the top k directions)."""
        a, mean_y = self._cross(i)
        dd = self.evals + lam * self.scale
        w = self.evecs @ (a / dd[:, None])
        ev, v = torch.linalg.eigh(a.T @ (a / dd[:, None]))
        ev, v = ev.flip(0).clamp(min=0), v.flip(1)
        out = {}
        for r in ranks:
            wr = (w @ v[:, :r]) @ v[:, :r].T
            bias = mean_y - self.mean_x @ wr if self.center else torch.zeros(wr.shape[1], dtype=wr.dtype)
            out[r] = (wr.T.float().contiguous(), bias.float())
        return out, ev.cumsum(0) / ev.sum().clamp(min=1e-300)


class CholeskyFit:
    """Per-lambda Cholesky solves of the ridge normal equations for every late layer at once."""

    def __init__(self, state, center=True, device=None):
        self.state = state
        self.center = center
        self.device = torch.device(device) if device is not None else state["sxx"].device
        if center:
            self.n, self.mean_x, cxx, self.scale = centred(state)
        else:
            self.n = state["n"]
            self.mean_x = None
            cxx, _ = raw_moments(state, state["layers"][0])
            self.scale = (cxx.diagonal().sum() / cxx.shape[0]).item()
        self.cxx = cxx.to(self.device)

    def _rhs(self, layers):
        key = tuple(layers)
        if getattr(self, "_rhs_key", None) == key:          # built once per layer set (one solve per lambda)
            return self._rhs_val
        cols, means = [], []
        for i in layers:
            if self.center:
                cxy, mean_y = centred_cross(self.state, i)
            else:
                _, cxy = raw_moments(self.state, i)
                mean_y = None
            cols.append(cxy.to(self.device))
            means.append(mean_y)
        self._rhs_key, self._rhs_val = key, (torch.cat(cols, 1), means)
        return self._rhs_val

    def layers(self, layers, lams):
        """{lam: {i: (weight, bias)}} for every layer in `layers`."""
        from . import solve
        rhs, means = self._rhs(layers)
        d = self.cxx.shape[0]
        mean_x = self.mean_x.to(self.device) if self.center else None
        out = {}
        for lam in lams:
            w_all = solve.ridge_solve(self.cxx, rhs, lam * self.scale)           # [d_in, L * d_out]
            res = {}
            for j, i in enumerate(layers):
                w = w_all[:, j * (rhs.shape[1] // len(layers)):(j + 1) * (rhs.shape[1] // len(layers))]
                if self.center:
                    bias = means[j].to(self.device) - mean_x @ w
                else:
                    bias = torch.zeros(w.shape[1], dtype=w.dtype, device=w.device)
                res[i] = (w.T.float().contiguous(), bias.float())
            out[lam] = res
            del w_all
        assert d == rhs.shape[0]
        return out

    def layer(self, i, lams):
        return {lam: v[i] for lam, v in self.layers([i], lams).items()}


# The reference's name for the eigen solver.
RidgeFit = EigenFit
