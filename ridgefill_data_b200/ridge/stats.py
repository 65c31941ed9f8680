"""Shifted sufficient statistics of the ridge regressions x -> y_i (code/kva/ridge.py:19-75).

For boundary rows x [n, d] and each late layer's true inputs y_i [n, d]:
  n, sx = sum(x - cx), sxx = sum((x - cx)(x - cx)^T), sy_i = sum(y_i - cy_i), sxy_i = sum((x - cx)(y_i - cy_i)^T)
with fixed shifts cx, cy_i (the first block's means) for numerical stability. Products are summed in
fp32 within row blocks and the blocks added into fp64 accumulators.

On a CUDA device the products run on the tcgen05 Gram kernel: the centred rows are split as
hi + lo (two bf16 terms, ~16 mantissa bits) and X^T Y is accumulated as hi^T hi + hi^T lo + lo^T hi
in one MN-major GEMM over the concatenated rows, fp32 per k-chunk and fp64 across chunks
(ops.gemm.gram_acc). On the CPU the products are plain fp32 matmuls.

Row weights: add(..., w) makes every sum weighted (n holds sum(w)); w=None is unweighted.
"""
from __future__ import annotations

import torch

BLOCK = 8192


def split_bf16(xc):
    """fp32 rows -> (hi, lo) bf16 with hi + lo ~= xc to ~2^-16 relative."""
    hi = xc.to(torch.bfloat16)
    lo = (xc - hi.float()).to(torch.bfloat16)
    return hi, lo


def cross_acc(acc, a, b, block=BLOCK):
    """acc [da, db] fp64 += a^T b for fp32 rows a [n, da], b [n, db]."""
    if a.is_cuda:
        from ..ops import gemm
        ah, al = split_bf16(a)
        if b is a:
            bh, bl = ah, al
        else:
            bh, bl = split_bf16(b)
        lhs = torch.cat((ah, ah, al), 0)
        rhs = torch.cat((bh, bl, bh), 0)
        if acc.is_cuda and acc.is_contiguous():
            gemm.gram_acc(acc, lhs, rhs, k_chunk=block)
        else:
            tmp = torch.zeros(acc.shape, dtype=torch.float64, device=a.device)
            gemm.gram_acc(tmp, lhs, rhs, k_chunk=block)
            acc += tmp.to(acc.device)
        return acc
    acc += (a.T @ b).to(acc.device, torch.float64)
    return acc


class RidgeStats:
    """Accumulators for one split over its late layers (fp64, on `device`)."""

    def __init__(self, split, layers, dim, device="cpu", out_dim=None):
        self.split = split
        self.layers = list(layers)
        self.dim = dim
        self.device = torch.device(device)
        width = dim if out_dim is None else out_dim

        def zeros(*shape):
            return torch.zeros(*shape, dtype=torch.float64, device=self.device)

        self.n = 0.0
        self.cx, self.cy = None, {}
        self.sx, self.sxx = zeros(dim), zeros(dim, dim)
        self.sy = {i: zeros(width) for i in self.layers}
        self.sxy = {i: zeros(dim, width) for i in self.layers}
        self._x = self._w = None
        self._block = BLOCK

    def _weighted(self, centred, start):
        """Centred rows times their row weights (unchanged when unweighted)."""
        if self._w is None:
            return centred
        return centred * self._w[start:start + centred.shape[0]]

    def _centred_x(self, start, device):
        return self._x[start:start + self._block].float() - self.cx.to(device)

    @torch.no_grad()
    def begin(self, x, block=BLOCK, w=None):
        """Split-layer rows x [n, d] of one document; add_layer then takes each late layer's rows."""
        if self.cx is None:
            self.cx = x[:block].float().mean(0)          # the shift: the first block's mean
        self._x, self._block = x, block
        self._w = None if w is None else w.to(x.device, torch.float32).unsqueeze(1)
        self.n += float(w.double().sum()) if w is not None else x.shape[0]
        for start in range(0, x.shape[0], block):
            xc = self._centred_x(start, x.device)
            xw = self._weighted(xc, start)
            self.sx += xw.sum(0).double().to(self.device)
            cross_acc(self.sxx, xw, xc, block)

    @torch.no_grad()
    def add_layer(self, i, y):
        """Layer i's true input rows y [n, d_out] for the rows given to begin()."""
        block = self._block
        if i not in self.cy:
            self.cy[i] = y[:block].float().mean(0)
        for start in range(0, y.shape[0], block):
            xw = self._weighted(self._centred_x(start, y.device), start)
            yc = y[start:start + block].float() - self.cy[i].to(y.device)
            self.sy[i] += self._weighted(yc, start).sum(0).double().to(self.device)
            cross_acc(self.sxy[i], xw, yc, block)

    def add(self, x, ys, block=BLOCK, w=None):
        self.begin(x, block, w)
        for i in self.layers:
            self.add_layer(i, ys[i])

    def state(self):
        """The accumulators as a host dict (shifts in fp64): split, layers, dim, n, cx, cy, sx, sxx, sy, sxy."""
        def host(t):
            return t.detach().cpu()

        out = {"split": self.split, "layers": self.layers, "dim": self.dim, "n": self.n,
               "cx": host(self.cx).double(), "sx": host(self.sx), "sxx": host(self.sxx)}
        out["cy"] = {i: host(v).double() for i, v in self.cy.items()}
        out["sy"] = {i: host(self.sy[i]) for i in self.sy}
        out["sxy"] = {i: host(self.sxy[i]) for i in self.sxy}
        return out


def residual(state):
    """Statistics of the target y - x (a ridge towards the identity map): shifts cy - cx, sums sy - sx and
    sxy - sxx (code/kva/ridge.py:134-139)."""
    sx = state["sx"].double()
    sxx = state["sxx"].double()
    res = dict(state, sx=sx, sxx=sxx)
    res["cy"] = {i: state["cy"][i] - state["cx"] for i in state["layers"]}
    res["sy"] = {i: state["sy"][i].double() - sx for i in state["layers"]}
    res["sxy"] = {i: state["sxy"][i].double() - sxx for i in state["layers"]}
    return res


def _moved(s, s2, n, d_row, d_col, s_col=None):
    """A cross sum about shifted centres: the sum of (x + d_row)(y + d_col)^T given s2 = sum x y^T, s = sum x,
    s_col = sum y (defaults to s) and the row count n."""
    s_col = s if s_col is None else s_col
    return s2 + torch.outer(s, d_col) + torch.outer(d_row, s_col) + n * torch.outer(d_row, d_col)


def combine(a, b, w=1.0):
    """Statistics of a's rows plus w times b's rows, with b moved onto a's shifts (Chan et al.'s pairwise update;
    code/kva/ridge.py:142-156). Both are state() dicts over the same split and layers."""
    nb = b["n"]
    dx = b["cx"] - a["cx"]
    out = dict(a, n=a["n"] + w * nb)
    out["sx"] = a["sx"] + w * (b["sx"] + nb * dx)
    out["sxx"] = a["sxx"] + w * _moved(b["sx"], b["sxx"], nb, dx, dx)
    out["sy"], out["sxy"] = {}, {}
    for i in a["layers"]:
        dy = b["cy"][i] - a["cy"][i]
        out["sy"][i] = a["sy"][i] + w * (b["sy"][i] + nb * dy)
        out["sxy"][i] = a["sxy"][i] + w * _moved(b["sx"], b["sxy"][i], nb, dx, dy, s_col=b["sy"][i])
    return out


def raw_moments(state, i):
    """Uncentred sum(x x^T) and sum(x y_i^T) (fp64) rebuilt from the shifted sums."""
    n, cx, sx = state["n"], state["cx"].double(), state["sx"].double()
    xx = _moved(sx, state["sxx"].double(), n, cx, cx)
    xy = _moved(sx, state["sxy"][i].double(), n, cx, state["cy"][i].double(), s_col=state["sy"][i].double())
    return xx, xy
