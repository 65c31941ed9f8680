"""Analytic prefill cost (multiply-accumulates) per arm, from the model shape (code/kva/compute.py semantics).

Counted per token: every linear map (attention q/k/v/o or Gated DeltaNet in/out projections, MLP or the
active experts of an MoE MLP), causal attention (QK^T and PV: 2 x keys x heads x head_dim), the GDN conv
and recurrence (4 x value heads x dk x dv; 3 without the output read), the ridge projector (hidden^2 per
prefix token per late layer) and the lm_head on the last token. Norms, RoPE, softmax and other
elementwise work are not counted. Arms:
  exact     every layer on every token
  ridgefill layers < S on every token; layers >= S: the P = N - T prefix tokens get projector + fill only
            (attention: K/V projections; GDN: in-projections, conv, state update without output), the tail
            runs exactly over the whole context
  noproj    ridgefill without the projector (identity fill)
  skip      layers >= S see only the tail
  swiftkv   late layers' K/V for every token, the full late layers for the last token only
  bypass    ridgefill plus r exact prefix rows (mean position pos x P)
  repair    the late layers run exactly over the first R cached rows (between turns)
The counting rules are the reference's so analytic speedups stay comparable; `seconds()` adds a B200 time
estimate (GEMM MACs at the measured bf16 rate, the attention/scan work at stated fractions of it).
"""
from __future__ import annotations

from ..models.config import ModelConfig


class CostModel:
    def __init__(self, cfg: ModelConfig):
        self.cfg = cfg
        c = cfg
        self.L, self.H, self.V = c.n_layers, c.hidden, c.vocab
        self.hq, self.hkv, self.d = c.n_heads, c.n_kv, c.head_dim
        self.types = list(c.layer_types)
        self.gated = c.gated_attn
        self.nk, self.nv, self.dk, self.dv, self.kc = c.gdn_nk, c.gdn_nv, c.gdn_dk, c.gdn_dv, c.conv_k

    # ---- per-token MACs
    def mlp(self):
        c = self.cfg
        if c.moe:
            routed = 3 * self.H * c.moe_intermediate * c.top_k
            shared = 3 * self.H * c.shared_intermediate + self.H
            return routed + shared + self.H * c.n_experts
        return 3 * self.H * c.intermediate

    def attn_linear(self):
        q = self.H * self.hq * self.d * (2 if self.gated else 1)
        return q + 2 * self.H * self.hkv * self.d + self.hq * self.d * self.H

    def attn_fill(self):
        return 2 * self.H * self.hkv * self.d

    def gdn_inproj(self):
        conv = 2 * self.nk * self.dk + self.nv * self.dv
        return self.H * conv + 2 * self.H * self.nv + conv * self.kc

    def gdn_linear(self):
        return self.gdn_inproj() + 2 * self.H * self.nv * self.dv        # + z and out_proj

    def gdn_rec(self, read=True):
        return (4 if read else 3) * self.nv * self.dk * self.dv

    def attn_ctx(self, first, last):
        """QK^T + PV MACs of tokens at positions first..last-1 (each attends to position + 1 keys)."""
        n = last - first
        return 2 * self.hq * self.d * n * (first + last + 1) / 2

    def layer_exact(self, i, first, last):
        n = last - first
        if self.types[i] == "attn":
            return n * (self.attn_linear() + self.mlp()) + self.attn_ctx(first, last)
        return n * (self.gdn_linear() + self.gdn_rec() + self.mlp())

    def layer_fill(self, i, n):
        if self.types[i] == "attn":
            return n * self.attn_fill()
        return n * (self.gdn_inproj() + self.gdn_rec(read=False))

    def proj(self, i, proj_types=None, rank=None):
        if proj_types is not None and self.types[i] not in proj_types:
            return 0
        return self.H * self.H if rank is None else min(self.H * self.H, 2 * self.H * rank)

    # ---- arms
    def exact(self, n):
        return sum(self.layer_exact(i, 0, n) for i in range(self.L)) + self.H * self.V

    def ridgefill(self, n, split, tail, projector=True, kvfold=False, proj_types=None, rank=None, context=0,
                  refresh=None):
        p = max(0, n - tail)
        c = sum(self.layer_exact(i, 0, n) for i in range(split))
        for i in range(split, self.L):
            c += (self.layer_exact(i, 0, p) if i == refresh else self.layer_fill(i, p)) + self.layer_exact(i, p, n)
            if projector and not (kvfold and self.types[i] == "attn"):
                wide = 1 + context if refresh is None or i <= refresh else 1
                c += p * wide * self.proj(i, proj_types, rank)
        return c + self.H * self.V

    def skip(self, n, split, tail):
        return (sum(self.layer_exact(i, 0, n) for i in range(split))
                + sum(self.layer_exact(i, 0, tail) for i in range(split, self.L)) + self.H * self.V)

    def tail_budget(self, n, split, tail):
        """Fewest extra tail rows E for which skip with tail + E costs at least ridgefill at (split, tail)."""
        target, lo, hi = self.ridgefill(n, split, tail), 0, n - tail
        while lo < hi:
            mid = (lo + hi) // 2
            if self.skip(n, split, tail + mid) >= target:
                hi = mid
            else:
                lo = mid + 1
        return lo

    def swiftkv(self, n, split=16):
        c = sum(self.layer_exact(i, 0, n) for i in range(split))
        c += (self.L - split) * n * (2 * self.H * self.hkv * self.d)
        c += sum(self.layer_exact(i, n - 1, n) for i in range(split, self.L))
        return c + self.H * self.V

    def qattn_select(self, n, split, window=64, layers=(3, 7, 11, 15)):
        q = self.H * self.hq * self.d * (2 if self.gated else 1)
        used = [i for i in layers if i < split and self.types[i] == "attn"]
        return len(used) * (window * q + self.attn_ctx(n - window, n) / 2)

    def bypass(self, n, split, tail, rows, select=None, gdn="efficient", pos=0.5, proj_types=None, rank=None,
               refresh=None):
        p = max(0, n - tail)
        r = max(0, min(int(rows), p))
        if gdn not in ("efficient", "reference"):
            raise ValueError(gdn)
        ref = gdn == "reference"
        c = sum(self.layer_exact(i, 0, n) for i in range(split))
        for i in range(split, self.L):
            c += self.layer_exact(i, p, n) + (p if ref else p - r) * self.proj(i, proj_types, rank)
            if i == refresh:
                c += self.layer_exact(i, 0, p)
                continue
            c += self.layer_fill(i, p - r)
            if self.types[i] == "attn":
                c += r * (self.attn_linear() + self.mlp() + 2 * self.hq * self.d * pos * (p + 1))
            else:
                c += r * (self.gdn_linear() + self.gdn_rec() + self.mlp())
            if ref and self.types[i] == "gdn":
                c += (p - r) * self.nv * self.dk * self.dv
        if select == "qattn":
            c += self.qattn_select(n, split)
        return c + self.H * self.V

    def bypass_arm(self, n, split, tail, kind, rows=None, budget=None, gdn="efficient", pos=0.5, proj_types=None,
                   rank=None, refresh=None):
        """A bypass arm of select kind `kind` with `rows` exact rows, or round(budget n) (the qattn rule);
        tail_match spends them on the exact tail instead."""
        if rows is None:
            rows = round(budget * n)
        if kind == "tail_match":
            return self.ridgefill(n, split, tail + rows, proj_types=proj_types, rank=rank, refresh=refresh)
        if kind not in ("digits", "qattn", "random"):
            raise ValueError(f"bypass kind {kind!r}")
        return self.bypass(n, split, tail, rows, select=kind, gdn=gdn, pos=pos, proj_types=proj_types, rank=rank,
                           refresh=refresh)

    def bypass_speedup(self, n, split, tail, kind, rows=None, budget=None, gdn="efficient", pos=0.5, proj_types=None,
                       rank=None):
        return self.exact(n) / self.bypass_arm(n, split, tail, kind, rows, budget, gdn, pos, proj_types, rank)

    def repair(self, split, rows):
        return sum(self.layer_exact(i, 0, rows) for i in range(split, self.L))

    def repair_selected(self, split, rows, prefix, pos=0.5):
        c = 0
        for i in range(split, self.L):
            if self.types[i] == "attn":
                c += rows * (self.attn_linear() + self.mlp() + 2 * self.hq * self.d * pos * (prefix + 1))
            else:
                c += rows * (self.gdn_linear() + self.gdn_rec() + self.mlp())
        return c

    def speedup(self, n, fill, split=None, tail=0, fill_by_type=None, rank=None, context=0, refresh=None):
        base = self.exact(n)
        if fill == "exact":
            return 1.0
        if fill == "swiftkv_native":
            return base / self.swiftkv(n, split)
        if fill == "kvfold":
            return base / self.ridgefill(n, split, tail, kvfold=True)
        if fill == "by_type":
            return base / self.ridgefill(n, split, tail, proj_types=proj_types_of(fill_by_type), rank=rank)
        return base / self.ridgefill(n, split, tail, projector=fill == "proj", rank=rank, context=context,
                                     refresh=refresh)

    # ---- B200 time estimate
    def seconds(self, macs, tflops=1414.3, eff=0.85):
        """MACs -> seconds at `eff` of the measured sustained bf16 rate (TFLOP/s, 2 FLOPs per MAC)."""
        return 2 * macs / (tflops * 1e12 * eff)


def proj_types_of(fill_by_type):
    """The late layer types ('attn', 'gdn') a fill_by_type runs the ridge map on."""
    return {"attn" if t == "attention" else t for t, f in fill_by_type.items() if f == "proj"}


def diagnostic(fill, fill_by_type=None, exact_part=None, rescale=None):
    """True for arms that read the true late-layer inputs (not deployable)."""
    return (exact_part is not None or rescale in ("knorm", "kdir", "vnorm")
            or "oracle" in (fill_by_type.values() if fill == "by_type" else (fill,)))
