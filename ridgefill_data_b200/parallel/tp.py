"""Tensor parallelism for the B200 models (one rank per GPU).

Sharding (column-parallel in, row-parallel out; activations replicated across ranks):
  attention   query heads split evenly; each rank keeps the K/V heads its query heads read (KV heads are
              replicated when there are fewer KV heads than ranks, e.g. 4 KV heads at TP 8); o_proj keeps the
              columns of the local heads
  GDN         key heads and value heads split evenly (value head h reads key head h // (nv / nk), so a rank's
              value heads read only its own key heads); in_proj rows, conv channels, A_log / dt_bias and out_proj
              columns follow
  MLP         the packed gate/up rows in whole 128-row blocks, down_proj the matching columns
  ridge maps  column-sharded: each rank computes output features [r d / N, (r + 1) d / N) of x_l = h_S W_l^T + c_l
              and the full x_l is gathered on every rank before the layer's RMSNorm + K/V / GDN projections
  norms, embedding and lm_head stay replicated
Communication per layer (the two row-parallel products, o_proj or out_proj and down_proj, summed over ranks; the
map fill's column gather in late layers):
  nccl        GEMM (residual added on rank 0 only) then an NCCL all-reduce; map slice then NCCL all-gather: the
              baseline
  fused       parallel/fused.py: GEMM epilogues store their tiles straight into peer memory (partials into the row
              owner's receive slot; map columns into every rank's x_l), the owner reduces, every rank gathers
  nvls        parallel/nvls.py: NVSwitch multicast: partials reduced in the switch (multimem.ld_reduce) and the sums
              multicast to every rank (multimem.st) by one kernel with its own cross-rank barriers; map slices
              multicast into every rank's x_l. With overlap > 1 the row-parallel product goes in row chunks: each
              chunk's GEMM runs on most SMs while the previous chunk's all-reduce runs on 32 CTAs on a second stream
With fill="rows" the map fill is row-parallel instead (parallel/rowfill.py): each rank maps a block of prefix rows
through the whole map and the unsharded fill projection, and an all-to-all delivers each rank its heads' columns.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm as G


class TensorParallel:
    def __init__(self, group=None, mode="nccl", fill="columns", overlap=1, overlap_min_rows=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.mode = mode
        self.fused = None
        self.fused_fill = None
        if fill not in ("columns", "rows"):
            raise ValueError(f"TP map-fill layout {fill!r} (columns | rows)")
        self.row_fill = None
        if fill == "rows" and self.world > 1:           # parallel/rowfill.py: row blocks and an all-to-all
            from .rowfill import RowParallelFill
            self.row_fill = RowParallelFill(group)
        if mode == "fused" and self.world > 1:
            from .fused import FusedMapFill, FusedRowParallel
            self.fused = FusedRowParallel(group)
            self.fused_fill = FusedMapFill(group)
        elif mode == "nvls" and self.world > 1:
            from .nvls import NvlsMapFill, NvlsRowParallel
            self.fused = NvlsRowParallel(group)
            self.fused_fill = NvlsMapFill(group)
            self.fused.overlap = int(overlap)            # row chunks: GEMM of one beside the all-reduce of another
            if overlap_min_rows is not None:
                self.fused.overlap_min_rows = int(overlap_min_rows)
        elif mode not in ("nccl", "fused", "nvls"):
            raise ValueError(f"TP communication mode {mode!r} (nccl | fused | nvls)")

    def row_parallel(self, y, w, h):
        """h + sum over ranks of y_r w_r^T (each rank holds its K-slice y_r, w_r)."""
        if self.world == 1:
            return G.linear(y, w, residual=h)
        if self.fused is not None:
            return self.fused(y, w, h)
        a = G.linear(y, w, residual=h if self.rank == 0 else None)
        dist.all_reduce(a, group=self.group)
        return a

    def map_fill(self, b, W, B):
        """x = b W^T + c with the map column-sharded over ranks (this rank computes output features
        [r d / N, (r + 1) d / N)); returns the full [rows, d] on every rank."""
        d = W.shape[0]
        if self.world == 1:
            return G.linear(b, W, bias=B)
        c0, c1 = self.rank * d // self.world, (self.rank + 1) * d // self.world
        if self.fused_fill is not None:
            return self.fused_fill(b, W[c0:c1], B[c0:c1], d)
        part = G.linear(b, W[c0:c1], bias=B[c0:c1])
        out = torch.empty(self.world * b.shape[0], c1 - c0, dtype=part.dtype, device=part.device)
        dist.all_gather_into_tensor(out, part, group=self.group)
        return out.view(self.world, b.shape[0], c1 - c0).permute(1, 0, 2).reshape(b.shape[0], d)

    def owns(self, t):
        """True when t lives in a rotating communication buffer (reused a few layers later)."""
        return self.fused is not None and hasattr(self.fused, "owns") and self.fused.owns(t)

    def close(self):
        for f in (self.fused, self.fused_fill):
            if f is not None:
                f.close()
        self.fused = self.fused_fill = None


def _span(total, world, rank, what):
    if total % world:
        raise ValueError(f"{what}: {total} is not divisible by {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def shard_attention(w, cfg, rank, world):
    """Slice one packed attention layer in place; returns (local q heads, local kv heads)."""
    hd, hq, hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv
    qh = hd * (2 if cfg.gated_attn else 1)
    h0, h1 = _span(hq, world, rank, "query heads")
    rep = hq // hkv
    k0, k1 = h0 // rep, (h1 - 1) // rep + 1
    qkv = w["qkv_p"]
    qw = hq * qh
    q = qkv[h0 * qh:h1 * qh]
    k = qkv[qw + k0 * hd:qw + k1 * hd]
    v = qkv[qw + hkv * hd + k0 * hd:qw + hkv * hd + k1 * hd]
    p = torch.cat((q, k, v)).contiguous()
    nq = (h1 - h0) * qh
    nkv = (k1 - k0) * hd
    w.update(qkv_p=p, q=p[:nq], k=p[nq:nq + nkv], v=p[nq + nkv:], o=w["o"][:, h0 * hd:h1 * hd].contiguous())
    return h1 - h0, k1 - k0


def shard_gdn(w, cfg, rank, world):
    """Slice one packed Gated DeltaNet layer in place; returns (local key heads, local value heads)."""
    nk, nv, dk, dv = cfg.gdn_nk, cfg.gdn_nv, cfg.gdn_dk, cfg.gdn_dv
    a0, a1 = _span(nk, world, rank, "GDN key heads")
    v0, v1 = _span(nv, world, rank, "GDN value heads")
    p = w["in_p"]
    kd, vd = nk * dk, nv * dv
    C = 2 * kd + vd
    rows = [p[a0 * dk:a1 * dk], p[kd + a0 * dk:kd + a1 * dk], p[2 * kd + v0 * dv:2 * kd + v1 * dv],
            p[C + v0:C + v1], p[C + nv + v0:C + nv + v1], p[C + 2 * nv + v0 * dv:C + 2 * nv + v1 * dv]]
    conv = w["conv"]
    conv_l = torch.cat((conv[a0 * dk:a1 * dk], conv[kd + a0 * dk:kd + a1 * dk],
                        conv[2 * kd + v0 * dv:2 * kd + v1 * dv])).contiguous()
    np_ = torch.cat(rows).contiguous()
    nkl, nvl = a1 - a0, v1 - v0
    Cl = 2 * nkl * dk + nvl * dv
    w.update(in_p=np_, qkv=np_[:Cl], b=np_[Cl:Cl + nvl], a=np_[Cl + nvl:Cl + 2 * nvl], z=np_[Cl + 2 * nvl:],
             conv=conv_l, A_log=w["A_log"][v0:v1].contiguous(), dt_bias=w["dt_bias"][v0:v1].contiguous(),
             out=w["out"][:, v0 * dv:v1 * dv].contiguous())
    return nkl, nvl


def shard_mlp(w, rank, world, block=128):
    gu = w["gu_p"]
    nblk = gu.shape[0] // (2 * block)
    b0, b1 = _span(nblk, world, rank, "FFN 128-row blocks")
    w.update(gu_p=gu[b0 * 2 * block:b1 * 2 * block].contiguous(),
             down=w["down"][:, b0 * block:b1 * block].contiguous())


def shard(model, tp: TensorParallel):
    """Shard a B200 model's weights for tp.rank of tp.world (in place) and attach the reduction."""
    cfg = model.cfg
    rank, world = tp.rank, tp.world
    if world == 1:
        model.tp = tp
        return model
    if getattr(tp, "row_fill", None) is not None:
        tp.row_fill.prepare(model)           # the unsharded fill projections, before the slicing below
    local = {}
    for i, w in enumerate(model.W):
        if model.layer_types[i] == "attn":
            local["attn"] = shard_attention(w, cfg, rank, world)
        else:
            local["gdn"] = shard_gdn(w, cfg, rank, world)
        if not cfg.moe:
            shard_mlp(w, rank, world)
    if cfg.moe:       # the MoE MLPs are expert-parallel over the same ranks
        from .ep import ExpertParallel
        ExpertParallel(tp.group, tp).shard(model)
    if "attn" in local:
        model.n_heads, model.n_kv = local["attn"]
    if "gdn" in local:
        model.nk, model.nv = local["gdn"]
        model.conv_dim = 2 * model.nk * cfg.gdn_dk + model.nv * cfg.gdn_dv
        model.vd = model.nv * cfg.gdn_dv
    model.tp = tp
    torch.cuda.empty_cache()
    return model
