"""Row-parallel RidgeFill prefix fill under tensor parallelism (opt-in: TensorParallel(fill="rows")).

The default fill is column-parallel: every rank maps all P prefix rows through its column slice of each late
layer's map and all-gathers the full x_l (P x d values arrive at every rank per layer), because the layer's
RMSNorm needs whole rows before the sharded K/V or GDN projections can run. At TP 8 on the 27B hybrid that gather
dominates the fill.

Here each rank takes a contiguous block of P / N rows instead and runs it through the whole map, the row-wise
RMSNorm and the layer's fill projection for every head (the unsharded k|v rows of an attention layer, or the
conv-channel, b and a rows of a GDN layer, kept aside before sharding). An all-to-all then hands every rank the
columns of its own heads for all P rows, which is exactly what its sharded K/V write or GDN scan consumes:

    bytes received per rank and layer   column fill: P x d x (N - 1) / N     row fill: P x cols(local heads)

(27B hybrid, N = 8: d = 5120 against about 1300 columns for a GDN layer and 512 for an attention layer whose 4 KV
heads are replicated over 8 ranks). The FLOPs are the same as the column fill's; the price is memory: each rank
keeps the whole maps (they already sit on every rank) and the unsharded fill projections (about 5 GB for the 27B
hybrid).

Rows are padded to a multiple of N with zeros; the padded rows are dropped after the exchange. The exchange is a
torch.distributed all_to_all_single, so the same code runs on NCCL and, for the tests, on gloo.
"""
from __future__ import annotations

import torch
import torch.distributed as dist
import torch.nn.functional as F


def _ranges(*spans):
    return torch.cat([torch.arange(a, b) for a, b in spans if b > a])


def _head_span(total, world, rank, what):
    if total % world:
        raise ValueError(f"{what}: {total} is not divisible by {world} ranks")
    per = total // world
    return rank * per, (rank + 1) * per


def attention_columns(cfg, world):
    """Per rank, the columns of the unsharded [k | v] fill projection that its KV heads read (KV heads shared by
    several ranks, as at 4 KV heads over 8 ranks, go to each of them)."""
    hd, hq, hkv = cfg.head_dim, cfg.n_heads, cfg.n_kv
    group = hq // hkv
    plan = []
    for r in range(world):
        h0, h1 = _head_span(hq, world, r, "query heads")
        k0, k1 = h0 // group, (h1 - 1) // group + 1
        plan.append(_ranges((k0 * hd, k1 * hd), (hkv * hd + k0 * hd, hkv * hd + k1 * hd)))
    return plan


def gdn_columns(cfg, world):
    """Per rank, the columns of the unsharded [conv channels | b | a] projection of a GDN layer that its key and
    value heads read, in the order of the rank's sharded in_proj (q block, k block, v block, b, a)."""
    nk, nv, dk, dv = cfg.gdn_nk, cfg.gdn_nv, cfg.gdn_dk, cfg.gdn_dv
    kd, vd = nk * dk, nv * dv
    conv = 2 * kd + vd
    plan = []
    for r in range(world):
        a0, a1 = _head_span(nk, world, r, "GDN key heads")
        v0, v1 = _head_span(nv, world, r, "GDN value heads")
        plan.append(_ranges((a0 * dk, a1 * dk), (kd + a0 * dk, kd + a1 * dk), (2 * kd + v0 * dv, 2 * kd + v1 * dv),
                            (conv + v0, conv + v1), (conv + nv + v0, conv + nv + v1)))
    return plan


class RowParallelFill:
    """The row-block fill of one tensor-parallel group. prepare() must see the model before tp.shard() slices it."""

    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.proj = {}            # layer -> unsharded fill projection [cols, d]
        self.cols = {}            # layer -> per rank, the projection columns its heads read

    # ------------------------------------------------------------------------------------------ set-up
    def prepare(self, model):
        """Keep every layer's unsharded fill projection and the column plan of its layer type."""
        cfg = model.cfg
        plans = {}
        for i, w in enumerate(model.W):
            if model.layer_types[i] == "attn":
                q_rows = cfg.n_heads * cfg.head_dim * (2 if cfg.gated_attn else 1)
                self.proj[i] = w["qkv_p"][q_rows:].clone()
                kind = "attn"
            else:
                conv = 2 * cfg.gdn_nk * cfg.gdn_dk + cfg.gdn_nv * cfg.gdn_dv
                self.proj[i] = w["in_p"][:conv + 2 * cfg.gdn_nv].clone()
                kind = "gdn"
            if kind not in plans:
                plans[kind] = [c.to(self.proj[i].device) for c in
                               (attention_columns if kind == "attn" else gdn_columns)(cfg, self.world)]
            self.cols[i] = plans[kind]

    # ------------------------------------------------------------------------------------------ pieces
    def row_block(self, P):
        """(first row, end row, rows per rank after padding) of this rank's block of P rows."""
        per = -(-P // self.world)
        lo = min(P, self.rank * per)
        return lo, min(P, lo + per), per

    def exchange(self, local, plan, P):
        """local [rows of this rank's block, cols] -> [P, this rank's columns]: every rank sends each peer the
        peer's columns of its own rows (an all-to-all)."""
        per = -(-P // self.world)
        width = plan[self.rank].numel()
        if any(c.numel() != width for c in plan):
            raise ValueError("the column plan gives the ranks different widths")
        padded = local
        if local.shape[0] < per:
            padded = F.pad(local, (0, 0, 0, per - local.shape[0]))
        send = torch.stack([padded.index_select(1, c) for c in plan]).contiguous()      # [N, per, width]
        recv = torch.empty_like(send)
        dist.all_to_all_single(recv, send, group=self.group)
        return recv.reshape(self.world * per, width)[:P]

    def project_rows(self, i, rows, norm, linear):
        """This rank's rows of layer i's inputs -> the fill projection for every head: linear(norm(rows), W)."""
        return linear(norm(rows), self.proj[i])

    # ------------------------------------------------------------------------------------------ B200 fill
    def fill_layer(self, model, i, b, pos, cache, w, c):
        """The prefix fill of late layer i on a B200 model: the map over this rank's row block, the exchange,
        then the rank's own K/V write or GDN state pass."""
        from ..ops import gemm as G
        P = b.shape[0]
        lo, hi, _ = self.row_block(P)
        if hi > lo:
            x = G.linear(b[lo:hi], w, bias=c)
            local = self.project_rows(i, x, lambda t: model._norm(t, model.W[i]["ln1"]), G.linear)
        else:                                   # fewer rows than ranks: this rank only receives
            local = b.new_zeros(0, self.proj[i].shape[0])
        mine = self.exchange(local, self.cols[i], P)
        if model.layer_types[i] == "attn":
            model._write_kv(i, mine, pos, cache[i])
        else:
            model._gdn_core_dev(i, mine, cache, False)
