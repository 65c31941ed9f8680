"""Expert parallelism for the MoE layers (one rank per GPU), used together with tensor parallelism of the
attention / Gated DeltaNet layers, so every rank holds every token's activations when the MLP starts.

Rank r owns experts [r E / N, (r + 1) E / N). Every rank routes all tokens (the router is replicated), keeps the
(token, slot) pairs whose expert it owns, gathers those rows expert-sorted, runs its experts on the grouped
tcgen05 GEMM and forms its partial sum_k w y for every token; rank 0 also adds the residual and the gated shared
expert. The partials are summed over ranks (the expert combine) with the tensor-parallel reduction: NCCL
all-reduce, or (nvls mode) the combine writes straight into the symmetric partial buffer and the NVSwitch multicast
all-reduce of parallel/nvls.py sums it. With replicated activations this moves one
[tokens, d] all-reduce per MoE layer instead of an all-to-all dispatch of up to top_k copies of each row.
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm as G
from ..ops import moe as MO


class ExpertParallel:
    def __init__(self, group=None, tp=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.tp = tp

    def shard(self, model):
        E = model.cfg.n_experts
        if E % self.world:
            raise ValueError(f"{E} experts are not divisible by {self.world} ranks")
        per = E // self.world
        self.e0, self.E_local = self.rank * per, per
        for i, w in enumerate(model.W):
            if "experts_gu_p" in w:
                w["experts_gu_p"] = w["experts_gu_p"][self.e0:self.e0 + per].contiguous()
                w["experts_down"] = w["experts_down"][self.e0:self.e0 + per].contiguous()
        model.ep = self
        torch.cuda.empty_cache()
        return model

    def moe(self, model, w, h, x, logits):
        E, k = model.cfg.n_experts, model.cfg.top_k
        idx, wts = MO.router_topk(logits, E, k)
        xp, pos, seg, tiles = MO.align(idx, self.E_local, x, e0=self.e0)
        act = MO.grouped(xp, w["experts_gu_p"], seg, tiles, swiglu=True)
        y = MO.grouped(act, w["experts_down"], seg, tiles, swiglu=False)
        nvls = getattr(self.tp, "fused", None) if self.world > 1 else None
        nvls = nvls if hasattr(nvls, "allreduce_") else None
        rows, d = h.shape
        out = nvls.partial_view(rows, d) if nvls is not None else None   # combine straight into the symmetric buffer
        if self.rank == 0:
            ys = G.linear(G.swiglu_linear(x, w["sh_gu_p"]), w["sh_down"])
            part = MO.combine(h, y, pos, wts, ys, logits[:, E], out=out)
        else:
            part = MO.combine(None, y, pos, wts, n=rows, d=d, out=out)
        if nvls is not None:
            return nvls.allreduce_(rows, d)                              # NVSwitch multicast all-reduce
        if self.world > 1:
            dist.all_reduce(part, group=self.group)
        return part
