"""Tensor-parallel weight slicing (parallel/tp.py) on the CPU: every rank's slice of a packed attention, Gated
DeltaNet and MLP layer holds exactly its heads / blocks, the ranks together cover every query head, value head and
FFN block once, each rank keeps the K/V heads its query heads read (replicated when there are fewer K/V heads than
ranks), and the local value-to-key head mapping equals the global one."""
from types import SimpleNamespace

import pytest
import torch

from ridgefill_data_b200.parallel.tp import shard_attention, shard_gdn, shard_mlp

CFG = SimpleNamespace(head_dim=8, n_heads=8, n_kv=2, gated_attn=True, gdn_nk=4, gdn_nv=8, gdn_dk=4, gdn_dv=6)
D = 16


def _row_ids(n, cols):
    """[n, cols] whose row r holds r everywhere (a row's value names it)."""
    return torch.arange(n, dtype=torch.float32)[:, None].expand(n, cols).clone()


def _col_ids(rows, n):
    return torch.arange(n, dtype=torch.float32)[None, :].expand(rows, n).clone()


def _attn_layer():
    hd, hq, hkv = CFG.head_dim, CFG.n_heads, CFG.n_kv
    qh = hd * (2 if CFG.gated_attn else 1)
    return dict(qkv_p=_row_ids(hq * qh + 2 * hkv * hd, D), o=_col_ids(D, hq * hd))


def _gdn_layer():
    nk, nv, dk, dv = CFG.gdn_nk, CFG.gdn_nv, CFG.gdn_dk, CFG.gdn_dv
    C = 2 * nk * dk + nv * dv
    return dict(in_p=_row_ids(C + 2 * nv + nv * dv, D), conv=_row_ids(C, 4), A_log=torch.arange(nv, dtype=torch.float32),
                dt_bias=torch.arange(nv, dtype=torch.float32) + 100, out=_col_ids(D, nv * dv))


@pytest.mark.parametrize("world", [2, 4, 8])
def test_attention_slices(world):
    hd, hq, hkv = CFG.head_dim, CFG.n_heads, CFG.n_kv
    qh, rep = 2 * hd, hq // hkv
    qw = hq * qh
    seen_q = []
    for rank in range(world):
        w = _attn_layer()
        nq, nkv = shard_attention(w, CFG, rank, world)
        rows = w["qkv_p"][:, 0].long().tolist()
        heads = sorted({r // qh for r in rows[:nq * qh]})
        assert rows[:nq * qh] == [h * qh + j for h in heads for j in range(qh)]         # whole q (+ gate) heads
        kv_heads = sorted({h // rep for h in heads})                                      # the K/V heads they read
        assert nkv == len(kv_heads)
        assert rows[nq * qh:nq * qh + nkv * hd] == [qw + g * hd + j for g in kv_heads for j in range(hd)]
        assert rows[nq * qh + nkv * hd:] == [qw + (hkv + g) * hd + j for g in kv_heads for j in range(hd)]
        assert w["o"][0].long().tolist() == [h * hd + j for h in heads for j in range(hd)]
        assert torch.equal(w["q"], w["qkv_p"][:nq * qh])
        seen_q += heads
    assert sorted(seen_q) == list(range(hq))


@pytest.mark.parametrize("world", [2, 4])
def test_gdn_slices_and_head_mapping(world):
    nk, nv, dk, dv = CFG.gdn_nk, CFG.gdn_nv, CFG.gdn_dk, CFG.gdn_dv
    kd, C = nk * dk, 2 * nk * dk + nv * dv
    seen_v = []
    for rank in range(world):
        w = _gdn_layer()
        nkl, nvl = shard_gdn(w, CFG, rank, world)
        a0, v0 = rank * nk // world, rank * nv // world
        rows = w["in_p"][:, 0].long().tolist()
        Cl = 2 * nkl * dk + nvl * dv
        want = ([a0 * dk + j for j in range(nkl * dk)] + [kd + a0 * dk + j for j in range(nkl * dk)]
                + [2 * kd + v0 * dv + j for j in range(nvl * dv)] + [C + v0 + j for j in range(nvl)]
                + [C + nv + v0 + j for j in range(nvl)] + [C + 2 * nv + v0 * dv + j for j in range(nvl * dv)])
        assert rows == want
        assert w["conv"][:, 0].long().tolist() == want[:Cl]
        assert w["A_log"].long().tolist() == list(range(v0, v0 + nvl))
        assert w["dt_bias"].long().tolist() == [100 + v for v in range(v0, v0 + nvl)]
        assert w["out"][0].long().tolist() == [v0 * dv + j for j in range(nvl * dv)]
        for h in range(nvl):               # local value head h reads local key head h / (nvl / nkl): the global pair
            assert a0 + h // (nvl // nkl) == (v0 + h) // (nv // nk)
        seen_v += list(range(v0, v0 + nvl))
    assert seen_v == list(range(nv))


@pytest.mark.parametrize("world", [2, 4])
def test_mlp_blocks(world):
    block, nblk = 4, 8
    gu = _row_ids(2 * block * nblk, D)
    down = _col_ids(D, block * nblk)
    got_rows, got_cols = [], []
    for rank in range(world):
        w = dict(gu_p=gu.clone(), down=down.clone())
        shard_mlp(w, rank, world, block=block)
        got_rows += w["gu_p"][:, 0].long().tolist()
        got_cols += w["down"][0].long().tolist()
        # a rank's gate/up rows are whole [gate block; up block] pairs and its down columns the same features
        feats = w["down"][0].long().tolist()
        assert [r for r in w["gu_p"][:, 0].long().tolist()] == [
            2 * block * (f // block) + (f % block) + u * block for f0 in range(0, len(feats), block)
            for u in (0, 1) for f in feats[f0:f0 + block]]
    assert got_rows == list(range(2 * block * nblk)) and got_cols == list(range(block * nblk))


def test_uneven_split_is_refused():
    with pytest.raises(ValueError, match="not divisible"):
        shard_attention(_attn_layer(), CFG, 0, 3)
