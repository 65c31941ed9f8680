"""Row-parallel map fill (parallel/rowfill.py) on gloo ranks (CPU): every rank's exchanged fill projection must
equal its heads' columns of the same projection computed whole on one rank, for attention layers (with KV heads
replicated over more ranks than there are KV heads) and GDN layers, and for prefix lengths that do not divide by
the rank count. The sharded column layout is also checked against the head slicing that tp.shard applies."""
import os
import socket
from datetime import timedelta
from types import SimpleNamespace

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ridgefill_data_b200.parallel import rowfill as RF

CFG = SimpleNamespace(head_dim=8, n_heads=8, n_kv=2, gated_attn=True, gdn_nk=4, gdn_nv=8, gdn_dk=4, gdn_dv=6)


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _norm(x):
    return x * torch.rsqrt(x.square().mean(-1, keepdim=True) + 1e-6)


def _rank(rank, world, port, P, kind, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    try:
        g = torch.Generator().manual_seed(0)            # every rank draws the same inputs
        d = 16
        b = torch.randn(P, d, generator=g)
        w_map, c_map = torch.randn(d, d, generator=g) / 4, torch.randn(d, generator=g)
        plan = (RF.attention_columns if kind == "attn" else RF.gdn_columns)(CFG, world)
        cols = 2 * CFG.n_kv * CFG.head_dim if kind == "attn" else \
            2 * CFG.gdn_nk * CFG.gdn_dk + CFG.gdn_nv * CFG.gdn_dv + 2 * CFG.gdn_nv
        proj = torch.randn(cols, d, generator=g) / 4
        fill = RF.RowParallelFill()
        fill.proj[0] = proj
        lo, hi, _ = fill.row_block(P)
        x = torch.nn.functional.linear(b[lo:hi], w_map, c_map)
        local = fill.project_rows(0, x, _norm, torch.nn.functional.linear) if hi > lo else b.new_zeros(0, cols)
        got = fill.exchange(local, plan, P)
        whole = torch.nn.functional.linear(_norm(torch.nn.functional.linear(b, w_map, c_map)), proj)
        want = whole.index_select(1, plan[rank])
        ok = got.shape == want.shape and torch.allclose(got, want, atol=1e-5, rtol=1e-5)
        with open(f"{out}.{rank}", "w") as f:
            f.write("ok" if ok else f"mismatch {tuple(got.shape)} {tuple(want.shape)}")
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,P,kind", [(2, 10, "attn"), (4, 10, "attn"), (4, 5, "gdn"), (2, 7, "gdn"),
                                          (4, 3, "attn")])
def test_exchange_matches_whole_projection(tmp_path, world, P, kind):
    out = tmp_path / "r"
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, world, port, P, kind, str(out))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
        if p.is_alive():
            p.kill()
    for r in range(world):
        assert (tmp_path / f"r.{r}").read_text() == "ok", r


def test_column_plan_matches_head_sharding():
    """The attention plan picks the rows tp.shard_attention keeps for k and v; the GDN plan the rows
    tp.shard_gdn keeps for the conv channels, b and a (ranks in order)."""
    from ridgefill_data_b200.parallel import tp as TP
    d, hd = 16, CFG.head_dim
    qh = hd * 2
    qw = CFG.n_heads * qh
    for world in (2, 4, 8):
        full = torch.arange((qw + 2 * CFG.n_kv * hd) * d, dtype=torch.float32).reshape(-1, d)
        plan = RF.attention_columns(CFG, world)
        for r in range(world):
            w = {"qkv_p": full.clone(), "o": torch.zeros(d, CFG.n_heads * hd)}
            nq, nkv = TP.shard_attention(w, CFG, r, world)
            kept = w["qkv_p"][nq * qh:]                      # the rank's k | v rows
            assert torch.equal(kept, full[qw:][plan[r]])
    kd, vd, nv = CFG.gdn_nk * CFG.gdn_dk, CFG.gdn_nv * CFG.gdn_dv, CFG.gdn_nv
    conv = 2 * kd + vd
    full = torch.arange((conv + 2 * nv + vd) * d, dtype=torch.float32).reshape(-1, d)
    for world in (2, 4):
        plan = RF.gdn_columns(CFG, world)
        for r in range(world):
            w = {"in_p": full.clone(), "conv": torch.zeros(conv, 4), "A_log": torch.zeros(nv),
                 "dt_bias": torch.zeros(nv), "out": torch.zeros(d, vd)}
            nkl, nvl = TP.shard_gdn(w, CFG, r, world)
            width = 2 * nkl * CFG.gdn_dk + nvl * CFG.gdn_dv + 2 * nvl
            assert torch.equal(w["in_p"][:width], full[:conv + 2 * nv][plan[r]])


def test_fill_layout_is_refused_when_unknown():
    from ridgefill_data_b200.parallel import tp as TP
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(_port()))
    dist.init_process_group("gloo", rank=0, world_size=1)
    try:
        with pytest.raises(ValueError, match="layout"):
            TP.TensorParallel(mode="nccl", fill="diagonal")
        assert TP.TensorParallel(mode="nccl", fill="rows").row_fill is None      # one rank: nothing to exchange
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world", [2])
def test_prepare_on_packed_b200_weights(monkeypatch, world):
    """prepare() keeps the unsharded fill projections of a packed B200 hybrid; after tp.shard, each rank's plan
    columns of them are exactly the rows its sharded attention k|v and GDN conv / b / a projections hold. (The
    model is built on the CPU with the device set-up skipped: only its packed weights are read here.)"""
    from ridgefill_data_b200.models import b200
    from ridgefill_data_b200.models.checkpoint import RandomSource
    from ridgefill_data_b200.models.tiny import tiny_configs
    from ridgefill_data_b200.parallel import tp as TP
    monkeypatch.setattr(b200._B200, "_kernel_setup", lambda self: setattr(self, "_rope_tables", None))
    cfg = tiny_configs(8, 64)["qwen3.5-9b"].replace(intermediate=512)      # 4 FFN blocks of 128 rows
    if cfg.n_heads % world or cfg.gdn_nk % world or cfg.gdn_nv % world:
        pytest.skip("head counts do not split over this many ranks")
    for rank in range(world):
        model = b200.B200Hybrid(cfg, RandomSource(cfg, seed=0), device="cpu", dtype=torch.bfloat16)
        fill = RF.RowParallelFill.__new__(RF.RowParallelFill)
        fill.group, fill.rank, fill.world, fill.proj, fill.cols = None, rank, world, {}, {}
        fill.prepare(model)
        fake = SimpleNamespace(rank=rank, world=world, row_fill=None, group=None)
        TP.shard(model, fake)
        for i, w in enumerate(model.W):
            mine = fill.proj[i].index_select(0, fill.cols[i][rank])
            if model.layer_types[i] == "attn":
                q_rows = model.n_heads * cfg.head_dim * (2 if cfg.gated_attn else 1)
                assert torch.equal(mine, w["qkv_p"][q_rows:]), (rank, i)
            else:
                assert torch.equal(mine, w["in_p"][:model.conv_dim + 2 * model.nv]), (rank, i)
