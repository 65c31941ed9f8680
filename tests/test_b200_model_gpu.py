"""B200 models (sm_100a kernels) vs the torch models on the same random weights (bf16, cuda): exact
forward logits, ridge-fill prefill through the engine, decode steps."""
import pytest
import torch

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.prefill import finish, run_lower
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.config import ModelConfig, _hybrid_types
from ridgefill_data_b200.ridge.projector import Projector

pytestmark = pytest.mark.gpu

HYB = ModelConfig(arch="qwen3_5", n_layers=8, hidden=512, vocab=1024, n_heads=4, n_kv=1, head_dim=256,
                  intermediate=1024, eps=1e-6, rope_theta=1e7, partial_rotary=0.25, layer_types=_hybrid_types(8),
                  gdn_nk=2, gdn_nv=4, gdn_dk=128, gdn_dv=128, conv_k=4, name="tiny-hybrid")
LLAMA = ModelConfig(arch="llama", n_layers=4, hidden=512, vocab=1024, n_heads=8, n_kv=2, head_dim=64,
                    intermediate=1536, eps=1e-5, rope_theta=5e5, rope_type="llama3",
                    rope_llama3=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                     original_max_position_embeddings=8192), name="tiny-llama-gpu")
QWEN3 = ModelConfig(arch="qwen3", n_layers=4, hidden=512, vocab=1024, n_heads=4, n_kv=2, head_dim=128,
                    intermediate=1024, eps=1e-6, rope_theta=1e6, name="tiny-qwen3-gpu")


def _pair(cfg):
    ref = from_config(cfg, seed=0, device="cuda", std=0.05)
    dut = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    return ref, dut


def _fp32(cfg):
    return from_config(cfg, seed=0, device="cuda", std=0.05, dtype=torch.float32)


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm()).item()


@pytest.mark.parametrize("cfg", [HYB, LLAMA, QWEN3], ids=lambda c: c.name)
def test_forward_exact_matches_torch(cfg):
    ref, dut = _pair(cfg)
    ids = torch.randint(0, cfg.vocab, (333,), generator=torch.Generator().manual_seed(1)).cuda()
    keep = torch.arange(300, 333, device="cuda")
    lr, _ = ref.forward_exact(ids, keep=keep)
    ld, _ = dut.forward_exact(ids, keep=keep)
    l32, _ = _fp32(cfg).forward_exact(ids, keep=keep)
    # the kernel path is no further from fp32 than the torch bf16 path (plus a small margin)
    assert _rel(ld, l32) < 1.5 * _rel(lr, l32) + 5e-3, (_rel(ld, l32), _rel(lr, l32))
    assert (ld.argmax(-1) == l32.argmax(-1)).float().mean() > 0.8


@pytest.mark.parametrize("cfg", [HYB, LLAMA], ids=lambda c: c.name)
def test_ridge_fill_prefill_matches_torch(cfg):
    ref, dut = _pair(cfg)
    split = cfg.n_layers // 2
    g = torch.Generator(device="cuda").manual_seed(3)
    d = cfg.hidden
    W = {i: (torch.eye(d, device="cuda") + 0.01 * torch.randn(d, d, device="cuda", generator=g)).bfloat16()
         for i in range(split, cfg.n_layers)}
    B = {i: (0.01 * torch.randn(d, device="cuda", generator=g)).bfloat16() for i in range(split, cfg.n_layers)}
    arm = Arm("ridgefill", split=split, tail=100, fill="proj", projector=Projector(split, W, B))
    ids = torch.randint(0, cfg.vocab, (400,), generator=torch.Generator().manual_seed(2)).cuda()
    out = {}
    for name, m in (("ref", ref), ("dut", dut), ("f32", _fp32(cfg))):
        hs, lower = run_lower(m, ids, [split])
        out[name] = finish(m, ids, hs[split], lower, arm, 4)
    e_dut, e_ref = _rel(out["dut"][0], out["f32"][0]), _rel(out["ref"][0], out["f32"][0])
    assert e_dut < 1.5 * e_ref + 5e-3, (e_dut, e_ref)
    for i in range(split, cfg.n_layers):
        cr, cd = out["ref"][1][i], out["dut"][1][i]
        if cfg.layer_types[i] == "attn":
            assert _rel(cd["k"], cr["k"]) < 3e-2 and _rel(cd["v"], cr["v"]) < 3e-2
        else:
            assert _rel(cd["rec"], cr["rec"]) < 5e-2


def test_decode_steps_match_torch():
    ref, dut = _pair(HYB)
    f32 = _fp32(HYB)
    ids = torch.randint(0, HYB.vocab, (130,), generator=torch.Generator().manual_seed(4)).cuda()
    models = dict(ref=ref, dut=dut, f32=f32)
    caches = {k: m.forward_exact(ids[:128])[1] for k, m in models.items()}
    for t in (128, 129):
        pos = torch.tensor([t], device="cuda")
        lg = {}
        for k, m in models.items():
            h = m.embed(ids[t:t + 1])
            for i in range(HYB.n_layers):
                h = m.layer(i, h, pos, caches[k])
            lg[k] = m.logits(h)
        e_dut, e_ref = _rel(lg["dut"], lg["f32"]), _rel(lg["ref"], lg["f32"])
        assert e_dut < 1.5 * e_ref + 5e-3, (t, e_dut, e_ref)


MOE = ModelConfig(arch="qwen3_5_moe", n_layers=4, hidden=512, vocab=1024, n_heads=4, n_kv=1, head_dim=256,
                  intermediate=0, eps=1e-6, rope_theta=1e7, partial_rotary=0.25, layer_types=_hybrid_types(4),
                  gdn_nk=2, gdn_nv=4, gdn_dk=128, gdn_dv=128, conv_k=4, n_experts=16, top_k=4,
                  moe_intermediate=256, shared_intermediate=256, name="tiny-moe")


def test_router_topk_matches_torch():
    from ridgefill_data_b200.ops import moe as MO
    from ridgefill_data_b200.ops.oracle import router_topk
    torch.manual_seed(0)
    logits = torch.randn(300, 520, device="cuda")
    idx, w = MO.router_topk(logits, 512, 10)
    rw, ri = router_topk(logits[:, :512], 10)
    assert torch.equal(idx.long(), ri) and torch.allclose(w, rw, atol=1e-6)


def test_moe_forward_matches_torch():
    ref, dut = _pair(MOE)
    ids = torch.randint(0, MOE.vocab, (333,), generator=torch.Generator().manual_seed(1)).cuda()
    keep = torch.arange(300, 333, device="cuda")
    lr, _ = ref.forward_exact(ids, keep=keep)
    ld, _ = dut.forward_exact(ids, keep=keep)
    l32, _ = _fp32(MOE).forward_exact(ids, keep=keep)
    assert _rel(ld, l32) < 1.5 * _rel(lr, l32) + 5e-3, (_rel(ld, l32), _rel(lr, l32))


@pytest.mark.parametrize("cfg", [HYB, LLAMA, QWEN3], ids=lambda c: c.name)
def test_exact_rows_layer_rows_matches_fp32(cfg):
    """layer_rows on the kernels (K/V of every row, queries of the exact rows at their positions on the tcgen05
    attention, GDN over every row) against the fp32 oracle's layer_rows, one late layer at a time."""
    dut, f32 = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200"), _fp32(cfg)
    n = 300
    g = torch.Generator(device="cuda").manual_seed(7)
    h = torch.randn(n, cfg.hidden, device="cuda", generator=g)
    pos = torch.arange(n, device="cuda")
    rows = torch.tensor(sorted({3, 17, 64, 65, 130, 200, 257, 299}), device="cuda")
    for i in range(cfg.n_layers):
        cd, cf = dut.new_cache(), f32.new_cache()
        yd = dut.layer_rows(i, h.bfloat16(), pos, rows, cd)
        yf = f32.layer_rows(i, h, pos, rows, cf)
        assert yd.shape == yf.shape == (rows.numel(), cfg.hidden)
        assert _rel(yd, yf) < 3e-2, (i, _rel(yd, yf))
        if cfg.layer_types[i] == "attn":
            assert _rel(cd[i]["k"], cf[i]["k"]) < 3e-2 and _rel(cd[i]["v"], cf[i]["v"]) < 3e-2
        else:
            assert _rel(cd[i]["rec"], cf[i]["rec"]) < 5e-2
        # the selected rows' outputs equal the whole layer's outputs at those rows
        cl = dut.new_cache()
        full = dut.layer(i, h.bfloat16(), pos, cl)[rows]
        assert _rel(yd, full) < 2e-2, (i, _rel(yd, full))


@pytest.mark.parametrize("cfg", [HYB, LLAMA], ids=lambda c: c.name)
def test_exact_rows_finish_matches_fp32(cfg):
    """A bypass arm (ridge fill plus exact prefix rows) through finish() on the kernels against fp32."""
    split = cfg.n_layers // 2
    g = torch.Generator(device="cuda").manual_seed(3)
    d = cfg.hidden
    W = {i: (torch.eye(d, device="cuda") + 0.01 * torch.randn(d, d, device="cuda", generator=g)).bfloat16()
         for i in range(split, cfg.n_layers)}
    B = {i: (0.01 * torch.randn(d, device="cuda", generator=g)).bfloat16() for i in range(split, cfg.n_layers)}
    arm = Arm("bypass", split=split, tail=100, fill="proj", projector=Projector(split, W, B))
    ids = torch.randint(0, cfg.vocab, (400,), generator=torch.Generator().manual_seed(2)).cuda()
    rows = [5, 6, 40, 128, 129, 250, 299]
    ref, dut = _pair(cfg)
    out = {}
    for name, m in (("ref", ref), ("dut", dut), ("f32", _fp32(cfg))):
        hs, lower = run_lower(m, ids, [split])
        out[name] = finish(m, ids, hs[split], lower, arm, 4, exact_rows=rows)
    e_dut, e_ref = _rel(out["dut"][0], out["f32"][0]), _rel(out["ref"][0], out["f32"][0])
    assert e_dut < 1.5 * e_ref + 5e-3, (e_dut, e_ref)
    # the exact rows change the answer: without them the logits differ
    hs, lower = run_lower(dut, ids, [split])
    plain = finish(dut, ids, hs[split], lower, arm, 4)[0]
    assert _rel(plain, out["dut"][0]) > 0


@pytest.mark.parametrize("slots", [1, 3])
def test_streamed_maps_equal_resident_maps(slots):
    """Maps streamed from pinned host memory through a ring of device slots (copies on a side stream, ordered by
    events) give bitwise the fill of resident maps, through the batched fill and the per-layer path."""
    from ridgefill_data_b200.ridge.projector import StreamedProjector
    cfg = HYB
    dut = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    split = cfg.n_layers // 2
    g = torch.Generator(device="cuda").manual_seed(3)
    d = cfg.hidden
    W = {i: (torch.eye(d, device="cuda") + 0.01 * torch.randn(d, d, device="cuda", generator=g)).bfloat16()
         for i in range(split, cfg.n_layers)}
    B = {i: (0.01 * torch.randn(d, device="cuda", generator=g)).bfloat16() for i in range(split, cfg.n_layers)}
    ids = torch.randint(0, cfg.vocab, (400,), generator=torch.Generator().manual_seed(2)).cuda()
    res = Arm("ridgefill", split=split, tail=100, fill="proj", projector=Projector(split, W, B))
    sp = StreamedProjector(split, W, B, slots=slots)
    stream = Arm("ridgefill", split=split, tail=100, fill="proj", projector=sp)
    for rows in (None, [3, 50, 200]):            # batched fill; per-layer path with exact rows
        out = {}
        for name, arm in (("res", res), ("str", stream)):
            hs, lower = run_lower(dut, ids, [split], maps=arm.projector)
            out[name] = finish(dut, ids, hs[split], lower, arm, 4, exact_rows=rows)[0]
        assert torch.equal(out["res"], out["str"]), rows
    assert sp.resident_bytes() == min(slots, cfg.n_layers - split) * (d * d + d) * 2


def test_gdn_state_checkpoints_match_fp32():
    """GDN recurrent-state checkpoints on the kernels (exact layers and cache-only fills) against the fp32 oracle:
    the same absolute positions, the same states within bf16 tolerance."""
    ref, dut = _pair(HYB)
    f32 = _fp32(HYB)
    ids = torch.randint(0, HYB.vocab, (333,), generator=torch.Generator().manual_seed(5)).cuda()
    _, cd = dut.forward_exact(ids, gdn_checkpoint_every=128)
    _, cr = ref.forward_exact(ids, gdn_checkpoint_every=128)
    _, cf = f32.forward_exact(ids, gdn_checkpoint_every=128)
    for i, t in enumerate(HYB.layer_types):
        if t != "gdn":
            continue
        kd, kf = cd[i]["checkpoints"], cf[i]["checkpoints"]
        assert sorted(kd) == sorted(kf) == sorted(cr[i]["checkpoints"]) == [128, 256]
        for p in kf:   # no further from fp32 than the torch bf16 path (errors grow with depth for both)
            e_dut, e_ref = _rel(kd[p], kf[p]), _rel(cr[i]["checkpoints"][p], kf[p])
            assert e_dut < 1.5 * e_ref + 2e-2, (i, p, e_dut, e_ref)
        e_dut, e_ref = _rel(cd[i]["rec"], cf[i]["rec"]), _rel(cr[i]["rec"], cf[i]["rec"])
        assert e_dut < 1.5 * e_ref + 2e-2, (i, e_dut, e_ref)
    # a fill with checkpoints
    g = torch.Generator(device="cuda").manual_seed(9)
    x = torch.randn(300, HYB.hidden, device="cuda", generator=g)
    pos = torch.arange(300, device="cuda")
    i = HYB.layer_types.index("gdn")
    c1, c2 = dut.new_cache(), f32.new_cache()
    k1 = dut.fill(i, x.bfloat16(), pos, c1, checkpoint_every=64)
    k2 = f32.fill(i, x, pos, c2, checkpoint_every=64)
    assert sorted(k1) == sorted(k2) == [64, 128, 192, 256]
    assert all(_rel(k1[p], k2[p]) < 5e-2 for p in k2)
