"""Fill impact and the weighted fit on tiny checkpoints (CPU, fp32): the differentiable tail path against the
inference path, the first-order impact against a finite difference of the loss, the lookup statistics
against dense formulas, and the row weights."""
import math

import pytest
import torch

from ridgefill_data_b200.engine import impact as IM
from ridgefill_data_b200.engine.prefill import run_lower
from ridgefill_data_b200.eval.data import zipf_docs
from ridgefill_data_b200.models.base import load
from ridgefill_data_b200.ops import oracle as ops
from ridgefill_data_b200.ridge import wfit
from ridgefill_data_b200.ridge.fit import EigenFit


def _dense_attn(q, k, v, scale):
    hq, nq, d = q.shape
    hkv, nk, _ = k.shape
    rep = hq // hkv
    kk, vv = k.repeat_interleave(rep, 0), v.repeat_interleave(rep, 0)
    s = (q @ kk.transpose(1, 2)) * scale
    qpos = torch.arange(nk - nq, nk)
    s = s.masked_fill(torch.arange(nk)[None, :] > qpos[:, None], -math.inf)
    return (torch.softmax(s, -1) @ vv).transpose(0, 1).reshape(nq, -1)


def test_attention_backward_matches_autograd():
    g = torch.Generator().manual_seed(0)
    q = torch.randn(4, 7, 8, generator=g, requires_grad=True)
    k = torch.randn(2, 19, 8, generator=g, requires_grad=True)
    v = torch.randn(2, 19, 8, generator=g, requires_grad=True)
    w = torch.randn(7, 32, generator=g)
    (IM.CausalAttention.apply(q, k, v, 0.3) * w).sum().backward()
    got = [t.grad.clone() for t in (q, k, v)]
    for t in (q, k, v):
        t.grad = None
    (_dense_attn(q, k, v, 0.3) * w).sum().backward()
    for a, t in zip(got, (q, k, v)):
        torch.testing.assert_close(a, t.grad, rtol=1e-4, atol=1e-5)


def test_delta_rule_diff_matches_recurrence_and_gradients():
    g = torch.Generator().manual_seed(1)
    h, n, dk, dv = 2, 70, 8, 6
    q = ops.l2norm(torch.randn(h, n, dk, generator=g)) * dk ** -0.5
    k = ops.l2norm(torch.randn(h, n, dk, generator=g))
    v = torch.randn(h, n, dv, generator=g, requires_grad=True)
    beta = torch.rand(h, n, generator=g)
    lg = -torch.rand(h, n, generator=g) * 0.2
    s0 = torch.randn(h, dk, dv, generator=g) * 0.1
    out = IM.delta_rule_diff(q, k, v, lg, beta, s0, chunk=16)
    ref, _ = ops.delta_rule_recurrent(q, k, v, lg, beta, s0)
    torch.testing.assert_close(out, ref, rtol=1e-4, atol=1e-5)
    wt = torch.randn_like(out)
    (out * wt).sum().backward()
    gv = v.grad.clone()
    v.grad = None
    ref, _ = ops.delta_rule_recurrent(q, k, v, lg, beta, s0)
    (ref * wt).sum().backward()
    torch.testing.assert_close(gv, v.grad, rtol=1e-4, atol=1e-5)


@pytest.fixture(scope="module", params=["tiny_llama", "tiny_qwen35"])
def model(request):
    path, _ = request.getfixturevalue(request.param)
    return load(path, dtype=torch.float32)


def _setup(model, n=48, P=32, split=2):
    ids = torch.randint(0, 300, (n,), generator=torch.Generator().manual_seed(5))
    hs, _ = run_lower(model, ids, [split])
    h = hs[split]
    rows = torch.arange(n - P - 1)                       # tail rows whose next token is scored
    tgt = ids[P + 1:]
    return ids, h, rows, tgt


def test_tail_loss_at_exact_caches_is_exact_loss(model):
    split, P = 2, 32
    ids, h, rows, tgt = _setup(model)
    late_in = {}
    true, loss = IM.exact_late(model, h, split, P, rows + P, tgt, hook=lambda i, x: late_in.__setitem__(i, x[:P]))
    kv, gdn = IM.fill_late(model, split, P, lambda i: late_in[i])
    for i in kv:
        torch.testing.assert_close(kv[i][0], true[i][0])
    with torch.no_grad():
        got = IM.tail_loss(model, split, h[P:], torch.arange(P, h.shape[0]), kv, gdn, rows, tgt)
    assert abs(float(got) - loss) < 1e-4


def test_impact_is_the_directional_derivative(model):
    split, P = 2, 32
    ids, h, rows, tgt = _setup(model)
    true, _ = IM.exact_late(model, h, split, P, rows + P, tgt)
    kv, gdn = IM.fill_late(model, split, P, lambda i: h[:P])          # identity fill
    res, loss0 = IM.impact(model, split, h[P:], P, kv, true, gdn, rows, tgt)
    assert res["impact"].shape == (P,) and torch.isfinite(res["impact"]).all()
    assert (res["err"] >= 0).all() and (res["grad_norm"] >= 0).all()
    eps = 1e-3
    moved = {i: (k + eps * (true[i][0] - k), v + eps * (true[i][1] - v)) for i, (k, v) in kv.items()}
    pos = torch.arange(P, h.shape[0])
    with torch.no_grad():
        l_eps = float(IM.tail_loss(model, split, h[P:], pos, moved, gdn, rows, tgt))
    fd = (l_eps - loss0) / eps
    assert abs(fd - float(res["impact"].sum())) < 2e-2 * max(1.0, abs(fd))


def test_received_mass_and_row_stats_match_dense():
    g = torch.Generator().manual_seed(2)
    hq, hkv, n, d = 4, 2, 40, 8
    q, k = torch.randn(hq, n, d, generator=g), torch.randn(hkv, n, d, generator=g)
    scale = d ** -0.5
    s = (q @ k.repeat_interleave(2, 0).transpose(1, 2)) * scale
    mask = torch.ones(n, n, dtype=torch.bool).tril()
    p = torch.softmax(s.masked_fill(~mask, -math.inf), -1)                      # [hq, n, n]
    off = p * (~torch.eye(n, dtype=torch.bool))
    tot, low, ent = IM.received_mass(q, k, scale, rows_below=25, entropy=True)
    torch.testing.assert_close(tot, off.sum((0, 1)).double(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(low, off[:, :25].sum((0, 1)).double(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(ent, torch.special.entr(p).sum((0, 2)).double(), rtol=1e-5, atol=1e-6)
    strided = IM.received_mass(q, k, scale, stride=2)
    torch.testing.assert_close(strided, 2 * off[:, ::2].sum((0, 1)).double(), rtol=1e-5, atol=1e-6)
    e, sink, near = IM.row_stats(q, k, scale, local=4)
    torch.testing.assert_close(sink, p[..., 0].mean(0).double(), rtol=1e-5, atol=1e-6)
    recent = (torch.arange(n)[:, None] - torch.arange(n)[None, :] < 4) & mask
    torch.testing.assert_close(near, (p * recent).sum(-1).mean(0).double(), rtol=1e-5, atol=1e-6)
    torch.testing.assert_close(e, torch.special.entr(p).sum(-1).mean(0).double(), rtol=1e-5, atol=1e-6)


def test_row_features():
    dist, first, bigram = IM.repetition([5, 6, 5, 6, 7], cap=100)
    assert first == [1.0, 1.0, 0.0, 0.0, 1.0]
    assert bigram == [0.0, 0.0, 0.0, 1.0, 0.0]
    assert dist[2] == pytest.approx(math.log(2)) and dist[0] == pytest.approx(math.log(100))
    x = torch.randn(10, 6)
    torch.testing.assert_close(IM.row_norm(x), x.norm(dim=-1).double())
    torch.testing.assert_close(IM.velocity(x, 2 * x), torch.full((10,), 0.5, dtype=torch.float64))
    torch.testing.assert_close(IM.log_max_act(x), x.abs().amax(-1).log().double())


def test_rank_fraction_and_row_weights():
    r = wfit.rank_fraction(torch.tensor([3.0, 1.0, 3.0, 2.0]))
    torch.testing.assert_close(r, torch.tensor([2.5, 0.0, 2.5, 1.0], dtype=torch.float64) / 4)
    qfp = torch.tensor([100.0, 1.0, 2.0, 3.0, 4.0])
    for shape in wfit.SHAPES:
        w = wfit.row_weights(qfp, shape)
        assert w[0] == 1.0 and w[1:].mean().item() == pytest.approx(1.0)
        assert (w[1:].diff() >= 0).all()
    with pytest.raises(ValueError):
        wfit.row_weights(qfp, "bogus")


def test_weighted_capture_and_leverage(model):
    docs = zipf_docs(3, 40, 300, seed=4)
    st = wfit.capture_weighted(model, docs, 2, shape="rank", log=None).state()
    assert st["n"] == pytest.approx(sum(len(d["ids"]) for d in docs), rel=1e-6)   # weights have mean 1 per doc
    maps = EigenFit(st).layer(3, [0.01])[0.01]
    assert torch.isfinite(maps[0]).all()
    mean, L = IM.leverage_map(st, 0.01)
    x = torch.randn(5, model.hidden)
    lev = IM.log_leverage(x, mean, L)
    assert lev.shape == (5,) and torch.isfinite(lev).all()


def test_impact_is_bounded_by_error_times_sensitivity(model):
    """The ImpactBound statements (code/lean/kva_lean/KvaLean/ImpactBound.lean) on this framework's impact: per row
    |impact_j| <= |g_j| |delta_j| (Cauchy-Schwarz); with rows S kept exact, |sum over the others| <= e sum_{j not in S}
    |g_j| for e the largest error; and the S holding the largest gradient norms leaves the smallest outside mass."""
    split, P = 2, 32
    ids, h, rows, tgt = _setup(model)
    true, _ = IM.exact_late(model, h, split, P, rows + P, tgt)
    kv, gdn = IM.fill_late(model, split, P, lambda i: h[:P])
    res, _ = IM.impact(model, split, h[P:], P, kv, true, gdn, rows, tgt)
    d2 = torch.zeros(P, dtype=torch.float64)
    for i, (k, v) in kv.items():
        for fill, exact in ((k, true[i][0]), (v, true[i][1])):
            d2 += (exact.float() - fill.float()).square().sum((0, 2)).double()
    delta, g, imp = d2.sqrt(), res["grad_norm"].double(), res["impact"].double()
    assert (imp.abs() <= g * delta * (1 + 1e-5) + 1e-9).all()
    e = float(delta.max())
    gen = torch.Generator().manual_seed(3)
    for m in (0, 4, 16):
        top = set(torch.topk(g, m).indices.tolist()) if m else set()
        outside = [j for j in range(P) if j not in top]
        assert abs(float(imp[outside].sum())) <= e * float(g[outside].sum()) * (1 + 1e-5) + 1e-9
        for _ in range(20):                              # no other set of m rows leaves less sensitivity outside
            other = set(torch.randperm(P, generator=gen)[:m].tolist())
            rest = [j for j in range(P) if j not in other]
            assert float(g[outside].sum()) <= float(g[rest].sum()) + 1e-12
