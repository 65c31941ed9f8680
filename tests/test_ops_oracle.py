"""Oracle op checks (code/tests/test_ops.py strategy): chunked delta rule vs the recurrent definition
(incl. checkpoints and continuation), causal conv vs F.conv1d, blocked attention vs dense masked softmax."""
import torch
import torch.nn.functional as F

from ridgefill_data_b200.ops import oracle as ops


def _gdn_inputs(h=3, n=150, dk=8, dv=6, seed=0):
    g = torch.Generator().manual_seed(seed)
    q = ops.l2norm(torch.randn(h, n, dk, generator=g)) * dk ** -0.5
    k = ops.l2norm(torch.randn(h, n, dk, generator=g))
    v = torch.randn(h, n, dv, generator=g)
    gg = -F.softplus(torch.randn(h, n, generator=g))
    beta = torch.sigmoid(torch.randn(h, n, generator=g))
    return q, k, v, gg, beta


def test_delta_rule_chunked_matches_recurrent():
    q, k, v, g, b = _gdn_inputs()
    o1, s1, _ = ops.delta_rule(q, k, v, g, b, chunk=16)
    o2, s2 = ops.delta_rule_recurrent(q, k, v, g, b)
    assert torch.allclose(o1, o2, atol=1e-5) and torch.allclose(s1, s2, atol=1e-5)


def test_delta_rule_continuation_and_checkpoints():
    q, k, v, g, b = _gdn_inputs(n=128)
    o_full, s_full, ck = ops.delta_rule(q, k, v, g, b, chunk=16, checkpoint_every=32)
    assert sorted(ck) == [32, 64, 96, 128]
    _, s_half, _ = ops.delta_rule(q[:, :64], k[:, :64], v[:, :64], g[:, :64], b[:, :64], chunk=16)
    assert torch.allclose(ck[64], s_half, atol=1e-5)
    o2, s2, _ = ops.delta_rule(q[:, 64:], k[:, 64:], v[:, 64:], g[:, 64:], b[:, 64:], s_half, chunk=16)
    assert torch.allclose(o2, o_full[:, 64:], atol=1e-5) and torch.allclose(s2, s_full, atol=1e-5)
    _, s_fill, _ = ops.delta_rule(q, k, v, g, b, chunk=16, need_out=False)
    assert torch.allclose(s_fill, s_full)


def test_causal_conv_matches_conv1d_and_continues():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(40, 12, generator=g)
    w = torch.randn(12, 4, generator=g)
    out, st = ops.causal_conv(x, None, w)
    ref = F.silu(F.conv1d(F.pad(x.T[None], (3, 0)), w[:, None, :], groups=12))[0].T
    assert torch.allclose(out, ref, atol=1e-5)
    o1, s1 = ops.causal_conv(x[:17], None, w)
    o2, _ = ops.causal_conv(x[17:], s1, w)
    assert torch.allclose(torch.cat((o1, o2)), out, atol=1e-6)
    assert torch.allclose(st, x[-3:])


def _dense_attention(q, k, v, scale, qpos):
    hq, nq, d = q.shape
    rep = hq // k.shape[0]
    kk = k.repeat_interleave(rep, 0).float()
    vv = v.repeat_interleave(rep, 0).float()
    s = q.float() @ kk.transpose(1, 2) * scale
    s = s.masked_fill(torch.arange(k.shape[1])[None, None, :] > qpos[None, :, None], float("-inf"))
    return (torch.softmax(s, -1) @ vv).transpose(0, 1).reshape(nq, -1)


def test_blocked_attention_matches_dense(monkeypatch):
    g = torch.Generator().manual_seed(2)
    q = torch.randn(4, 50, 16, generator=g)
    k = torch.randn(2, 80, 16, generator=g)
    v = torch.randn(2, 80, 16, generator=g)
    ref = _dense_attention(q, k, v, 0.25, torch.arange(30, 80))
    assert torch.allclose(ops.attend(q, k, v, 0.25), ref, atol=1e-5)
    monkeypatch.setattr(ops, "ATTN_BLOCK_SCORES", 4 * 80 * 16)   # force 16-query blocks
    assert torch.allclose(ops.attend(q, k, v, 0.25), ref, atol=1e-5)
    qpos = torch.tensor([0, 3, 9, 10, 40, 79])
    ref2 = _dense_attention(q[:, :6], k, v, 0.25, qpos)
    assert torch.allclose(ops.attend_at(q[:, :6], k, v, 0.25, qpos), ref2, atol=1e-5)


def test_router_topk_renormalised():
    logits = torch.randn(7, 16)
    w, idx = ops.router_topk(logits, 4)
    assert torch.allclose(w.sum(-1), torch.ones(7))
    assert (idx == torch.topk(logits, 4).indices).all()
