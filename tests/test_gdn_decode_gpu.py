"""The batched GDN decode step (csrc/gdn_decode.cu) against the token-by-token oracle (ops/oracle.py: causal_conv,
l2norm, delta_rule_recurrent, the gates of models/hybrid.py), in place against out of place, and batched against
one sequence at a time, including a batch past the kernel's per-launch sequence count."""
import pytest
import torch

from ridgefill_data_b200.ops import oracle

pytestmark = pytest.mark.gpu

NK, NV, DK, DV, KC = 2, 6, 128, 128, 4
C = 2 * NK * DK + NV * DV


def _inputs(R, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    rnd = lambda *s, scale=1.0: torch.randn(*s, device="cuda", generator=g) * scale   # noqa: E731
    width = C + 2 * NV + NV * DV                                  # q|k|v, b, a, z (z unused here)
    proj = rnd(R, width).bfloat16()
    conv_w = rnd(C, KC, scale=0.5).bfloat16()
    A_log = rnd(NV, scale=0.5)
    dt_bias = rnd(NV, scale=0.5)
    conv = [rnd(KC - 1, C).bfloat16() for _ in range(R)]
    rec = [rnd(NV, DK, DV, scale=0.1) for _ in range(R)]
    return proj, conv_w, A_log, dt_bias, conv, rec


def _oracle(proj, conv_w, A_log, dt_bias, conv, rec):
    """Per sequence: the oracle's conv + SiLU (bf16 out), l2norm (q times dk^-0.5) rounded to bf16 like the kernels'
    q / k, sigmoid gate rounded to bf16, then one recurrent delta-rule step in fp32."""
    outs, recs, convs = [], [], []
    rep = NV // NK
    for r in range(proj.shape[0]):
        y, new_conv = oracle.causal_conv(proj[r:r + 1, :C], conv[r], conv_w)
        q, k, v = y.split([NK * DK, NK * DK, NV * DV], -1)
        q = (oracle.l2norm(q.float().view(NK, DK)) * DK ** -0.5).bfloat16().float().repeat_interleave(rep, 0)
        k = oracle.l2norm(k.float().view(NK, DK)).bfloat16().float().repeat_interleave(rep, 0)
        v = v.float().view(NV, DV)
        b = proj[r, C:C + NV].float()
        a = proj[r, C + NV:C + 2 * NV].float()
        beta = torch.sigmoid(b).bfloat16().float()
        gdec = -A_log.exp() * torch.nn.functional.softplus(a + dt_bias)
        o, S = oracle.delta_rule_recurrent(q[:, None], k[:, None], v[:, None], gdec[:, None], beta[:, None],
                                           rec[r].clone())
        outs.append(o[:, 0].reshape(-1))
        recs.append(S)
        convs.append(new_conv)
    return torch.stack(outs), recs, convs


def _run(proj, conv_w, A_log, dt_bias, conv, rec, in_place):
    from ridgefill_data_b200.ops import kernels as K
    R = proj.shape[0]
    out = torch.empty(R, NV * DV, dtype=torch.bfloat16, device="cuda")
    conv_s = [c.clone() for c in conv]
    rec_s = [s.clone() for s in rec]
    conv_d = conv_s if in_place else [torch.empty_like(c) for c in conv_s]
    rec_d = rec_s if in_place else [torch.empty_like(s) for s in rec_s]
    K.gdn_decode_step(proj, conv_w, A_log, dt_bias, conv_s, conv_d, rec_s, rec_d, out, NK, NV, DK, DV, C, C + NV)
    return out, rec_d, conv_d


def test_decode_step_matches_recurrent_oracle():
    from ridgefill_data_b200.ops._ext import check_errors
    args = _inputs(3, seed=1)
    out, rec, conv = _run(*args, in_place=False)
    torch.cuda.synchronize()
    check_errors()
    ref_out, ref_rec, ref_conv = _oracle(*args)
    err = (out.float() - ref_out).abs().max().item() / ref_out.abs().max().item()
    assert err < 1e-2, err
    for a, b in zip(rec, ref_rec):
        assert (a - b).abs().max().item() / b.abs().max().item() < 5e-3
    for a, b in zip(conv, ref_conv):
        assert torch.equal(a, b)


def test_in_place_equals_out_of_place_and_batch_equals_single():
    args = _inputs(20, seed=2)                       # 20 sequences: two launches of the kernel pair
    proj, conv_w, A_log, dt_bias, conv, rec = args
    out_a, rec_a, conv_a = _run(*args, in_place=False)
    out_b, rec_b, conv_b = _run(*args, in_place=True)
    assert torch.equal(out_a, out_b)
    assert all(torch.equal(x, y) for x, y in zip(rec_a, rec_b))
    assert all(torch.equal(x, y) for x, y in zip(conv_a, conv_b))
    for r in (0, 7, 19):
        o1, r1, c1 = _run(proj[r:r + 1], conv_w, A_log, dt_bias, conv[r:r + 1], rec[r:r + 1], in_place=False)
        assert torch.equal(o1[0], out_a[r]) and torch.equal(r1[0], rec_a[r]) and torch.equal(c1[0], conv_a[r])
