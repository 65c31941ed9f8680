"""Native checks on the GPU: the standalone identity-fill program (no Python inside) and the device scorer
(log-sum-exp, argmax, target log-probs, KL) against an fp64 torch reference; the fill debug tap through a
B200 prefill (identity fill bitwise, ridge maps within bf16 rounding)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_identity_check_program():
    from ridgefill_data_b200.native import build_native, run
    build_native(["identity_check"])
    code, out = run("identity_check", 777, 1024)
    assert code == 0, out
    assert '"mismatches": 0' in out


def test_score_rows_matches_fp64():
    from ridgefill_data_b200.ops.kernels import score_rows
    g = torch.Generator(device="cuda").manual_seed(0)
    rows, V = 7, 248320
    x = torch.randn(rows, V, device="cuda", generator=g) * 3
    q = x + 0.3 * torch.randn(rows, V, device="cuda", generator=g)
    x[2, 17] = x[2].max() + 1          # a clear argmax
    x[3, 5] = x[3, 9] = x[3].max() + 2  # a tie: the lower index wins
    t = torch.randint(0, V, (rows,), device="cuda", generator=g)
    out = score_rows(x, targets=t, ref=q)
    lp = torch.log_softmax(x.double(), -1)
    lq = torch.log_softmax(q.double(), -1)
    torch.testing.assert_close(out["lse"], torch.logsumexp(x.double(), -1), rtol=0, atol=1e-9)
    torch.testing.assert_close(out["logprob"], lp.gather(1, t[:, None])[:, 0], rtol=0, atol=1e-9)
    torch.testing.assert_close(out["kl"], (lq.exp() * (lq - lp)).sum(-1), rtol=1e-9, atol=1e-10)
    assert out["argmax"][2].item() == 17 and out["argmax"][3].item() == 5
    assert torch.equal(out["ref_argmax"].long(), q.argmax(-1))


def test_fill_tap_identity_and_maps():
    from ridgefill_data_b200.engine.arm import Arm
    from ridgefill_data_b200.engine.prefill import prefill, run_lower
    from ridgefill_data_b200.engine.taps import FillTap, attached
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.config import PRESETS
    from ridgefill_data_b200.ridge.projector import Projector
    cfg = PRESETS["qwen3.8-27b"].replace(n_layers=8, layer_types=["gdn", "gdn", "gdn", "attn"] * 2, vocab=4096)
    m = from_config(cfg, backend="b200", device="cuda")
    ids = torch.randint(0, cfg.vocab, (1024,), generator=torch.Generator().manual_seed(1))
    split = 4
    hs, _ = run_lower(m, ids, [split])
    tap = FillTap(rows=112)
    with attached(m, tap):
        prefill(m, ids, Arm("id", split=split, tail=512, fill="identity"), keep=1)
    assert sorted(tap.got) == list(range(split, 8))
    assert all(v == 0 for v in tap.check_identity(hs[split]).values())
    gen = torch.Generator().manual_seed(2)
    d = cfg.hidden
    W = {i: (torch.eye(d) + 0.01 * torch.randn(d, d, generator=gen)).bfloat16() for i in range(split, 8)}
    B = {i: (0.01 * torch.randn(d, generator=gen)).bfloat16() for i in range(split, 8)}
    proj = Projector(split, W, B)
    tap = FillTap(rows=112)
    with attached(m, tap):
        prefill(m, ids, Arm("rf", split=split, tail=512, fill="proj", projector=proj), keep=1)
    assert max(tap.check_maps(hs[split], proj).values()) < 2e-2


def test_row_cosine_matches_torch():
    from ridgefill_data_b200.ops.kernels import row_cosine
    g = torch.Generator(device="cuda").manual_seed(3)
    a = torch.randn(1000, 4, 128, device="cuda", generator=g).bfloat16()
    b = (a.float() + 0.5 * torch.randn(1000, 4, 128, device="cuda", generator=g)).bfloat16()
    got = row_cosine(a, b)
    want = torch.nn.functional.cosine_similarity(a.float(), b.float(), dim=-1)
    torch.testing.assert_close(got, want, rtol=1e-4, atol=1e-5)


@pytest.mark.parametrize("hq,hkv,hd,n,w", [(8, 2, 128, 1000, 64), (24, 4, 256, 777, 64), (4, 4, 64, 130, 17)])
def test_window_mass_matches_softmax_column_sums(hq, hkv, hd, n, w):
    from ridgefill_data_b200.ops.kernels import window_mass
    g = torch.Generator(device="cuda").manual_seed(4)
    q = torch.randn(hq, w, hd, device="cuda", generator=g).bfloat16()
    kbuf = torch.randn(hkv, n + 37, hd, device="cuda", generator=g).bfloat16()    # cache buffer with spare rows
    k = kbuf[:, :n]
    qpos = torch.arange(n - w, n, device="cuda")
    scale = hd ** -0.5
    got = window_mass(q, k, qpos, scale)
    rep = hq // hkv
    s = (q.float() @ k.float().repeat_interleave(rep, 0).transpose(1, 2)) * scale
    s = s.masked_fill(torch.arange(n, device="cuda")[None, :] > qpos[:, None], float("-inf"))
    want = torch.softmax(s, -1).sum((0, 1)).double()
    torch.testing.assert_close(got, want, rtol=2e-3, atol=2e-4)


def test_embedding_gather_reports_bad_ids():
    from ridgefill_data_b200.ops import kernels as K
    from ridgefill_data_b200.ops._ext import check_errors
    table = torch.randn(50, 64, device="cuda").bfloat16()
    out = K.embed(table, torch.tensor([3, 7], device="cuda"))
    torch.testing.assert_close(out, table[[3, 7]])
    check_errors()
    bad = K.embed(table, torch.tensor([3, 99], device="cuda"))
    torch.cuda.synchronize()
    assert torch.equal(bad[1], torch.zeros_like(bad[1]))
    with pytest.raises(RuntimeError, match="gather index"):
        check_errors()


@pytest.mark.parametrize("what", ["gemm", "attention", "gdn"])
def test_kernels_are_deterministic(what):
    """Run twice, bitwise equal (the determinism the reference's bitwise canaries rely on)."""
    from ridgefill_data_b200.eval.checks import rerun_bitwise
    from ridgefill_data_b200.ops import gemm as G
    from ridgefill_data_b200.ops import kernels as K
    g = torch.Generator(device="cuda").manual_seed(9)
    if what == "gemm":
        x = torch.randn(1000, 512, device="cuda", generator=g).bfloat16()
        w = torch.randn(768, 512, device="cuda", generator=g).bfloat16()
        fn = lambda: G.linear(x, w)  # noqa: E731
    elif what == "attention":
        q = torch.randn(8, 300, 128, device="cuda", generator=g).bfloat16()
        k = torch.randn(2, 300, 128, device="cuda", generator=g).bfloat16()
        v = torch.randn_like(k)

        def fn():
            out = torch.empty(300, 8 * 128, device="cuda", dtype=torch.bfloat16)
            K.attention(q, k, v, 300, 128 ** -0.5, out)
            return out
    else:
        n, nk, nv = 700, 1, 2
        C = 2 * nk * 128 + nv * 128
        proj = (torch.randn(n, C + 2 * nv, device="cuda", generator=g) * 0.5).bfloat16()
        conv_w = (torch.randn(C, 4, device="cuda", generator=g) / 2).bfloat16()
        q, kk, v, beta, gg = K.gdn_prep(proj, C, C + nv, conv_w, None, torch.rand(nv, device="cuda"),
                                        torch.zeros(nv, device="cuda"), nk, nv, 128, 128)

        def fn():
            st = torch.zeros(nv, 128, 128, device="cuda")
            out = torch.empty(n, nv * 128, device="cuda", dtype=torch.bfloat16)
            K.gdn_scan(q, kk, v, beta, gg, st, out, groups=3)
            return torch.cat((out.float().flatten(), st.flatten()))
    same, _ = rerun_bitwise(fn)
    assert same
