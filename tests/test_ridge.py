"""Ridge statistics and fits: shifted sums vs naive sums, eigen vs Cholesky vs a direct solve,
residual/combine identities, the plain (uncentred) form, map file format."""
import pytest
import torch

from ridgefill_data_b200.ridge import fit as rfit
from ridgefill_data_b200.ridge import projector as rp
from ridgefill_data_b200.ridge.stats import RidgeStats, combine, raw_moments, residual


def _data(n=300, d=12, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(n, d, generator=g) * 2 + 5
    ys = {i: x @ torch.randn(d, d, generator=g) * 0.3 + torch.randn(n, d, generator=g) * 0.1 + i
          for i in (3, 4)}
    return x, ys


def test_stats_match_naive_sums():
    x, ys = _data()
    st = RidgeStats(3, [3, 4], 12)
    st.add(x[:100], {i: y[:100] for i, y in ys.items()}, block=64)
    st.add(x[100:], {i: y[100:] for i, y in ys.items()}, block=64)
    s = st.state()
    xx, xy = raw_moments(s, 4)
    assert torch.allclose(xx, x.double().T @ x.double(), rtol=1e-5)
    assert torch.allclose(xy, x.double().T @ ys[4].double(), rtol=1e-5)


def test_eigen_matches_cholesky_and_direct():
    x, ys = _data()
    st = RidgeStats(3, [3, 4], 12)
    st.add(x, ys)
    s = st.state()
    lam = 0.03
    e = rfit.EigenFit(s).layer(4, [lam])[lam]
    c = rfit.CholeskyFit(s).layer(4, [lam])[lam]
    xd, yd = x.double(), ys[4].double()
    xc, yc = xd - xd.mean(0), yd - yd.mean(0)
    cxx = xc.T @ xc
    w = torch.linalg.solve(cxx + lam * cxx.diagonal().mean() * torch.eye(12, dtype=torch.float64), xc.T @ yc)
    b = yd.mean(0) - xd.mean(0) @ w
    for got in (e, c):
        assert torch.allclose(got[0].double(), w.T, atol=1e-4)
        assert torch.allclose(got[1].double(), b, atol=1e-3)


def test_plain_form_uncentred():
    x, ys = _data()
    st = RidgeStats(3, [3, 4], 12)
    st.add(x, ys)
    s = st.state()
    xd, yd = x.double(), ys[3].double()
    xtx = xd.T @ xd
    lam = 1e-2
    w = torch.linalg.solve(xtx + lam * xtx.trace() / 12 * torch.eye(12, dtype=torch.float64), xd.T @ yd)
    for cls in (rfit.EigenFit, rfit.CholeskyFit):
        got_w, got_b = cls(s, center=False).layer(3, [lam])[lam]
        assert torch.allclose(got_w.double(), w.T, atol=1e-4) and float(got_b.abs().max()) == 0.0


def test_residual_and_combine():
    x, ys = _data()
    a = RidgeStats(3, [3, 4], 12)
    a.add(x[:150], {i: y[:150] for i, y in ys.items()})
    b = RidgeStats(3, [3, 4], 12)
    b.add(x[150:], {i: y[150:] for i, y in ys.items()})
    full = RidgeStats(3, [3, 4], 12)
    full.add(x, ys)
    c = combine(a.state(), b.state(), 1.0)
    for i in (3, 4):
        ref = raw_moments(full.state(), i)[1]
        assert (raw_moments(c, i)[1] - ref).abs().max() < 1e-6 * ref.abs().max()
    r = residual(full.state())
    xy = raw_moments(r, 4)[1]
    ref = x.double().T @ (ys[4] - x).double()
    assert (xy - ref).abs().max() < 1e-6 * ref.abs().max()


def test_projector_roundtrip_and_refusals(tmp_path):
    W = {5: torch.randn(8, 8), 6: torch.randn(8, 8)}
    B = {5: torch.randn(8), 6: torch.randn(8)}
    p = rp.Projector(5, W, B)
    path = tmp_path / "m.safetensors"
    p.save(path, dict(model="t", lam=0.03, rows=10))
    assert rp.meta_of(path)["split"] == "5" and rp.meta_of(path)["rows"] == "10"
    q = rp.Projector.load(path, dtype=torch.float32)
    assert q.split == 5 and torch.allclose(q.W[6], W[6].bfloat16().float())
    bad = rp.Projector(5, {5: torch.full((2, 2), 2e4)}, {5: torch.zeros(2)})
    with pytest.raises(ValueError):
        bad.save(tmp_path / "bad.safetensors", {})
    from ridgefill_data_b200.utils.integrity import IntegrityError
    with pytest.raises(IntegrityError):
        rp.Projector.load(path, sha256="0" * 64)


def test_i8_roundtrip(tmp_path):
    from safetensors.torch import save_file
    w = torch.randn(16, 256) * 0.05
    b = torch.randn(16)
    codes, scale, bias = rp.quant_i8(w, b)
    save_file({"proj.7.codes": codes, "proj.7.scale": scale, "proj.7.bias": bias}, str(tmp_path / "p7.safetensors"))
    p = rp.Projector.load_i8({7: tmp_path / "p7.safetensors"}, split=7, dtype=torch.float32)
    assert (p.W[7] - w).abs().max() < 2e-3


def test_st_roundtrip(tmp_path):
    st = {9: torch.randn(4, 8, 6)}
    rp.save_st(tmp_path / "c.safetensors", st)
    got = rp.load_st(tmp_path / "c.safetensors")
    assert torch.equal(got[9], st[9])


def test_unitrms_and_kvfold_fits(tmp_path):
    """--unitrms / --kvfold: one capture gives the raw control, the unit-RMS-target maps and the K/V fold; the fold
    predicts the late attention layers' pre-RoPE K / V from the unit-RMS boundary state better than chance, and
    the files load back (KVFold with its n_kv / eps)."""
    import torch
    from ridgefill_data_b200.engine.prefill import kv_target
    from ridgefill_data_b200.eval.data import zipf_docs
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.tiny import tiny_configs
    from ridgefill_data_b200.ridge import sweep
    from ridgefill_data_b200.ridge.projector import KVFold, Projector
    cfg = tiny_configs(8, 64)["qwen3.5-9b"]
    model = from_config(cfg, seed=0, device="cpu", dtype=torch.float32)
    docs = zipf_docs(6, 256, 4000, seed=3)
    held = zipf_docs(2, 256, 4000, seed=4)
    res = sweep.fit(model, docs, [4], (1e-3, 1e-1), held=held, out_dir=tmp_path, name="tiny", log=None,
                    unitrms=True, kvfold=True)
    r = res[4]
    assert (tmp_path / "tiny-sweep-s4-rawctl.safetensors").exists()
    assert (tmp_path / "tiny-sweep-s4-unitrms.safetensors").exists()
    assert Projector.load(tmp_path / "tiny-sweep-s4-unitrms.safetensors").meta["target"] == "y / rms(y)"
    fold = KVFold.load(tmp_path / "tiny-kvfold-s4.safetensors")
    assert fold.n_kv == model.n_kv and sorted(fold.W) == [i for i in range(4, 8) if model.layer_types[i] == "attn"]
    got = {}
    ids = torch.as_tensor(held[0]["ids"])
    model.forward_exact(ids, hook=lambda i, h: got.__setitem__(i, h) if i != "final" else None)
    i = sorted(fold.W)[0]
    k, v = fold.kv(i, got[4])
    true = kv_target(model, i, got[i]).unflatten(-1, (2, model.n_kv, -1))
    cos = torch.nn.functional.cosine_similarity(k.float(), true[:, 0].float(), dim=-1).mean()
    assert cos > 0.3 and r["kvfold"]["mean_kv_cos"][str(r["kvfold"]["lambda_star"])] > 0.3
    assert r["unitrms"]["lambda_star"] in (1e-3, 1e-1)


def test_ridge_matches_the_reference():
    """Sufficient statistics (plain and row-weighted), eigen fits for a lambda grid and the reduced-rank fits with
    their energy shares against the reference's kva/ridge.py on the same rows (baseline/_ref)."""
    import sys
    from pathlib import Path
    ref_root = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
    if not (ref_root / "kva" / "ridge.py").exists():
        pytest.skip("baseline/_ref not installed")
    sys.path.insert(0, str(ref_root))
    from kva import ridge as RR
    from ridgefill_data_b200.ridge.fit import EigenFit
    from ridgefill_data_b200.ridge.stats import RidgeStats
    g = torch.Generator().manual_seed(9)
    d = 24
    docs = [torch.randn(n, d, generator=g) for n in (90, 130, 61)]
    maps = {1: torch.randn(d, d, generator=g), 2: torch.randn(d, d, generator=g)}
    for weighted in (False, True):
        ours, ref = RidgeStats(0, [1, 2], d), RR.RidgeStats(0, [1, 2], d, "cpu")
        for x in docs:
            ys = {i: x @ m + 0.1 * torch.randn(x.shape[0], d, generator=g) for i, m in maps.items()}
            w = torch.rand(x.shape[0], generator=g) + 0.5 if weighted else None
            ours.add(x, ys, block=64, w=w)
            ref.add(x, ys, block=64, w=w)
        a, b = ours.state(), ref.state()
        assert a["n"] == pytest.approx(b["n"])
        for k in ("cx", "sx", "sxx"):
            torch.testing.assert_close(a[k], b[k], rtol=1e-9, atol=1e-7)
        for k in ("cy", "sy", "sxy"):
            for i in (1, 2):
                torch.testing.assert_close(a[k][i], b[k][i], rtol=1e-9, atol=1e-7)
        lams = [1e-4, 1e-2, 1.0]
        fo, fr = EigenFit(a), RR.RidgeFit(b)
        for i in (1, 2):
            wo, wr = fo.layer(i, lams), fr.layer(i, lams)
            for lam in lams:
                torch.testing.assert_close(wo[lam][0], wr[lam][0], rtol=1e-5, atol=1e-6)
                torch.testing.assert_close(wo[lam][1], wr[lam][1], rtol=1e-5, atol=1e-6)
            (ro, eo), (rr, er) = fo.reduced_rank(i, 1e-2, [4, 12]), fr.reduced_rank(i, 1e-2, [4, 12])
            torch.testing.assert_close(eo, er, rtol=1e-9, atol=1e-12)
            for r in (4, 12):
                torch.testing.assert_close(ro[r][0], rr[r][0], rtol=1e-5, atol=1e-6)


def test_lean_fit_selects_the_same_lambda_and_maps(tiny_llama):
    """fit(lean=True) solves, scores and drops one lambda at a time; it must pick the lambda the full path picks and
    return the same maps for it."""
    from ridgefill_data_b200.eval.data import zipf_docs
    from ridgefill_data_b200.models.base import load
    from ridgefill_data_b200.ridge import sweep
    path, _ = tiny_llama
    m = load(path, dtype=torch.float32)
    docs = zipf_docs(4, 96, 300, seed=1)
    held = zipf_docs(2, 96, 300, seed=3)
    lams = (1e-3, 0.03, 1.0)
    full = sweep.fit(m, docs, [2], lambdas=lams, held=held, log=None)[2]
    lean = sweep.fit(m, docs, [2], lambdas=lams, held=held, log=None, lean=True)[2]
    assert lean["lambda_star"] == full["lambda_star"]
    for c in [str(x) for x in lams] + ["identity"]:
        assert abs(lean["mean_read_cos"][c] - full["mean_read_cos"][c]) < 1e-9
    best = full["lambda_star"]
    for i, (w, b) in full["maps"][best].items():
        wl, bl = lean["maps"][best][i]
        assert torch.allclose(w, wl) and torch.allclose(b, bl)
