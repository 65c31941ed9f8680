"""Paired statistics against scipy's BCa bootstrap (the oracle), plus the p-value, Holm, MDE and non-inferiority
rules."""
import numpy as np
import pytest
from scipy import stats as sps

from ridgefill_data_b200.eval import stats as ST


def test_bca_matches_scipy():
    rng = np.random.default_rng(1)
    x = rng.gamma(2.0, 1.5, size=60) - 2.5
    ours = ST.bca(x, n_resamples=4000, seed=7)
    ref = sps.bootstrap((x,), np.mean, method="BCa", n_resamples=4000, confidence_level=0.95,
                        random_state=np.random.default_rng(7), vectorized=True)
    lo, hi = ref.confidence_interval
    width = hi - lo
    assert abs(ours.lo - lo) < 0.03 * width and abs(ours.hi - hi) < 0.03 * width
    assert ours.estimate == pytest.approx(x.mean())


def test_bca_ratio_and_strata():
    rng = np.random.default_rng(2)
    num, den = rng.normal(1.0, 0.3, 40), rng.normal(2.0, 0.2, 40)
    r = ST.bca(np.stack([num, den], 1), stat=lambda m: m[..., 0] / m[..., 1], n_resamples=2000)
    assert r.lo < num.mean() / den.mean() < r.hi
    strata = ["a"] * 20 + ["b"] * 20
    s = ST.bca(num, strata=strata, weighting="stratum", n_resamples=2000)
    assert s.estimate == pytest.approx((num[:20].mean() + num[20:].mean()) / 2)
    with pytest.raises(ST.IntervalUndefined):
        ST.bca(np.stack([num, np.r_[0.0, np.zeros(39)]], 1), stat=lambda m: m[..., 0] / m[..., 1], n_resamples=200)


def test_degenerate_and_refusals():
    r = ST.bca(np.full(10, 0.5), n_resamples=200)
    assert r.degenerate and r.lo == r.hi == 0.5
    assert ST.pvalue(r, 0.5) == 1.0
    with pytest.raises(ST.StatsError):
        ST.bca([1.0])
    with pytest.raises(ST.StatsError):
        ST.paired({"a": 1.0}, {"b": 2.0}, what="x")
    units, xa, xb = ST.paired({"a": 1.0, "b": 2.0}, {"a": 0.5, "b": 1.0, "c": 3.0}, what="x", subset=True)
    assert units == ["a", "b"] and xb.tolist() == [0.5, 1.0]


def test_pvalue_agrees_with_interval():
    rng = np.random.default_rng(3)
    for shift in (0.0, 0.3, 0.8):
        x = rng.normal(shift, 1.0, 80)
        r = ST.bca(x, n_resamples=3000)
        p = ST.pvalue(r)
        assert (p < 0.05) == r.excludes(0.0) or abs(p - 0.05) < 0.01


def test_holm_and_mde():
    adj = ST.holm({"a": 0.01, "b": 0.04, "c": 0.03})
    assert adj == {"a": pytest.approx(0.03), "c": pytest.approx(0.06), "b": pytest.approx(0.06)}
    assert ST.mde(1.0, 100) == pytest.approx((1.959964 + 0.841621) / 10, rel=1e-5)
    sd, n, m = ST.mde_paired([1.0, 2.0, 3.0])
    assert n == 3 and sd == pytest.approx(1.0)


def test_noninferiority():
    rng = np.random.default_rng(4)
    good = rng.normal(0.0, 0.5, 100)
    assert ST.noninferiority(good, upper=0.5).passed
    assert not ST.noninferiority(good + 1.0, upper=0.5).passed
    assert not ST.noninferiority(np.zeros(30), upper=0.5).passed                      # degenerate
    none_worse = ST.noninferiority(np.zeros(96), lower=-5.0, unit_range=(-100, 100))
    assert none_worse.passed and none_worse.method == "exact-binomial-floor"
    assert none_worse.lo == pytest.approx(-100 * (1 - 0.05 ** (1 / 96)))
    with pytest.raises(ST.StatsError):
        ST.noninferiority(good)


def test_paired_tables(tmp_path):
    import json
    from ridgefill_data_b200.eval import tables as TB
    rng = np.random.default_rng(7)
    for j in range(30):
        base = float(rng.normal(2.0, 0.3))
        runs = {"exact": {"nll": base}, "ridgefill": {"nll": base + 0.01 + float(rng.normal(0, 0.005))},
                "identity": {"nll": base + 0.3 + float(rng.normal(0, 0.05))}}
        (tmp_path / f"p{j}.json").write_text(json.dumps(dict(name=f"p{j}", runs=runs)))
    (tmp_path / "broken.json").write_text(json.dumps(dict(name="b", runs={"exact": {"nll": float("nan")}})))
    rows = TB.paired_table(TB.load_records(tmp_path), "nll", "exact", n_resamples=1000, upper=0.05)
    by = {r["arm"]: r for r in rows}
    assert by["ridgefill"]["n"] == 30 and by["ridgefill"]["lo"] < 0.01 < by["ridgefill"]["hi"]
    assert by["ridgefill"]["noninferior"] and not by["identity"]["noninferior"]
    assert by["identity"]["p_holm"] < 0.01
    md = TB.markdown(rows, "nll", "exact")
    assert md.count("\n") == 3 and "ridgefill" in md
    tex = TB.latex(rows, "nll", "exact")
    assert tex.startswith("\\begin{tabular}") and "\\checkmark" in tex


def test_statistics_match_the_reference():
    """BCa intervals (plain, ratio, stratified), p-values, Holm, MDE and non-inferiority against the reference's
    finals/stats.py (installed in baseline/_ref): the same declared seed and resample count give the same numbers."""
    import importlib.util
    from pathlib import Path
    path = Path(__file__).resolve().parent.parent / "baseline" / "_ref" / "finals" / "stats.py"
    if not path.exists():
        pytest.skip("baseline/_ref not installed")
    spec = importlib.util.spec_from_file_location("ref_finals_stats", path)
    RS = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(RS)
    assert (RS.SEED, RS.N_RESAMPLES) == (ST.SEED, ST.N_RESAMPLES)
    rng = np.random.default_rng(5)
    x = rng.normal(0.2, 1.0, 70)
    pairs = np.stack([rng.normal(1.0, 0.2, 50), rng.normal(2.0, 0.2, 50)], 1)
    strata = ["a"] * 30 + ["b"] * 40
    cases = [(x, {}), (pairs, dict(stat=lambda m: m[..., 0] / m[..., 1])),
             (x, dict(strata=strata, weighting="stratum")), (x, dict(strata=strata))]
    for data, kw in cases:
        a, b = ST.bca(data, n_resamples=2000, **kw), RS.bca(data, n_resamples=2000, **kw)
        assert (a.estimate, a.lo, a.hi) == pytest.approx((b.estimate, b.lo, b.hi), rel=1e-12, abs=1e-12)
        assert ST.pvalue(a) == pytest.approx(RS.pvalue(b), abs=1e-12)
    p = {"a": 0.01, "b": 0.04, "c": 0.03, "d": 0.2}
    assert ST.holm(p) == pytest.approx(RS.holm(p))
    assert ST.mde(1.3, 64) == pytest.approx(RS.mde(1.3, 64))
    for kw in (dict(upper=0.5), dict(lower=-0.5), dict(lower=-5.0, unit_range=(-100, 100))):
        a, b = ST.noninferiority(x, n_resamples=2000, **kw), RS.noninferiority(x, n_resamples=2000, **kw)
        assert a.passed == b.passed and (a.lo, a.hi) == pytest.approx((b.lo, b.hi), rel=1e-12, abs=1e-12)
    z = np.zeros(96)
    a, b = ST.noninferiority(z, lower=-5.0, unit_range=(-100, 100)), RS.noninferiority(z, lower=-5.0,
                                                                                       unit_range=(-100, 100))
    assert (a.passed, a.method) == (b.passed, b.method) and a.lo == pytest.approx(b.lo)
    assert ST.tost(x, upper=0.5, n_resamples=500).passed == RS.tost(x, upper=0.5, n_resamples=500).passed
