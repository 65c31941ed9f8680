"""Statistics of paired arm-vs-reference results (the rules of code/finals/stats.py): BCa bootstrap intervals,
p-values by inverting the interval, Holm's step-down adjustment, minimum detectable effects and one-sided
non-inferiority (two one-sided tests when both margins are given).

Declared constants, kept equal to the reference's so that the same data give the same intervals: B = 5000
resamples drawn from numpy's default_rng(20261004), a 95% two-sided level, alpha 0.05 and power 0.80. The
resampling unit is the pairing unit (a prompt, a document, a row); with strata every stratum is resampled within
itself, strata in sorted label order, one integer draw of shape (B, stratum size) each.

BCa (Efron 1987): from the resampled statistics t_b and the leave-one-unit-out statistics t_(i),
    z0 = Phi^-1(share of t_b below the estimate, ties counted one half)
    a  = sum(d^3) / (6 (sum d^2)^(3/2)),   d_i = mean(t_(.)) - t_(i)
and the interval ends are the linearly interpolated quantiles of t_b at Phi(z0 + (z0 + z) / (1 - a (z0 + z))) for
z = Phi^-1((1 - level) / 2) and its negation. An estimand weighs every unit once ("unit") or averages the stratum
means ("stratum"). Data without any variation give a zero-width interval flagged degenerate, which a
non-inferiority test never takes as evidence (except through the bounded-data binomial floor).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field
from statistics import NormalDist

import numpy as np

SEED = 20261004
N_RESAMPLES = 5000
LEVEL = 0.95
ALPHA = 0.05
POWER = 0.80
_PHI = NormalDist()

# how each reported estimand weighs its units
ESTIMANDS = dict(nll="unit", accuracy="unit", longbench="stratum", agreement="unit", kl="unit")


class StatsError(ValueError):
    """The declared statistic is not defined for these inputs."""


class IntervalUndefined(StatsError):
    """The statistic is infinite or NaN on some resample or leave-one-out set (the point estimate is kept)."""

    def __init__(self, estimate, n_bad, n_resamples):
        self.estimate = estimate
        self.n_bad = n_bad
        self.n_resamples = n_resamples
        super().__init__(f"{n_bad}/{n_resamples} bootstrap resamples give a non-finite statistic")


def weighting_of(estimand):
    try:
        return ESTIMANDS[estimand]
    except KeyError:
        raise StatsError(f"estimand {estimand!r} is not declared (one of {sorted(ESTIMANDS)})") from None


def paired(a, b, *, what, subset=False):
    """Align two {unit: value} maps: (sorted units, values of a, values of b). Both must hold the same units, except
    that b may hold extra ones when subset is set."""
    if not a:
        raise StatsError(f"{what}: the first map is empty")
    missing_b = sorted(set(a) - set(b))
    extra_b = sorted(set(b) - set(a))
    if missing_b or (extra_b and not subset):
        raise StatsError(f"{what}: units do not pair up ({missing_b[:5]} lack a partner, {extra_b[:5]} are extra)")
    units = sorted(a)
    va = np.fromiter((a[u] for u in units), dtype=float, count=len(units))
    vb = np.fromiter((b[u] for u in units), dtype=float, count=len(units))
    if not np.isfinite(np.concatenate([va, vb])).all():
        raise StatsError(f"{what}: a paired value is NaN or infinite")
    return units, va, vb


class _Design:
    """Units, strata and weighting of one estimand; computes it on the data, on resamples and leaving each unit
    out."""

    def __init__(self, x, strata, weighting):
        self.x = x
        n = x.shape[0]
        if strata is None:
            self.groups = [np.arange(n)]
        else:
            labels = np.array([str(s) for s in strata])
            if labels.shape != (n,):
                raise StatsError(f"{labels.shape[0]} stratum labels for {n} units")
            self.groups = [np.flatnonzero(labels == lab) for lab in sorted(set(labels.tolist()))]
        self.by_unit = weighting == "unit"
        if not self.by_unit and any(len(g) < 2 for g in self.groups):
            raise StatsError("stratum weighting needs two or more units in every stratum")

    def point(self):
        if self.by_unit:
            return self.x.mean(axis=0)
        return np.mean([self.x[g].mean(axis=0) for g in self.groups], axis=0)

    def resampled(self, rng, B):
        draws = [g[rng.integers(0, len(g), (B, len(g)))] for g in self.groups]
        if self.by_unit:
            return self.x[np.concatenate(draws, axis=1)].mean(axis=1)
        return np.mean([self.x[d].mean(axis=1) for d in draws], axis=0)

    def leave_one_out(self):
        x = self.x
        if self.by_unit:
            return (x.sum(axis=0)[None, :] - x) / (x.shape[0] - 1)
        means = np.stack([x[g].mean(axis=0) for g in self.groups])
        total = means.sum(axis=0)
        out = np.empty_like(x)
        for j, g in enumerate(self.groups):
            without = (x[g].sum(axis=0)[None, :] - x[g]) / (len(g) - 1)
            out[g] = ((total - means[j])[None, :] + without) / len(self.groups)
        return out


@dataclass
class BCa:
    estimate: float
    lo: float
    hi: float
    n: int
    se: float
    z0: float
    a: float
    level: float
    n_resamples: int
    seed: int
    degenerate: bool
    theta_b: np.ndarray = field(repr=False)

    def excludes(self, null=0.0):
        return not self.lo <= null <= self.hi


def _below(values, at):
    """Share of values below `at`, a value equal to it counting one half."""
    return (np.count_nonzero(values < at) + np.count_nonzero(values <= at)) / (2 * values.size)


def bca(data, *, stat=None, strata=None, weighting="unit", n_resamples=N_RESAMPLES, seed=SEED, level=LEVEL):
    """BCa interval of stat(means) over units; data is [n] or [n, k] (the k columns of a unit move together) and
    stat maps [..., k] means to [...] (default: the first column)."""
    x = np.asarray(data, dtype=float)
    if x.ndim == 1:
        x = x.reshape(-1, 1)
    if x.ndim != 2:
        raise StatsError(f"expected data of shape (n,) or (n, k), not {x.shape}")
    n = x.shape[0]
    if n < 2:
        raise StatsError(f"{n} unit(s): a bootstrap interval needs two or more")
    if not np.isfinite(x).all():
        raise StatsError("the data hold NaN or infinite values")
    if weighting not in ("unit", "stratum"):
        raise StatsError(f"weighting must be 'unit' or 'stratum', not {weighting!r}")
    if not (0.0 < level < 1.0) or n_resamples < 100:
        raise StatsError(f"need 0 < level < 1 and at least 100 resamples (level {level}, {n_resamples} resamples)")
    if stat is None:
        stat = lambda m: m[..., 0]                                   # noqa: E731
    design = _Design(x, strata, weighting)
    boot_means = design.resampled(np.random.default_rng(seed), n_resamples)
    with np.errstate(divide="ignore", invalid="ignore"):
        t_b = np.asarray(stat(boot_means), dtype=float)
        est = float(stat(design.point()))
        t_j = np.asarray(stat(design.leave_one_out()), dtype=float)
    if not (math.isfinite(est) and np.isfinite(t_b).all() and np.isfinite(t_j).all()):
        raise IntervalUndefined(est, int((~np.isfinite(t_b)).sum()), n_resamples)
    se = float(t_b.std(ddof=1))
    d = t_j.mean() - t_j
    common = dict(n=n, level=level, n_resamples=n_resamples, seed=seed, theta_b=t_b)
    if se == 0.0 and not d.any():
        return BCa(est, est, est, se=0.0, z0=0.0, a=0.0, degenerate=True, **common)
    frac = _below(t_b, est)
    if frac <= 0.0 or frac >= 1.0:
        raise StatsError(f"no BCa interval: every resample lies on one side of the estimate {est:.6g}")
    z0 = _PHI.inv_cdf(frac)
    d2 = float((d * d).sum())
    accel = float((d ** 3).sum() / (6.0 * d2 ** 1.5)) if d2 > 0 else 0.0
    z = _PHI.inv_cdf((1.0 - level) / 2.0)

    def adjusted(zq):
        return _PHI.cdf(z0 + (z0 + zq) / (1.0 - accel * (z0 + zq)))

    lo, hi = np.quantile(t_b, [adjusted(z), adjusted(-z)])
    return BCa(est, float(lo), float(hi), se=se, z0=z0, a=accel, degenerate=False, **common)


def pvalue(res, null=0.0):
    """Two-sided p-value of the hypothesis theta = null: twice the BCa tail level at which an interval end reaches
    null, at least 1 / B."""
    B = res.n_resamples
    floor = 1.0 / B
    if res.degenerate:
        return 1.0 if res.estimate == null else floor
    g = float(np.clip(_below(res.theta_b, null), 0.5 / B, 1.0 - 0.5 / B))
    v = _PHI.inv_cdf(g) - res.z0
    den = 1.0 + res.a * v
    if den <= 0.0:
        return floor
    tail = _PHI.cdf(v / den - res.z0)
    return float(np.clip(2.0 * min(tail, 1.0 - tail), floor, 1.0))


def holm(pvals):
    """Holm step-down adjusted p-values of one family {name: p}: monotone in the raw order, capped at 1."""
    bad = {k: p for k, p in pvals.items() if not 0.0 <= p <= 1.0}
    if bad:
        raise StatsError(f"Holm adjustment of p-values outside [0, 1]: {bad}")
    ranked = sorted(pvals.items(), key=lambda kv: (kv[1], kv[0]))
    m = len(ranked)
    steps = np.minimum(1.0, np.array([(m - i) * p for i, (_, p) in enumerate(ranked)]))
    adj = np.maximum.accumulate(steps) if m else steps
    return {name: float(v) for (name, _), v in zip(ranked, adj)}


def mde(sd, n, alpha=ALPHA, power=POWER):
    """Minimum detectable effect of a two-sided test: (z(1 - alpha / 2) + z(power)) * sd / sqrt(n)."""
    if n < 2 or not (math.isfinite(sd) and sd >= 0):
        raise StatsError(f"an MDE needs n >= 2 units and a finite, non-negative sd (got n={n}, sd={sd})")
    return (_PHI.inv_cdf(1.0 - alpha / 2.0) + _PHI.inv_cdf(power)) * sd / math.sqrt(n)


def mde_paired(deltas, alpha=ALPHA, power=POWER):
    """(sd, n, MDE) of one-dimensional paired differences."""
    d = np.asarray(deltas, dtype=float)
    if d.ndim != 1 or len(d) < 2 or not np.isfinite(d).all():
        raise StatsError("an MDE of paired differences needs a 1-D array of two or more finite values")
    sd = float(d.std(ddof=1))
    return sd, len(d), mde(sd, len(d), alpha, power)


@dataclass
class NonInferiority:
    estimate: float
    lo: float
    hi: float
    lower: object
    upper: object
    passed: bool
    n: int
    alpha: float
    method: str
    reason: str


DEGENERATE = "degenerate: data without variation give no finite-sample guarantee"


def binomial_floor(n, alpha=ALPHA):
    """One-sided (1 - alpha) upper bound on the share of worse units when none of n is worse: 1 - alpha^(1/n)."""
    return 1.0 - alpha ** (1.0 / n)


def _check_range(x, unit_range, kw):
    a, b = float(unit_range[0]), float(unit_range[1])
    if x.ndim != 1:
        raise StatsError("a unit_range bound applies to one-dimensional paired differences")
    if kw.get("weighting", "unit") != "unit":
        raise StatsError("the binomial floor is defined for unit-weighted means")
    if not (a < 0.0 < b):
        raise StatsError(f"unit_range {unit_range} must contain 0 in its interior")
    if x.min() < a or x.max() > b:
        raise StatsError(f"paired differences fall outside unit_range {unit_range}")
    return a, b


def noninferiority(data, *, lower=None, upper=None, alpha=ALPHA, unit_range=None, **kw):
    """Test paired differences against one-sided margins. A side passes when its one-sided (1 - alpha) bound (an
    end of the (1 - 2 alpha) BCa interval) lies inside the margin. With unit_range = (a, b), a < 0 < b, the
    differences are bounded: on a side where no unit is worse, the bound is the exact binomial floor share times
    a or b, and on the other sides the floor replaces the BCa bound where it is the stricter one."""
    if lower is None and upper is None:
        raise StatsError("declare a lower or an upper margin")
    if lower is not None and upper is not None and lower >= upper:
        raise StatsError(f"the lower margin {lower} must lie below the upper margin {upper}")
    if not 0.0 < alpha < 0.5:
        raise StatsError(f"alpha must lie in (0, 0.5), not {alpha}")
    res = bca(data, level=1.0 - 2.0 * alpha, **kw)
    x = np.asarray(data, dtype=float)
    flat = res.degenerate or bool(np.all(x == x[:1]))
    pct = f"{100 * (1 - alpha):g}%"

    def refused():
        return NonInferiority(res.estimate, res.lo, res.hi, lower, upper, False, res.n, alpha, "bca", DEGENERATE)

    bounds = {"lower": res.lo, "upper": res.hi}
    methods, notes = set(), []
    if unit_range is None:
        if flat:
            return refused()
        methods.add("bca")
        notes.append(f"one-sided {pct} BCa bound")
    else:
        a, b = _check_range(x, unit_range, kw)
        share = binomial_floor(res.n, alpha)
        for side, margin in (("lower", lower), ("upper", upper)):
            if margin is None:
                continue
            floor = share * (a if side == "lower" else b)
            if (x >= 0).all() if side == "lower" else (x <= 0).all():
                bounds[side] = floor
                methods.add("exact-binomial-floor")
                notes.append(f"no unit worse: exact binomial floor ({100 * share:.2f}% worse units at most)")
                continue
            if flat:
                return refused()
            stricter = floor < bounds[side] if side == "lower" else floor > bounds[side]
            if stricter:
                bounds[side] = floor
            methods.add("exact-binomial-floor" if stricter else "bca")
            notes.append(f"one-sided {pct} BCa bound" + (", replaced by the stricter binomial floor" if stricter
                                                          else ""))
    lo, hi = bounds["lower"], bounds["upper"]
    passed = (lower is None or lo >= lower) and (upper is None or hi <= upper)
    method = "+".join(sorted(methods))
    return NonInferiority(res.estimate, float(lo), float(hi), lower, upper, bool(passed), res.n, alpha, method,
                          "; ".join(notes))


def tost(data, *, lower=None, upper=None, alpha=ALPHA, **kw):
    """The same test as noninferiority(), under its older name (an equivalence test when both margins are given)."""
    return noninferiority(data, lower=lower, upper=upper, alpha=alpha, **kw)
