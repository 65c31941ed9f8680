"""Statistics of paired arm-vs-reference results (code/finals/stats.py): BCa bootstrap intervals, p-values by
interval inversion, Holm's step-down adjustment, minimum detectable effects and one-sided non-inferiority tests.

Declared constants (kept as the reference declares them so intervals reproduce): 5000 resamples of units with seed
20261004, 95% two-sided level, alpha 0.05, power 0.80. A unit is one prompt / document / row holding every arm
(the pairing unit); strata (e.g. a task) resample within themselves.

BCa (Efron 1987, "Better bootstrap confidence intervals"): with theta_b the resampled statistics and theta_(i) the
leave-one-unit-out statistics,
    z0 = Phi^-1( (#{theta_b < theta} + #{theta_b <= theta}) / (2 B) )            (ties count one half)
    a  = sum d^3 / (6 (sum d^2)^1.5),  d = mean(theta_(.)) - theta_(i)            (jackknife acceleration)
    endpoint(z) = quantile of theta_b at Phi(z0 + (z0 + z) / (1 - a (z0 + z))),  z = -/+ Phi^-1(1 - level / 2 ... )
with linearly interpolated quantiles. Estimands are "unit" weighted (every unit once) or "stratum" weighted (the
mean of the stratum means). Identical paired differences give a degenerate zero-width interval (flagged), which a
non-inferiority test never accepts as evidence unless the bounded-data binomial floor decides.
Pure numpy + statistics.NormalDist; scipy serves as the oracle in the tests.
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
_N = NormalDist()

ESTIMANDS = {
    "nll": "unit",          # document-weighted mean of per-document arm-minus-exact NLL
    "accuracy": "unit",     # row-weighted (pooled over tasks and lengths)
    "longbench": "stratum", # mean of the task means
    "agreement": "unit",    # prompt-weighted share of agreeing decode steps
    "kl": "unit",           # prompt-weighted mean per-step KL
}


class StatsError(ValueError):
    """The statistic cannot be computed from these inputs as declared."""


class IntervalUndefined(StatsError):
    """The statistic is not finite on some resample or leave-one-out set; carries the point estimate."""

    def __init__(self, estimate, n_bad, n_resamples):
        super().__init__(f"the statistic is not finite on {n_bad} of {n_resamples} resamples")
        self.estimate, self.n_bad, self.n_resamples = estimate, n_bad, n_resamples


def weighting_of(estimand):
    if estimand not in ESTIMANDS:
        raise StatsError(f"undeclared estimand {estimand!r}: declared are {sorted(ESTIMANDS)}")
    return ESTIMANDS[estimand]


def paired(a, b, *, what, subset=False):
    """(sorted units, xa, xb) of two {unit: value} maps that must hold the same units (b may hold more when
    subset)."""
    ka, kb = set(a), set(b)
    if not ka:
        raise StatsError(f"{what}: no units on the first side")
    only_a, only_b = sorted(ka - kb), sorted(kb - ka)
    if only_a or (only_b and not subset):
        raise StatsError(f"{what}: unpaired units (first only {only_a[:5]}, second only {only_b[:5]})")
    units = sorted(ka)
    xa = np.array([a[u] for u in units], dtype=float)
    xb = np.array([b[u] for u in units], dtype=float)
    if not (np.isfinite(xa).all() and np.isfinite(xb).all()):
        raise StatsError(f"{what}: non-finite value in a paired unit")
    return units, xa, xb


def _strata(n, strata):
    if strata is None:
        return [np.arange(n)]
    labels = np.asarray([str(s) for s in strata])
    if labels.shape != (n,):
        raise StatsError(f"strata has {labels.shape[0]} labels for {n} units")
    return [np.flatnonzero(labels == lab) for lab in sorted(set(labels.tolist()))]


def _means(x, groups, weighting):
    if weighting == "unit":
        return x.mean(axis=0)
    return np.mean([x[g].mean(axis=0) for g in groups], axis=0)


def _loo_means(x, groups, weighting):
    """Leave-one-unit-out estimand means [n, k] in closed form."""
    n = x.shape[0]
    if weighting == "unit":
        return (x.sum(axis=0)[None, :] - x) / (n - 1)
    gm = np.stack([x[g].mean(axis=0) for g in groups])
    out = np.empty_like(x)
    for gi, g in enumerate(groups):
        others = gm.sum(axis=0) - gm[gi]
        out[g] = (others[None, :] + (x[g].sum(axis=0)[None, :] - x[g]) / (len(g) - 1)) / len(groups)
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
        return self.lo > null or self.hi < null


def bca(data, *, stat=None, strata=None, weighting="unit", n_resamples=N_RESAMPLES, seed=SEED, level=LEVEL):
    """BCa interval of stat(estimand means) over units. data [n] or [n, k] (a unit's columns resample together);
    stat maps [..., k] means to [...] (default: column 0)."""
    x = np.asarray(data, dtype=float)
    x = x[:, None] if x.ndim == 1 else x
    if x.ndim != 2:
        raise StatsError(f"data must be (n,) or (n, k), got {x.shape}")
    n, k = x.shape
    if n < 2:
        raise StatsError(f"BCa needs at least 2 units, got {n}")
    if not np.isfinite(x).all():
        raise StatsError("non-finite value in the data")
    if weighting not in ("unit", "stratum"):
        raise StatsError(f"unknown weighting {weighting!r}")
    if not 0.0 < level < 1.0 or n_resamples < 100:
        raise StatsError(f"level {level} / n_resamples {n_resamples} out of range")
    stat = stat or (lambda m: m[..., 0])
    groups = _strata(n, strata)
    if weighting == "stratum" and min(len(g) for g in groups) < 2:
        raise StatsError("stratum weighting needs at least 2 units per stratum")
    rng = np.random.default_rng(seed)
    picks = [g[rng.integers(0, len(g), (n_resamples, len(g)))] for g in groups]
    if weighting == "unit":
        idx = np.concatenate(picks, axis=1)
        means_b = x[idx].mean(axis=1)                                  # [B, k]
    else:
        means_b = np.mean([x[p].mean(axis=1) for p in picks], axis=0)
    with np.errstate(divide="ignore", invalid="ignore"):
        theta_b = np.asarray(stat(means_b), dtype=float)
        theta = float(stat(_means(x, groups, weighting)))
        theta_j = np.asarray(stat(_loo_means(x, groups, weighting)), dtype=float)
    if not (np.isfinite(theta_b).all() and np.isfinite(theta_j).all() and math.isfinite(theta)):
        raise IntervalUndefined(theta, int(np.count_nonzero(~np.isfinite(theta_b))), n_resamples)
    se = float(theta_b.std(ddof=1))
    d = theta_j.mean() - theta_j
    if se == 0.0 and not d.any():
        return BCa(theta, theta, theta, n, 0.0, 0.0, 0.0, level, n_resamples, seed, True, theta_b)
    share = (np.count_nonzero(theta_b < theta) + np.count_nonzero(theta_b <= theta)) / (2 * n_resamples)
    if not 0.0 < share < 1.0:
        raise StatsError(f"BCa undefined: the estimate {theta:.6g} lies outside every bootstrap resample")
    z0 = _N.inv_cdf(share)
    ss = float((d * d).sum())
    a = float((d ** 3).sum() / (6.0 * ss ** 1.5)) if ss > 0 else 0.0
    z = _N.inv_cdf((1.0 - level) / 2.0)
    levels = [_N.cdf(z0 + (z0 + zz) / (1.0 - a * (z0 + zz))) for zz in (z, -z)]
    lo, hi = np.quantile(theta_b, levels)
    return BCa(theta, float(lo), float(hi), n, se, z0, a, level, n_resamples, seed, False, theta_b)


def pvalue(res, null=0.0):
    """Two-sided p-value of theta = null: the level at which a BCa endpoint reaches null (floor 1 / B)."""
    floor = 1.0 / res.n_resamples
    if res.degenerate:
        return 1.0 if res.estimate == null else floor
    B = res.n_resamples
    g = (np.count_nonzero(res.theta_b < null) + np.count_nonzero(res.theta_b <= null)) / (2 * B)
    g = min(max(g, 1.0 / (2 * B)), 1.0 - 1.0 / (2 * B))
    v = _N.inv_cdf(g) - res.z0
    if 1.0 + res.a * v <= 0.0:
        return floor
    tail = _N.cdf(v / (1.0 + res.a * v) - res.z0)
    return float(min(1.0, max(floor, 2.0 * min(tail, 1.0 - tail))))


def holm(pvals):
    """Holm step-down adjusted p-values of one family {name: p} (monotone, capped at 1)."""
    order = sorted(pvals, key=lambda name: (pvals[name], name))
    out, running = {}, 0.0
    for i, name in enumerate(order):
        p = pvals[name]
        if not 0.0 <= p <= 1.0:
            raise StatsError(f"Holm: p-value of {name!r} is {p}")
        running = max(running, min(1.0, (len(order) - i) * p))
        out[name] = running
    return out


def mde(sd, n, alpha=ALPHA, power=POWER):
    """(z(1 - alpha / 2) + z(power)) sd / sqrt(n)."""
    if n < 2 or not math.isfinite(sd) or sd < 0:
        raise StatsError(f"MDE needs n >= 2 and a finite sd >= 0 (n {n}, sd {sd})")
    return (_N.inv_cdf(1.0 - alpha / 2.0) + _N.inv_cdf(power)) * sd / math.sqrt(n)


def mde_paired(deltas, alpha=ALPHA, power=POWER):
    d = np.asarray(deltas, dtype=float)
    if d.ndim != 1 or d.size < 2 or not np.isfinite(d).all():
        raise StatsError("MDE needs at least 2 finite paired deltas")
    sd = float(d.std(ddof=1))
    return sd, int(d.size), mde(sd, d.size, alpha, power)


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


DEGENERATE = "degenerate: zero observed variation is not a finite-sample guarantee"


def binomial_floor(n, alpha=ALPHA):
    """One-sided (1 - alpha) upper bound on the share of worse units when none of n is: 1 - alpha^(1/n)."""
    return 1.0 - alpha ** (1.0 / n)


def noninferiority(data, *, lower=None, upper=None, alpha=ALPHA, unit_range=None, **kw):
    """Paired differences against one-sided margins (both: two one-sided tests). Passes when the one-sided
    (1 - alpha) bounds (the ends of the (1 - 2 alpha) BCa interval) sit on the right side of the margins.
    unit_range (a < 0 < b): bounded per-unit differences; where no unit is worse in a margin's direction that bound
    is the exact binomial floor share x (a or b), and it replaces a less conservative BCa bound otherwise."""
    if lower is None and upper is None:
        raise StatsError("non-inferiority needs at least one declared margin")
    if lower is not None and upper is not None and not lower < upper:
        raise StatsError(f"margins out of order: {lower} >= {upper}")
    if not 0.0 < alpha < 0.5:
        raise StatsError(f"alpha {alpha} out of range")
    r = bca(data, level=1.0 - 2.0 * alpha, **kw)
    x = np.asarray(data, dtype=float)
    degenerate = r.degenerate or bool((x == x[:1]).all())
    lo, hi = r.lo, r.hi
    methods, reasons = set(), []
    if unit_range is None:
        if degenerate:
            return NonInferiority(r.estimate, lo, hi, lower, upper, False, r.n, alpha, "bca", DEGENERATE)
        methods.add("bca")
        reasons.append(f"one-sided {100 * (1 - alpha):g}% BCa bound")
    else:
        a, b = (float(v) for v in unit_range)
        if x.ndim != 1:
            raise StatsError("unit_range applies to (n,) paired differences only")
        if kw.get("weighting", "unit") != "unit":
            raise StatsError("the binomial floor holds for unit-weighted means only")
        if not a < 0.0 < b:
            raise StatsError(f"unit_range {unit_range} must hold 0 strictly inside")
        if x.min() < a or x.max() > b:
            raise StatsError(f"a paired difference lies outside unit_range {unit_range}")
        share = binomial_floor(r.n, alpha)
        for side, margin in (("lower", lower), ("upper", upper)):
            if margin is None:
                continue
            floor = share * (a if side == "lower" else b)
            none_worse = bool((x >= 0).all() if side == "lower" else (x <= 0).all())
            if none_worse:
                bound, m = floor, "exact-binomial-floor"
                reasons.append(f"no unit worse: exact binomial floor ({100 * share:.2f}% worse units at most)")
            elif degenerate:
                return NonInferiority(r.estimate, lo, hi, lower, upper, False, r.n, alpha, "bca", DEGENERATE)
            else:
                bca_bound = r.lo if side == "lower" else r.hi
                stricter = floor < bca_bound if side == "lower" else floor > bca_bound
                bound, m = (floor, "exact-binomial-floor") if stricter else (bca_bound, "bca")
                reasons.append(f"one-sided {100 * (1 - alpha):g}% BCa bound" +
                               (", replaced by the stricter binomial floor" if stricter else ""))
            if side == "lower":
                lo = bound
            else:
                hi = bound
            methods.add(m)
    ok = (lower is None or lo >= lower) and (upper is None or hi <= upper)
    method = methods.pop() if len(methods) == 1 else "+".join(sorted(methods))
    return NonInferiority(r.estimate, float(lo), float(hi), lower, upper, bool(ok), r.n, alpha, method,
                          "; ".join(reasons))


tost = noninferiority


def tost(data, *, lower=None, upper=None, alpha=ALPHA, **kw):
    """noninferiority() under the name the battery's earlier statistics used (equivalence when both margins are
    declared); the same rule, including the refusal of a degenerate interval."""
    return noninferiority(data, lower=lower, upper=upper, alpha=alpha, **kw)
