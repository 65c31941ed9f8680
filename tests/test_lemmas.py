"""The reference's formal lemmas (code/lean/kva_lean, Lean 4 + Mathlib; Lean is not on this machine) checked as
executable properties on this framework's own implementations, with hypothesis-generated cases. These are numeric
checks of the statements, not proofs.

  1  GDN prefix-error contraction      ops.oracle.delta_rule_recurrent: two trajectories with the same inputs
                                        differ by at most prod(exp g_t) times their initial difference
  2  speedup monotone and bounded       the two-cost model and eval.cost.CostModel: non-increasing in the split and
                                        the tail, at most L / S, at least 1
  3  running sums = batch ridge         ridge.stats.RidgeStats over two batches equals one batch
  4  uniform logit shift                softmax mass of a set never falls when its logits rise
  5  attention influence                ops.oracle.attend_at: changing one value row moves each query's output by
                                        exactly that row's attention weight times the change; later rows none
  6  attention key sensitivity          ops.oracle.attend: moving one key row by delta changes each weight by at
                                        most a_ij0 (exp|eps_i| - 1), eps_i = scale <q_i, delta>, and each output by
                                        at most a_ij0 (exp|eps_i| |dv| + 2 M (exp|eps_i| - 1)) with the value moved too
  9  QK-norm invariance                 ops.oracle.rms_norm (eps 0) ignores a positive scale of its input
  10 speedup with exact rows            CostModel.bypass: every exact row costs, the speedup falls with the rows
  11 count-matched random control       engine.select.random_rows: exactly k distinct rows, uniform over many prompts
  12 RMSNorm is not affine              ops.oracle.rms_norm does not keep midpoints
  13 context dependence                 causal attention output of a row depends on earlier rows (no per-row fill)
"""
import math

import pytest
import torch
from hypothesis import given, settings
from hypothesis import strategies as st

from ridgefill_data_b200.eval.cost import CostModel
from ridgefill_data_b200.models.config import PRESETS
from ridgefill_data_b200.ops import oracle as O
from ridgefill_data_b200.ridge.fit import EigenFit
from ridgefill_data_b200.ridge.stats import RidgeStats

FAST = settings(max_examples=40, deadline=None, derandomize=True)


@FAST
@given(st.integers(1, 12), st.integers(0, 2 ** 31 - 1), st.floats(0.0, 2.0))
def test_gdn_prefix_contraction(T, seed, beta_max):
    g = torch.Generator().manual_seed(seed)
    h, dk, dv = 2, 6, 4
    q = O.l2norm(torch.randn(h, T, dk, generator=g, dtype=torch.float64)).float()
    k = O.l2norm(torch.randn(h, T, dk, generator=g, dtype=torch.float64)).float()
    v = torch.randn(h, T, dv, generator=g)
    lg = -torch.rand(h, T, generator=g)                                   # alpha = exp(g) in (0, 1]
    beta = torch.rand(h, T, generator=g) * beta_max                       # beta in [0, 2]
    s0, s1 = torch.randn(h, dk, dv, generator=g), torch.randn(h, dk, dv, generator=g)
    _, a = O.delta_rule_recurrent(q, k, v, lg, beta, s0)
    _, b = O.delta_rule_recurrent(q, k, v, lg, beta, s1)
    for j in range(h):
        bound = math.exp(float(lg[j].sum())) * float((s0[j] - s1[j]).norm())
        assert float((a[j] - b[j]).norm()) <= bound * (1 + 1e-4) + 1e-5


def _speedup(L, S, N, T, c, f):
    return L * N * c / (S * N * c + (L - S) * (T * c + (N - T) * f))


@FAST
@given(st.integers(2, 80), st.integers(2, 10 ** 5), st.floats(0.1, 10.0), st.floats(0.0, 1.0), st.data())
def test_speedup_monotone_and_bounded(L, N, c, frac_f, data):
    f = frac_f * c
    S = data.draw(st.integers(1, L))
    T = data.draw(st.integers(0, N))
    s = _speedup(L, S, N, T, c, f)
    assert 1 - 1e-12 <= s <= L / S * (1 + 1e-12)
    if S < L:
        assert _speedup(L, S + 1, N, T, c, f) <= s * (1 + 1e-12)
    if T < N:
        assert _speedup(L, S, N, T + 1, c, f) <= s * (1 + 1e-12)
    if S == L or (T == 0 and f == 0):
        assert s == pytest.approx(L / S)


def test_cost_model_speedup_monotone():
    cm = CostModel(PRESETS["qwen3.8-27b"])
    n = 32768
    by_split = [cm.speedup(n, "proj", split=s, tail=4096) for s in range(4, 64, 4)]
    by_tail = [cm.speedup(n, "proj", split=32, tail=t) for t in (512, 1024, 2048, 4096, 8192, 16384)]
    assert all(a >= b for a, b in zip(by_split, by_split[1:]))
    assert all(a >= b for a, b in zip(by_tail, by_tail[1:]))
    assert all(s >= 1 for s in by_split + by_tail)


def test_running_sums_equal_batch_ridge():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(300, 12, generator=g, dtype=torch.float64)
    y = x @ torch.randn(12, 12, generator=g, dtype=torch.float64) + 0.1 * torch.randn(300, 12, generator=g,
                                                                                          dtype=torch.float64)
    one, two = RidgeStats(0, [1], 12), RidgeStats(0, [1], 12)
    one.add(x.float(), {1: y.float()})
    two.add(x[:170].float(), {1: y[:170].float()})
    two.add(x[170:].float(), {1: y[170:].float()})
    a = EigenFit(one.state()).layer(1, [1e-2])[1e-2]
    b = EigenFit(two.state()).layer(1, [1e-2])[1e-2]
    torch.testing.assert_close(a[0], b[0], rtol=1e-4, atol=1e-5)
    torch.testing.assert_close(a[1], b[1], rtol=1e-4, atol=1e-5)


@FAST
@given(st.integers(2, 30), st.integers(0, 2 ** 31 - 1), st.floats(0.0, 5.0))
def test_softmax_mass_never_falls_when_shifted_up(n, seed, delta):
    g = torch.Generator().manual_seed(seed)
    z = torch.randn(n, generator=g, dtype=torch.float64) * 3
    mask = torch.rand(n, generator=g) < 0.5
    before = torch.softmax(z, 0)[mask].sum()
    after = torch.softmax(z + delta * mask, 0)[mask].sum()
    assert float(after) >= float(before) - 1e-12
    if delta > 0 and 0 < int(mask.sum()) < n:
        assert float(after) > float(before) - 1e-15


def test_attention_value_influence_is_the_weight():
    g = torch.Generator().manual_seed(5)
    hq, n, d = 1, 9, 8
    q, k, v = (torch.randn(hq, n, d, generator=g, dtype=torch.float64) for _ in range(3))
    scale = d ** -0.5
    out = O.attend(q, k, v, scale)
    j = 3
    dv = torch.randn(d, generator=g, dtype=torch.float64)
    v2 = v.clone()
    v2[0, j] += dv
    moved = O.attend(q, k, v2, scale) - out
    s = (q[0] @ k[0].T) * scale
    s = s.masked_fill(torch.ones(n, n, dtype=torch.bool).triu(1), float("-inf"))
    a = torch.softmax(s, -1)
    torch.testing.assert_close(moved, a[:, j:j + 1] * dv[None, :], rtol=1e-5, atol=1e-6)   # fp32 scores
    assert float(moved[:j].abs().max()) == 0.0                        # earlier queries never see row j


@FAST
@given(st.integers(0, 2 ** 31 - 1), st.floats(0.01, 2.0))
def test_attention_key_sensitivity_is_bounded_by_the_weight(seed, size):
    g = torch.Generator().manual_seed(seed)
    n, d, j = 10, 8, 4
    q, k, v = (torch.randn(1, n, d, generator=g, dtype=torch.float64) for _ in range(3))
    scale = d ** -0.5
    dk = torch.randn(d, generator=g, dtype=torch.float64) * size
    dv = torch.randn(d, generator=g, dtype=torch.float64) * size
    causal = torch.ones(n, n, dtype=torch.bool).triu(1)

    def weights(kk):
        return torch.softmax(((q[0] @ kk[0].T) * scale).masked_fill(causal, float("-inf")), -1)
    k2, v2 = k.clone(), v.clone()
    k2[0, j] += dk
    v2[0, j] += dv
    a, a2 = weights(k), weights(k2)
    eps = ((q[0] @ dk) * scale).abs()
    grow = torch.expm1(eps)
    tol = 1e-5                                                          # attend's scores are fp32
    assert ((a2 - a).abs() <= a[:, j:j + 1] * grow[:, None] + tol).all()
    M = float(v[0].norm(dim=-1).max())
    key_only = (O.attend(q, k2, v, scale) - O.attend(q, k, v, scale)).norm(dim=-1)     # [n] (rows, features)
    assert (key_only <= 2 * M * a[:, j] * grow + tol).all()
    both = (O.attend(q, k2, v2, scale) - O.attend(q, k, v, scale)).norm(dim=-1)
    assert (both <= a[:, j] * (eps.exp() * dv.norm() + 2 * M * grow) + tol).all()
    assert float(both[:j].max()) == 0.0                                 # earlier queries never see row j


@FAST
@given(st.integers(0, 2 ** 31 - 1), st.floats(1e-3, 1e3))
def test_rms_norm_ignores_positive_scale(seed, c):
    x = torch.randn(4, 16, generator=torch.Generator().manual_seed(seed), dtype=torch.float64)
    w = torch.ones(16, dtype=torch.float64)
    torch.testing.assert_close(O.rms_norm(c * x, w, 0.0), O.rms_norm(x, w, 0.0), rtol=1e-5, atol=1e-6)  # fp32 math


def test_speedup_falls_with_exact_rows():
    cm = CostModel(PRESETS["llama-3.1-8b"])
    n, split, tail = 32768, 12, 4096
    costs = [cm.bypass(n, split, tail, r) for r in (0, 256, 1024, 4096, 16384)]
    assert all(a < b for a, b in zip(costs, costs[1:]))
    assert cm.bypass(n, split, tail, 0) == pytest.approx(cm.ridgefill(n, split, tail), rel=1e-12)


def test_causal_attention_is_context_dependent():
    g = torch.Generator().manual_seed(7)
    q, k, v = (torch.randn(2, 8, 8, generator=g, dtype=torch.float64) for _ in range(3))
    out = O.attend(q, k, v, 8 ** -0.5)
    k2 = k.clone()
    k2[:, 0] += 1.0                                   # change an earlier row only
    out2 = O.attend(q, k2, v, 8 ** -0.5)
    assert float((out2[5] - out[5]).abs().max()) > 1e-6     # a later row's output moves: no exact per-row fill


def test_random_control_is_count_matched_and_uniform():
    """Lemma 11 (count-matched random control): the random arm picks exactly k of P rows, uniformly, so its expected
    gain is k / P of the total; checked on engine.select.random_rows over many prompt names."""
    from ridgefill_data_b200.engine import select as SEL
    P, k, draws = 20, 5, 4000
    freq = torch.zeros(P)
    for j in range(draws):
        rows = SEL.random_rows(f"prompt-{j}", P, k)
        assert len(rows) == k and len(set(rows)) == k and all(0 <= r < P for r in rows)
        freq[rows] += 1
    share = freq / draws
    assert float((share - k / P).abs().max()) < 0.035          # ~5 standard errors at 4000 draws


@FAST
@given(st.integers(0, 2 ** 31 - 1))
def test_rms_norm_is_not_affine(seed):
    """Lemma 12: an affine fill keeps midpoints; RMSNorm does not (off a ray through the origin), so no affine map of
    the boundary state reproduces a normalised late input on every row."""
    g = torch.Generator().manual_seed(seed)
    x, y = torch.randn(2, 16, generator=g, dtype=torch.float64)
    w = torch.ones(16, dtype=torch.float64)
    f = lambda t: O.rms_norm(t, w, 0.0)  # noqa: E731
    gap = f((x + y) / 2) - (f(x) + f(y)) / 2
    assert float(gap.norm()) > 1e-4
