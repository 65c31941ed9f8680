"""Causality (changing only later tokens never changes earlier logits, for exact and filled arms, including a
tail-measured statistic kept off the scored rows) and multi-turn repair (zero repair is a no-op, partial repair
touches rows below R only, selected-row repair only the selected rows) on tiny checkpoints, CPU fp32
(the reference's test_causal_scoring / test_multiturn strategy)."""
import pytest
import torch

from ridgefill_data_b200.engine import multiturn as MT
from ridgefill_data_b200.engine.arm import Arm, exclude_scored
from ridgefill_data_b200.engine.prefill import finish, prefill, run_lower
from ridgefill_data_b200.eval.data import zipf_docs
from ridgefill_data_b200.models.base import load
from ridgefill_data_b200.ridge import sweep


@pytest.fixture(scope="module", params=["tiny_llama", "tiny_qwen35"])
def model(request):
    path, _ = request.getfixturevalue(request.param)
    return load(path, dtype=torch.float32)


@pytest.fixture(scope="module")
def maps(model):
    return sweep.fit(model, zipf_docs(4, 96, 300, seed=1), [2], held=zipf_docs(2, 96, 300, seed=3), log=None)[2]


def _ids(seed=7, n=100):
    return torch.randint(0, 300, (n,), generator=torch.Generator().manual_seed(seed))


@pytest.mark.parametrize("kind", ["exact", "proj", "identity", "proj_tail_bias"])
def test_later_tokens_never_change_earlier_logits(model, maps, kind):
    keep, changed = 12, 3
    ids = _ids()
    other = ids.clone()
    other[-changed:] = (other[-changed:] + 17) % 300
    if kind == "exact":
        arm = Arm("exact")
    elif kind == "identity":
        arm = Arm("id", split=2, tail=40, fill="identity")
    else:
        arm = Arm("rf", split=2, tail=40, fill="proj", projector=maps["projector"])
        if kind == "proj_tail_bias":   # a statistic over the tail rows, kept off the scored rows
            arm = exclude_scored(Arm("rf", split=2, tail=40, fill="proj", projector=maps["projector"],
                                     tail_bias_from=3), keep)
    a, _, _ = prefill(model, ids, arm, keep=keep)
    b, _, _ = prefill(model, other, arm, keep=keep)
    # rows whose inputs precede the changed tokens see identical prefixes
    assert torch.equal(a[:keep - changed], b[:keep - changed])
    assert not torch.equal(a[-1], b[-1])


def _late_cache(model, ids, split=2, tail=30):
    arm = Arm("id", split=split, tail=tail, fill="identity")
    hs, lower = run_lower(model, ids, [split])
    _, cache, P = finish(model, ids, hs[split], lower, arm, 1)
    return arm, hs[split], cache, P


def test_zero_repair_is_a_no_op(model):
    ids = _ids(3, 80)
    arm, hb, cache, P = _late_cache(model, ids)
    before = {i: {k: v.clone() for k, v in c.items() if torch.is_tensor(v)} for i, c in enumerate(cache)}
    MT.repair(model, cache, hb, arm.split, 0)
    for i, c in enumerate(cache):
        for k, v in before[i].items():   # reserve rows past the filled length are uninitialised (may hold NaN)
            torch.testing.assert_close(c[k], v, rtol=0, atol=0, equal_nan=True)


def test_partial_repair_touches_rows_below_r_only(model):
    ids = _ids(4, 80)
    arm, hb, cache, P = _late_cache(model, ids)
    _, exact = model.forward_exact(ids)
    R = 20
    before = {i: (cache[i]["k"].clone(), cache[i]["v"].clone()) for i in range(arm.split, model.n_layers)
              if model.layer_types[i] == "attn"}
    MT.repair(model, cache, hb, arm.split, R)
    for i, (k0, v0) in before.items():
        assert torch.equal(cache[i]["k"][:, R:], k0[:, R:]) and torch.equal(cache[i]["v"][:, R:], v0[:, R:])
        torch.testing.assert_close(cache[i]["k"][:, :R], exact[i]["k"][:, :R], atol=1e-5, rtol=1e-4)


def test_selected_repair_touches_selected_rows_only(model):
    if any(t != "attn" for t in model.layer_types):
        pytest.skip("selected-row repair rewrites attention K/V only")
    ids = _ids(5, 80)
    arm, hb, cache, P = _late_cache(model, ids)
    rows = [3, 11, 40]
    before = {i: cache[i]["k"].clone() for i in range(arm.split, model.n_layers)}
    MT.repair_selected(model, cache, arm, hb[:P], rows)
    others = [j for j in range(cache[arm.split]["k"].shape[1]) if j not in rows]
    for i, k0 in before.items():
        assert torch.equal(cache[i]["k"][:, others], k0[:, others])
        assert not torch.equal(cache[i]["k"][:, rows], k0[:, rows]) or i == arm.split
