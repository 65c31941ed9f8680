"""Engine end to end on tiny checkpoints (fp32, CPU): exactness controls, fills, fit -> maps -> prefill,
decode agreement (code/tests/test_qwen3.py:131-170 strategy)."""
import pytest
import torch

from ridgefill_data_b200.engine.arm import Arm, exclude_scored, pop_split, rounded_tail
from ridgefill_data_b200.engine.prefill import finish, oracle_tap, prefill, run_lower
from ridgefill_data_b200.engine import agree as AG
from ridgefill_data_b200.engine.decode import fork_cache
from ridgefill_data_b200.engine.scoring import kl
from ridgefill_data_b200.eval.data import zipf_docs
from ridgefill_data_b200.models.base import load
from ridgefill_data_b200.ridge import sweep


@pytest.fixture(scope="module", params=["tiny_llama", "tiny_qwen35"])
def model(request):
    path, _ = request.getfixturevalue(request.param)
    return load(path, dtype=torch.float32)


@pytest.fixture(scope="module")
def maps(model):
    docs = zipf_docs(6, 96, 300, seed=1)
    held = zipf_docs(2, 96, 300, seed=3)
    res = sweep.fit(model, docs, [2], held=held, log=None)
    return res[2]


def _ids(n=120, seed=11):
    return torch.randint(0, 300, (n,), generator=torch.Generator().manual_seed(seed))


def test_tail_covering_prompt_is_exact_bitwise(model, maps):
    ids = _ids()
    ref, _ = model.forward_exact(ids, keep=torch.arange(110, 120))
    arm = Arm("ridgefill", split=2, tail=120, fill="proj", projector=maps["projector"])
    got, _, P = prefill(model, ids, arm, keep=10)
    assert P == 0 and torch.equal(got, ref)


def test_oracle_fill_reproduces_exact(model):
    ids = _ids()
    store = {}
    hs, lower = run_lower(model, ids, [2], hook=oracle_tap(store, 2, 80))
    # the oracle needs every late layer's true inputs
    model.forward_exact(ids, hook=oracle_tap(store, 2, 80))
    arm = Arm("oracle", split=2, tail=40, fill="oracle")
    got, _, P = finish(model, ids, hs[2], lower, arm, 5, oracle=store)
    ref, _ = model.forward_exact(ids, keep=torch.arange(115, 120))
    assert P == 80 and torch.allclose(got, ref, atol=1e-4)


def test_ridge_fill_beats_identity_and_none(model, maps):
    ids = _ids(160, seed=12)
    ref, _ = model.forward_exact(ids, keep=torch.arange(150, 160))
    out = {}
    for fill in ("proj", "identity", "none"):
        arm = Arm(fill, split=2, tail=32, fill=fill, projector=maps["projector"])
        out[fill], _, _ = prefill(model, ids, arm, keep=10)
    k = {f: float(kl(ref, v).mean()) for f, v in out.items()}
    assert 0 < k["proj"] < 1 and 0 < k["identity"] < 1
    assert maps["lambda_star"] in sweep.LAMBDAS
    assert maps["mean_read_cos"][str(maps["lambda_star"])] > maps["mean_read_cos"]["identity"]


def test_exact_rows_and_decode(model, maps):
    ids = _ids(100, seed=13)
    arm = Arm("ridgefill", split=2, tail=30, fill="proj", projector=maps["projector"])
    hs, lower = run_lower(model, ids, [2])
    l1, c1, P = finish(model, ids, hs[2], lower, arm, 1)
    l2, c2, _ = finish(model, ids, hs[2], lower, arm, 1, exact_rows=[0, 5, 17])
    assert P == 70 and not torch.equal(l1, l2)
    # every prefix row exact == exact prefill
    l3, _, _ = finish(model, ids, hs[2], lower, arm, 1, exact_rows=list(range(70)))
    ref, cref = model.forward_exact(ids, keep=torch.tensor([99]))
    assert torch.allclose(l3, ref, atol=1e-4)
    fields, (y, lp) = AG.exact_record(model, 100, fork_cache(cref), ref, 4, Arm("exact"))
    agree = AG.compare(model, 100, c1, l1, 4, arm, y, lp)
    assert len(fields["gen"]) == 4 and len(agree["kl"]) == 4 and agree["kl_mean"] >= 0
    same, _ = AG.run(model, 100, fork_cache(cref), ref, 4, Arm("exact"))
    assert same == y                                                 # the exact run is reproducible


def test_arm_helpers():
    assert pop_split(32) == 22 and pop_split(36) == 24
    assert rounded_tail(10000, 4096, 256) >= 4096
    a = exclude_scored(Arm("x", split=2, tail=64, fill="proj", rescale="ktail"), 16)
    assert a.rescale_skip_last == 16
    with pytest.raises(ValueError):
        Arm("bad", fill="nope")
