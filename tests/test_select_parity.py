"""Row selection parity with the reference's kva/select.py (installed in baseline/_ref): for the same prompt, arms and
signal scores, choose() must pick the same exact rows, extra tail and counts for every selector kind, so bypass arms
run the same rows in either harness. The signals (window mass, predictor scores, key differences, fill deviations,
received mass, frequency tables) are supplied as seeded arrays to both."""
import sys
from pathlib import Path

import pytest
import torch

from ridgefill_data_b200.engine import select as SEL
from ridgefill_data_b200.engine.arm import Arm

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
if (REF / "kva" / "select.py").exists():
    sys.path.insert(0, str(REF))
    from kva import kva as RK
    from kva import select as RS
else:
    RS = None
pytestmark = pytest.mark.skipif(RS is None, reason="baseline/_ref not installed")

N, SPLIT, TAIL = 600, 4, 128
SPECS = [dict(kind="digits"), dict(kind="digits", budget=0.02), dict(kind="qattn", budget=0.05),
         dict(kind="qattn", budget=0.05, window="prefix"), dict(kind="pred", budget=0.05, predictor="p.st"),
         dict(kind="freq", budget=0.04, table="t.st"), dict(kind="keydiff", budget=0.05),
         dict(kind="deviation", budget=0.05), dict(kind="qfp", budget=0.05), dict(kind="band", lo=200, hi=300),
         dict(kind="start_recent", start=16, budget=0.05),
         dict(kind="blend", budget=0.06, share=0.5, first="qattn", second="pred", predictor="p.st"),
         dict(kind="blend", budget=0.06, share=0.3, first="qfp", second="freq", table="t.st"),
         dict(kind="blend", budget=0.06, share=0.5, first="qattn", second="keydiff")]


def _signals():
    g = torch.Generator().manual_seed(11)
    P = N - TAIL
    ids = torch.randint(0, 60, (N,), generator=g).tolist()
    digit_set = set(range(10))
    score = {k: torch.randn(P, generator=g, dtype=torch.float64) for k in ("mass", "pred", "keys", "dev", "recv")}
    freq = torch.randn(60, generator=g) - 5
    return ids, digit_set, score, freq


def _choose(mod, arm_cls, spec, matched=None):
    ids, digit_set, score, freq = _signals()
    arms = [arm_cls("sel", split=SPLIT, tail=TAIL, fill="identity", meta=dict(select=spec))]
    if matched:
        arms.append(arm_cls("ctl", split=SPLIT, tail=TAIL, fill="identity", meta=dict(select=dict(kind=matched,
                                                                                                 match="sel"))))
    return mod.choose(arms, N, ids, "prompt-7", digit_set,
                      mass_of=lambda split, layers, end: score["mass"],
                      pred_of=lambda split, path, P: score["pred"],
                      keys_of=lambda split, layers, P: score["keys"],
                      dev_of=lambda a, P: score["dev"],
                      freq_of=lambda path: freq, recv_of=lambda split, P: score["recv"], known=N)


@pytest.mark.parametrize("spec", SPECS, ids=lambda s: "-".join(f"{k}{v}" for k, v in s.items() if k != "kind")
                         or s["kind"])
def test_choose_matches_reference(spec):
    ours = _choose(SEL, Arm, spec)
    ref = _choose(RS, RK.Arm, spec)
    assert ours == ref


@pytest.mark.parametrize("kind", ["random", "tail_match"])
def test_matched_controls_match_reference(kind):
    spec = dict(kind="qattn", budget=0.05)
    ours = _choose(SEL, Arm, spec, matched=kind)
    ref = _choose(RS, RK.Arm, spec, matched=kind)
    assert ours == ref and ours["ctl"]["count"] == ours["sel"]["count"]
