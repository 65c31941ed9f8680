"""The quality serving mode (engine/quality.py) on the CPU oracle: row picking (rule tokens, repeated spans of the
prompt's end, window attention mass, the share cap), the prefill against finish() with the same exact rows, the
exact fallback below min_prompt, and the server's "quality" mode against the engine."""
import threading

import pytest
import torch

from ridgefill_data_b200.engine import select as S
from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.prefill import finish, prefill, run_lower
from ridgefill_data_b200.engine.quality import QualityMode, lexical_rows, pick_rows, prefill_quality, rule_rows
from ridgefill_data_b200.eval.data import synthetic_maps, uniform_prompt
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.tiny import tiny_configs
from ridgefill_data_b200.ridge.projector import Projector

CFG = tiny_configs(8, 64)["qwen3.5-9b"]
SPLIT, TAIL = 4, 16


@pytest.fixture(scope="module")
def setup():
    model = from_config(CFG, seed=0, device="cpu", dtype=torch.float32)
    W, B = synthetic_maps(CFG.hidden, SPLIT, CFG.n_layers, "cpu", dtype=torch.float32)
    arm = Arm("quality", split=SPLIT, tail=TAIL, fill="proj", projector=Projector(SPLIT, W, B))
    return model, arm


def test_rule_and_lexical_rows():
    ids = torch.arange(100, 400)                       # no repeats
    ids[10], ids[50] = 7, 9
    mode = QualityMode(digit_ids=frozenset({7}), special_ids=frozenset({9}), lexical_span_rows=8)
    assert rule_rows(ids, 200, mode) == [10, 50]
    assert rule_rows(ids, 30, mode) == [10]
    assert lexical_rows(ids, 250, mode) == []
    ids[-30:-24] = ids[120:126]                        # the prompt's end quotes rows 120-125
    ids[-30:-24] = ids[120:126]
    got = lexical_rows(ids, 250, mode)
    assert got[0] == 120 and set(range(120, 128)) <= set(got)
    # only the latest lexical_max_occurrences matches of a run
    ids2 = torch.arange(1000, 1400)
    for s in (10, 40, 70):
        ids2[s:s + 4] = torch.tensor([1, 2, 3, 4])
    ids2[-5:-1] = torch.tensor([1, 2, 3, 4])
    rows = lexical_rows(ids2, 300, QualityMode(lexical_span_rows=4))
    assert rows == [40, 41, 42, 43, 70, 71, 72, 73]


def test_pick_rows_priorities_and_cap():
    ids = torch.arange(1000, 1100)
    ids[5] = 7
    mass = torch.zeros(100, dtype=torch.float64)
    mass[[60, 61, 62]] = torch.tensor([3.0, 2.0, 1.0], dtype=torch.float64)
    mode = QualityMode(share=0.5, qattn_share=0.02, digit_ids=frozenset({7}))
    assert pick_rows(ids, 80, mode, mass) == [5, 60, 61]
    tight = QualityMode(share=1 / 80, qattn_share=0.02, digit_ids=frozenset({7}))
    assert pick_rows(ids, 80, tight, mass) == [5]     # the cap keeps the rule rows first


def test_prefill_quality_matches_finish_with_the_same_rows(setup):
    model, arm = setup
    ids = uniform_prompt(96, CFG.vocab, seed=3)
    mode = QualityMode(min_prompt=64, qattn_share=0.1, qattn_window=16)
    logits, cache, P, rows = prefill_quality(model, ids, arm, mode, keep=2)
    assert P == 96 - TAIL and rows and len(rows) <= round(0.5 * P)
    # the same rows through finish() by hand
    layers = S.qattn_layers(model, SPLIT)
    win = {}
    hs, lower = run_lower(model, ids, [SPLIT], hook=lambda i, h: win.__setitem__(i, h[-16:].clone())
                          if i in layers else None)
    mass = S.window_mass(model, win, lower, layers, end=96)
    want = pick_rows(ids, P, mode, mass)
    assert rows == want
    ref, _, _ = finish(model, ids, hs[SPLIT], lower, arm, 2, exact_rows=rows)
    assert torch.equal(logits, ref)
    plain, _, _ = prefill(model, ids, arm, keep=2)
    assert not torch.equal(logits, plain)              # the exact rows change the answer


def test_prefill_quality_runs_exact_below_min_prompt(setup):
    model, arm = setup
    ids = uniform_prompt(80, CFG.vocab, seed=4)
    logits, _, P, rows = prefill_quality(model, ids, arm, QualityMode(min_prompt=81), keep=1)
    exact, _, _ = prefill(model, ids, Arm("exact"), keep=1)
    assert P == 0 and rows == [] and torch.allclose(logits, exact, atol=1e-5, rtol=1e-5)


def test_server_quality_mode_matches_the_engine(setup):
    pytest.importorskip("fastapi")
    from ridgefill_data_b200.engine.decode import greedy
    from ridgefill_data_b200.serve.engine import Request, Scheduler
    model, arm = setup
    mode = QualityMode(min_prompt=64, qattn_share=0.1, qattn_window=16)
    qarm = Arm("quality", split=SPLIT, tail=TAIL, fill="proj", projector=arm.projector, meta={"quality": mode})
    ids = uniform_prompt(96, CFG.vocab, seed=5)
    evs, done = [], threading.Event()

    def emit(ev):
        evs.append(ev)
        if ev.get("stop"):
            done.set()
    sched = Scheduler(model, interleave=0).start()
    try:
        sched.submit(Request(ids=ids, n_predict=4, arm=qarm, emit=emit, ignore_eos=True))
        assert done.wait(60)
    finally:
        sched.stop()
    toks = [t for e in evs if not e.get("stop") for t in e["tokens"]]
    logits, cache, P, rows = prefill_quality(model, ids, arm, mode, keep=1)
    want, _ = greedy(model, ids, cache, logits, 4, arm)
    assert toks == want
    assert evs[-1]["timings"]["prompt_filled_n"] == P - len(rows)
