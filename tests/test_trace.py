"""Stage timer on the CPU (wall clock) and through the engine's fill stage."""
import time

import torch

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.prefill import finish, run_lower
from ridgefill_data_b200.models.base import load
from ridgefill_data_b200.utils.trace import StageTimer


def test_stage_timer_sums_per_name():
    t = StageTimer(device="cpu")
    for _ in range(2):
        with t.stage("a"):
            time.sleep(0.01)
    with t.stage("b"):
        pass
    rep = t.report()
    assert rep["a"] >= 20 and set(rep) == {"a", "b"}
    off = StageTimer(enabled=False, device="cpu")
    with off.stage("a"):
        pass
    assert off.report() == {}


def test_finish_times_the_fill(tiny_llama):
    path, _ = tiny_llama
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (60,), generator=torch.Generator().manual_seed(2))
    hs, lower = run_lower(m, ids, [2])
    t = StageTimer(device="cpu")
    m.fill_batch = lambda layers, b, pos, cache, projector=None: [m.fill(i, b, pos, cache) for i in layers]
    try:
        finish(m, ids, hs[2], lower, Arm("id", split=2, tail=20, fill="identity"), 1, timer=t)
    finally:
        del m.fill_batch
    assert "fill" in t.report()
