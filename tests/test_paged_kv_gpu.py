"""Paged K/V (models/kvpool.py) on the B200 kernels: a model serving its caches from one page pool gives bitwise the
logits of the contiguous caches, for RidgeFill prefill, exact rows and decode steps; two sequences interleaved in one
pool do not disturb each other; pages return to the pool; an exhausted pool refuses cleanly. The scheduler releases
a finished request's pages."""
import threading

import pytest
import torch

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.decode import step
from ridgefill_data_b200.engine.prefill import finish, run_lower
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.kvpool import KVPool, PoolExhausted
from ridgefill_data_b200.ridge.projector import Projector
from test_b200_model_gpu import HYB, QWEN3

pytestmark = pytest.mark.gpu


def _arm(cfg, split):
    g = torch.Generator(device="cuda").manual_seed(3)
    d = cfg.hidden
    W = {i: (torch.eye(d, device="cuda") + 0.01 * torch.randn(d, d, device="cuda", generator=g)).bfloat16()
         for i in range(split, cfg.n_layers)}
    B = {i: (0.01 * torch.randn(d, device="cuda", generator=g)).bfloat16() for i in range(split, cfg.n_layers)}
    return Arm("rf", split=split, tail=100, fill="proj", projector=Projector(split, W, B))


def _run(m, ids, arm, rows=None, decode=3):
    hs, lower = run_lower(m, ids, [arm.split])
    logits, cache, _ = finish(m, ids, hs[arm.split], lower, arm, 2, exact_rows=rows)
    outs = [logits]
    tok = int(logits[-1].argmax())
    for s in range(decode):
        lg = step(m, tok, ids.shape[0] + s, cache, arm)
        outs.append(lg)
        tok = int(lg[-1].argmax())
    return outs, cache


@pytest.mark.parametrize("cfg", [HYB, QWEN3], ids=lambda c: c.name)
def test_paged_equals_contiguous(cfg):
    m = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    split = cfg.n_layers // 2
    arm = _arm(cfg, split)
    ids = torch.randint(0, cfg.vocab, (333,), generator=torch.Generator().manual_seed(2)).cuda()
    for rows in (None, [5, 40, 200]):
        ref, _ = _run(m, ids, arm, rows)
        m.kv_pool = KVPool(m, pages=16, page_size=128)
        try:
            got, cache = _run(m, ids, arm, rows)
            for a, b in zip(got, ref):
                assert torch.equal(a, b)
            attn = m.kv_pool.layers[0]
            assert m.kv_pool.free_pages(attn) == 16 - 3        # 333 + 3 rows -> 3 pages of 128
            m.kv_pool.release(cache)
            assert m.kv_pool.free_pages(attn) == 16
        finally:
            m.kv_pool = None


def test_two_sequences_share_one_pool_and_exhaustion_refuses():
    cfg = HYB
    m = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    split = cfg.n_layers // 2
    arm = _arm(cfg, split)
    a = torch.randint(0, cfg.vocab, (300,), generator=torch.Generator().manual_seed(4)).cuda()
    b = torch.randint(0, cfg.vocab, (500,), generator=torch.Generator().manual_seed(5)).cuda()
    ref_a, _ = _run(m, a, arm)
    ref_b, _ = _run(m, b, arm)
    m.kv_pool = KVPool(m, pages=8, page_size=128)
    try:
        # interleave: prefill a, prefill b, then alternate decode steps
        ha, la = run_lower(m, a, [split])
        lga, ca, _ = finish(m, a, ha[split], la, arm, 2)
        hb, lb = run_lower(m, b, [split])
        lgb, cb, _ = finish(m, b, hb[split], lb, arm, 2)
        assert torch.equal(lga, ref_a[0]) and torch.equal(lgb, ref_b[0])
        ta, tb = int(lga[-1].argmax()), int(lgb[-1].argmax())
        for s in range(3):
            la_ = step(m, ta, 300 + s, ca, arm)
            lb_ = step(m, tb, 500 + s, cb, arm)
            assert torch.equal(la_, ref_a[s + 1]) and torch.equal(lb_, ref_b[s + 1])
            ta, tb = int(la_[-1].argmax()), int(lb_[-1].argmax())
        assert m.kv_pool.free_pages() == 8 - 3 - 4
        long = torch.randint(0, cfg.vocab, (700,), generator=torch.Generator().manual_seed(6)).cuda()
        with pytest.raises(PoolExhausted):
            run_lower(m, long, [split])
        m.kv_pool.release(ca)
        m.kv_pool.release(cb)
    finally:
        m.kv_pool = None


def test_scheduler_releases_pages():
    pytest.importorskip("fastapi")
    from ridgefill_data_b200.serve.engine import Request, Scheduler
    cfg = HYB
    m = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    arm = _arm(cfg, cfg.n_layers // 2)
    m.kv_pool = KVPool(m, pages=12, page_size=128)
    sched = Scheduler(m, interleave=1).start()
    try:
        dones = []
        for seed, n in ((7, 300), (8, 260), (9, 420)):
            ev = threading.Event()
            ids = torch.randint(0, cfg.vocab, (n,), generator=torch.Generator().manual_seed(seed))
            sched.submit(Request(ids=ids, n_predict=4, arm=arm, emit=lambda e, ev=ev: ev.set() if e.get("stop")
                                 else None, ignore_eos=True))
            dones.append(ev)
        assert all(ev.wait(120) for ev in dones)
    finally:
        sched.stop()
    assert sched.stats["errors"] == 0 and sched.stats["completed"] == 3
    assert m.kv_pool.free_pages() == 12
