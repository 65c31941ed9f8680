"""Decode as one CUDA graph per step (engine/decode_graph.py): replaying the captured device-position step gives the
same logits and the same caches as eager decode_batch, for several sequences of different lengths at once, with
contiguous caches and with the paged K/V pool, on the hybrid (attention + GDN) and a dense attention-only model."""
import pytest
import torch

from ridgefill_data_b200.engine.decode_graph import DecodeGraph
from ridgefill_data_b200.engine.prefill import run_lower
from ridgefill_data_b200.models.base import from_config

from test_b200_model_gpu import HYB, QWEN3

pytestmark = pytest.mark.gpu


def _prefill(m, lens, seed):
    g = torch.Generator().manual_seed(seed)
    caches, last = [], []
    for n in lens:
        ids = torch.randint(0, m.cfg.vocab, (n,), generator=g).cuda()
        with torch.no_grad():
            _, cache = run_lower(m, ids, [m.n_layers], reserve=64)
        caches.append(cache)
        last.append(int(ids[-1]))
    return caches, last


@pytest.mark.parametrize("cfg", [HYB, QWEN3], ids=lambda c: c.name)
@pytest.mark.parametrize("paged", [False, True])
def test_graph_decode_matches_eager(cfg, paged):
    from ridgefill_data_b200.models.kvpool import KVPool
    from ridgefill_data_b200.ops._ext import check_errors
    lens = [130, 257, 64]
    runs = {}
    for mode in ("eager", "graph"):
        m = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
        if paged:
            m.kv_pool = KVPool(m, 64, 128)
        caches, toks = _prefill(m, lens, seed=7)
        pos = list(lens)
        out = []
        dg = DecodeGraph(m, caches, headroom=8) if mode == "graph" else None
        with torch.no_grad():
            for _ in range(6):
                lg = dg.step(toks) if dg is not None else m.decode_batch(toks, pos, caches)
                lg = lg.clone()
                out.append(lg)
                toks = [int(t) for t in lg.argmax(-1)]
                pos = [p + 1 for p in pos]
        torch.cuda.synchronize()
        check_errors()
        if dg is not None:
            assert dg.lengths == pos and dg.room() == 2
        att = [i for i, t in enumerate(m.layer_types) if t == "attn"]
        kv = []
        for c, n in zip(caches, pos):
            assert c[att[0]]["n"] == n
            if not paged:
                kv.append(torch.cat([c[i]["kbuf"][:, :n].flatten() for i in att] +
                                    [c[i]["vbuf"][:, :n].flatten() for i in att]))
        gdn = [torch.cat([c[i]["rec"].flatten() for i, t in enumerate(m.layer_types) if t != "attn"])
               if any(t != "attn" for t in m.layer_types) else None for c in caches]
        runs[mode] = (torch.stack(out), kv, gdn)
        del m, caches, dg
        torch.cuda.empty_cache()
    le, kve, ge = runs["eager"]
    lg, kvg, gg = runs["graph"]
    assert torch.equal(le, lg), float((le - lg).abs().max())
    for a, b in zip(kve, kvg):
        assert torch.equal(a, b)
    for a, b in zip(ge, gg):
        if a is not None:
            assert torch.equal(a, b)


def test_graph_decode_refuses_past_its_room():
    m = from_config(QWEN3, seed=0, device="cuda", std=0.05, backend="b200")
    caches, toks = _prefill(m, [40], seed=3)
    dg = DecodeGraph(m, caches, headroom=2)
    with torch.no_grad():
        dg.step(toks)
        dg.step(toks)
        with pytest.raises(RuntimeError, match="room"):
            dg.step(toks)


def test_scheduler_graph_rounds_match_eager_rounds():
    """The server's decode rounds as graph replays produce the same tokens as eager rounds (two requests decoding
    together, one joining after the other's prefill)."""
    import threading
    from ridgefill_data_b200.engine.arm import Arm
    from ridgefill_data_b200.serve.engine import Request, Scheduler
    results = {}
    for graphs in (False, True):
        m = from_config(HYB, seed=0, device="cuda", std=0.05, backend="b200")
        sched = Scheduler(m, interleave=2, graphs=graphs, graph_min_tokens=4)
        evs, done = {}, {}
        for name, n, seed in (("a", 90, 1), ("b", 200, 2)):
            ids = torch.randint(0, HYB.vocab, (n,), generator=torch.Generator().manual_seed(seed))
            evs[name], done[name] = [], threading.Event()

            def emit(ev, name=name):
                evs[name].append(ev)
                if ev.get("stop"):
                    done[name].set()
            sched.submit(Request(ids=ids, n_predict=14, arm=Arm("exact"), emit=emit, ignore_eos=True))
        sched.start()
        try:
            assert all(d.wait(120) for d in done.values())
        finally:
            sched.stop()
        results[graphs] = {k: [t for e in v if not e.get("stop") for t in e["tokens"]] for k, v in evs.items()}
        if graphs:
            assert sched.stats["graph_steps"] > 0, sched.stats
        del m, sched
        torch.cuda.empty_cache()
    assert results[True] == results[False]


def test_greedy_graph_decode_matches_eager_steps(monkeypatch):
    """engine.decode.greedy: a long run replays one decode graph; its tokens equal the eager steps' (RF_DECODE_GRAPH=0)
    and the caller's recurrent-state tensors are left as they were."""
    from ridgefill_data_b200.engine.arm import Arm
    from ridgefill_data_b200.engine.decode import fork_cache, greedy
    from ridgefill_data_b200.engine.prefill import prefill
    m = from_config(HYB, seed=0, device="cuda", std=0.05, backend="b200")
    ids = torch.randint(0, HYB.vocab, (300,), generator=torch.Generator().manual_seed(21)).cuda()
    arm = Arm("exact")
    with torch.no_grad():
        logits, cache, _ = prefill(m, ids, arm, keep=1)
    gdn = [i for i, t in enumerate(m.layer_types) if t != "attn"]
    before = cache[gdn[0]]["rec"].clone()
    toks = {}
    for mode in ("0", "1"):
        monkeypatch.setenv("RF_DECODE_GRAPH", mode)
        c = fork_cache(cache)
        toks[mode], _ = greedy(m, ids, c, logits, 24, arm)
    assert toks["1"] == toks["0"]
    assert torch.equal(cache[gdn[0]]["rec"], before)
