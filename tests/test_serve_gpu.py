"""The serving scheduler on the B200 backend: two queued requests (exact and RidgeFill), the second prefill
interleaving decode rounds of the first, produce exactly the tokens of the engine's own prefill + greedy decode on
the same model (the kernels are deterministic, so any state clobbered by the interleaving would show)."""
import threading

import pytest
import torch

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.decode import greedy
from ridgefill_data_b200.engine.prefill import prefill
from ridgefill_data_b200.eval.data import synthetic_maps
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.config import ModelConfig, _hybrid_types
from ridgefill_data_b200.ridge.projector import Projector
from ridgefill_data_b200.serve.engine import Request, Scheduler

pytestmark = pytest.mark.gpu

HYB = ModelConfig(arch="qwen3_5", n_layers=8, hidden=512, vocab=1024, n_heads=4, n_kv=1, head_dim=256,
                  intermediate=1024, eps=1e-6, rope_theta=1e7, partial_rotary=0.25, layer_types=_hybrid_types(8),
                  gdn_nk=2, gdn_nv=4, gdn_dk=128, gdn_dv=128, conv_k=4, name="tiny-hybrid")


def test_scheduler_b200_interleaved_streams_match_engine():
    model = from_config(HYB, seed=0, device="cuda", std=0.05, backend="b200")
    W, B = synthetic_maps(HYB.hidden, 4, HYB.n_layers, "cuda")
    arms = [Arm("exact"), Arm("ridgefill", split=4, tail=256, fill="proj", projector=Projector(4, W, B))]
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, HYB.vocab, (300,), generator=g), torch.randint(0, HYB.vocab, (1100,), generator=g)]
    n_pred = [24, 6]
    want = []
    with torch.no_grad():
        for ids, arm, n in zip(prompts, arms, n_pred):
            logits, cache, _ = prefill(model, ids.cuda(), arm, keep=1)
            want.append(greedy(model, ids.cuda(), cache, logits, n, arm)[0])
    sched = Scheduler(model, interleave=1)
    got, done = [[], []], [threading.Event(), threading.Event()]
    for j in range(2):
        def emit(ev, j=j):
            got[j].append(ev)
            if ev.get("stop"):
                done[j].set()
        sched.submit(Request(ids=prompts[j], n_predict=n_pred[j], arm=arms[j], emit=emit, ignore_eos=True))
    sched.start()
    try:
        assert done[0].wait(120) and done[1].wait(120)
    finally:
        sched.stop()
    for j in range(2):
        assert "error" not in got[j][-1], got[j][-1]
        assert [t for e in got[j] if not e.get("stop") for t in e["tokens"]] == want[j]
    assert got[1][-1]["timings"]["prompt_filled_n"] == 1100 - 256
    assert sched.stats["interleaved_rounds"] > 0
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("gated", [True, False])
def test_decode_batch_b200_matches_single_steps(gated):
    """decode_batch on the sm_100a model: every row bitwise equal to that sequence's single decode step, both with
    the default tensor-core GEMV taking the 1-16 row products and with every product on the tile GEMMs (each sums a
    row the same way whatever the row count). With the CUDA-core GEMV for 1-2 rows (set_gemv_mma(False)) a single
    step sums in another order than the batched rows' tile GEMMs, so there the rows agree within bf16 rounding."""
    from ridgefill_data_b200.engine.decode import fork_cache, step
    from ridgefill_data_b200.ops._ext import ext
    cfg = HYB if gated else ModelConfig(arch="llama", n_layers=4, hidden=512, vocab=1024, n_heads=8, n_kv=2,
                                        head_dim=64, intermediate=1536, eps=1e-5, rope_theta=5e5,
                                        name="tiny-llama-gpu")
    model = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    g = torch.Generator().manual_seed(9)
    seqs = []
    with torch.no_grad():
        for n in (200, 333, 517):
            ids = torch.randint(0, cfg.vocab, (n,), generator=g).cuda()
            logits, cache, _ = prefill(model, ids, Arm("exact"), keep=1)
            seqs.append((int(logits[-1].argmax()), n, cache))
        runs = {}
        for kind in ("tile", "mma", "simt"):
            was = (ext().set_gemv(kind != "tile"), ext().set_gemv_mma(kind == "mma"),
                   ext().set_gemv_max_rows(2 if kind == "simt" else 16))
            try:
                single = [step(model, t, p, fork_cache(c), None)[-1] for t, p, c in seqs]
                batched = model.decode_batch([t for t, _, _ in seqs], [p for _, p, _ in seqs],
                                             [fork_cache(c) for _, _, c in seqs])
            finally:
                ext().set_gemv(was[0])
                ext().set_gemv_mma(was[1])
                ext().set_gemv_max_rows(was[2])
            runs[kind] = (single, batched)
    for kind in ("tile", "mma"):
        single, batched = runs[kind]
        for r in range(3):
            assert torch.equal(batched[r], single[r]), (kind, (batched[r] - single[r]).abs().max())
    single, batched = runs["simt"]
    for r in range(3):
        assert (batched[r] - single[r]).abs().max() / single[r].abs().max() < 3e-2
