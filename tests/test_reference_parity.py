"""Cross-implementation parity on the CPU: the reference's own RidgeFill (its kva package, installed unmodified in
baseline/_ref; run through kva.kva.run_lower / finish / greedy and Model.forward_exact) against this framework's
engine on the torch backend, with the same seeded weights and maps, for every tiny model family and every arm option
finish() takes. Both run bf16 weights on the CPU, so the first-token logits (and the greedy tokens that follow) must
agree bitwise. Skipped where baseline/_ref is not installed."""
import sys
from pathlib import Path

import pytest
import torch

ROOT = Path(__file__).resolve().parent.parent
sys.path.insert(0, str(ROOT / "baseline"))
import reference_arm as R  # noqa: E402

from ridgefill_data_b200.engine.arm import Arm  # noqa: E402
from ridgefill_data_b200.engine.prefill import prefill  # noqa: E402
from ridgefill_data_b200.eval.data import synthetic_maps, uniform_prompt  # noqa: E402
from ridgefill_data_b200.models.base import from_config  # noqa: E402
from ridgefill_data_b200.models.tiny import tiny_configs  # noqa: E402
from ridgefill_data_b200.ridge.projector import Projector  # noqa: E402

try:
    MODS = R.import_reference()
except R.Unavailable as e:          # a fresh checkout without the reference install
    MODS = None
    WHY = str(e)

pytestmark = pytest.mark.skipif(MODS is None, reason="baseline/_ref not installed")
CONFIGS = tiny_configs(8, 64)


@pytest.mark.parametrize("name", sorted(CONFIGS))
@pytest.mark.parametrize("fill", ["proj", "identity", "exact"])
def test_ridgefill_logits_match_reference(name, fill):
    cfg = CONFIGS[name]
    split, tail, n = 4, 16, 64
    ref_model, _, ref_step = R.build(cfg, split, tail, "cpu", MODS)
    RK = MODS[2]
    ids = uniform_prompt(n, cfg.vocab, seed=3)
    ours = from_config(cfg, seed=0, device="cpu", dtype=torch.bfloat16)
    with torch.no_grad():
        if fill == "proj":
            ref = ref_step(ids)
            W, B = synthetic_maps(cfg.hidden, split, cfg.n_layers, "cpu")
            arm = Arm("ridgefill", split=split, tail=tail, fill="proj", projector=Projector(split, W, B))
        elif fill == "identity":
            hs, lower = RK.run_lower(ref_model, ids, [split])
            ref, _, _ = RK.finish(ref_model, ids, hs[split], lower,
                                  RK.Arm("identity", split=split, tail=tail, fill="identity"), keep=1)
            arm = Arm("identity", split=split, tail=tail, fill="identity")
        else:
            ref, _ = ref_model.forward_exact(ids, keep=torch.tensor([n - 1]))     # keep: row indices
            arm = Arm("exact")
        got, _, _ = prefill(ours, ids, arm, keep=1)
    assert torch.equal(got.float(), ref.float()[-1:]), (got - ref[-1:]).abs().max()


def _arm_cases(cfg, split):
    """(case name, Arm kwargs, finish kwargs kind) for every arm option the reference's finish() takes."""
    cases = [("exact_rows", dict(fill="proj"), "rows"), ("none", dict(fill="none"), None),
             ("none+rows", dict(fill="none"), "rows"), ("f1", dict(fill="proj", f1=True), None),
             ("tail_bias", dict(fill="proj", tail_bias_from=split + 1, tail_bias_skip_last=2), None),
             ("ktail", dict(fill="proj", rescale="ktail", rescale_skip_last=2), None),
             ("vtail", dict(fill="proj", rescale="vtail"), None),
             ("refresh", dict(fill="proj", refresh=split), "refresh"),
             ("oracle", dict(fill="oracle"), "oracle"), ("kexact", dict(fill="proj", exact_part="k"), "oracle"),
             ("knorm", dict(fill="proj", rescale="knorm"), "oracle"), ("context", dict(fill="proj", context=1), "mix"),
             ("kvfold", dict(fill="kvfold") if cfg.arch == "llama" or cfg.arch == "qwen3"
              else dict(fill_by_type={"attention": "kvfold", "gdn": "proj"}), "kvfold")]
    if cfg.arch.startswith("qwen3_5"):
        cases += [("by_type", dict(fill_by_type={"attention": "identity", "gdn": "proj"}), None),
                  ("st", dict(fill="proj"), "st")]
    if cfg.swift_layers is not None:
        cases += [("swiftkv", dict(fill="swiftkv"), "swift"), ("swiftkv_native", dict(fill="swiftkv_native"), "swift")]
    return cases


CASES = [(name, case) for name in sorted(CONFIGS)
         for case, _, _ in _arm_cases(CONFIGS[name], 4)]


@pytest.mark.parametrize("name,case", CASES)
def test_arm_options_match_reference(name, case):
    """Every arm option of finish() (exact rows, skip fills, f1, tail bias, K/V tail rescales, refresh, oracle
    splices and rescales, context maps, K/V folds, per-type fills, GDN state corrections, SwiftKV): the same
    first-token logits, bitwise, from the reference's kva.finish and this engine's finish."""
    from ridgefill_data_b200.engine import prefill as EP
    from ridgefill_data_b200.ridge.projector import KVFold
    cfg = CONFIGS[name]
    split, tail, n = 4, 16, 64
    RK = MODS[2]
    ref_model, _, _ = R.build(cfg, split, tail, "cpu", MODS)
    ours = from_config(cfg, seed=0, device="cpu", dtype=torch.bfloat16)
    kw, kind = next((k, t) for c, k, t in _arm_cases(cfg, split) if c == case)
    kw = dict(kw)
    if kind == "swift":
        split = cfg.swift_layers
    W, B = synthetic_maps(cfg.hidden, split, cfg.n_layers, "cpu")
    ref_kw, our_kw = dict(kw), dict(kw)
    if kind == "mix":                                        # projector input [b, c_{S-1}]: width 2 d
        W = {i: 0.01 * torch.randn(cfg.hidden, 2 * cfg.hidden, generator=torch.Generator().manual_seed(i)).bfloat16()
             for i in range(split, cfg.n_layers)}
        B = {i: torch.zeros(cfg.hidden, dtype=torch.bfloat16) for i in W}
    meta = {"context": "1"} if kind == "mix" else None
    ref_kw["projector"], our_kw["projector"] = RK.Projector(split, W, B, meta), Projector(split, W, B, meta)
    if kind == "refresh":
        Wr, Br = synthetic_maps(cfg.hidden, split + 1, cfg.n_layers, "cpu", seed=7)
        ref_kw["refresh_projector"], our_kw["refresh_projector"] = RK.Projector(split + 1, Wr, Br), \
            Projector(split + 1, Wr, Br)
    if kind == "kvfold":
        kvd = 2 * cfg.n_kv * cfg.head_dim
        att = [i for i in range(split, cfg.n_layers) if ours.layer_types[i] == "attn"]
        Wk = {i: 0.05 * torch.randn(kvd, cfg.hidden, generator=torch.Generator().manual_seed(50 + i)).bfloat16()
              for i in att}
        Bk = {i: torch.zeros(kvd, dtype=torch.bfloat16) for i in att}
        ref_kw["kvfold"], our_kw["kvfold"] = RK.KVFold(split, Wk, Bk, cfg.n_kv, cfg.eps), \
            KVFold(split, Wk, Bk, cfg.n_kv, cfg.eps)
    if kind == "st":
        g = torch.Generator().manual_seed(1)
        st = {i: 0.01 * torch.randn(cfg.gdn_nv, cfg.gdn_dk, cfg.gdn_dv, generator=g)
              for i in range(split, cfg.n_layers) if ours.layer_types[i] == "gdn"}
        ref_kw["st"] = our_kw["st"] = st
    if "fill_by_type" in kw:
        ref_kw["fill"] = "by_type"
    t = 0 if kw.get("fill") == "swiftkv_native" else tail
    ref_arm, our_arm = RK.Arm("x", split=split, tail=t, **ref_kw), Arm("x", split=split, tail=t, **our_kw)
    ids = uniform_prompt(n, cfg.vocab, seed=3)
    fin_r, fin_o = {}, {}
    with torch.no_grad():
        if kind == "rows":
            fin_r["exact_rows"] = fin_o["exact_rows"] = [1, 5, 30]
        if kind == "oracle":
            P = n - tail
            ro, oo = {}, {}
            rh, rl = RK.run_lower(ref_model, ids, [split])
            RK.finish(ref_model, ids, rh[split], rl, RK.Arm("exact", split=split), 1, hook=RK.oracle_tap(ro, split, P))
            oh, ol = EP.run_lower(ours, ids, [split])
            EP.finish(ours, ids, oh[split], ol, Arm("exact", split=split), 1, hook=EP.oracle_tap(oo, split, P))
            fin_r["oracle"], fin_o["oracle"] = ro, oo
        mr, mo = {}, {}
        rh, rl = RK.run_lower(ref_model, ids, [split], mix=(lambda i, a: mr.__setitem__(i, a)) if kind == "mix" else None)
        oh, ol = EP.run_lower(ours, ids, [split], mix=(lambda i, a: mo.__setitem__(i, a)) if kind == "mix" else None)
        if kind == "mix":
            fin_r["mix"], fin_o["mix"] = mr, mo
        ref, rcache, _ = RK.finish(ref_model, ids, rh[split], rl, ref_arm, 1, **fin_r)
        got, ocache, _ = EP.finish(ours, ids, oh[split], ol, our_arm, 1, **fin_o)
        assert torch.equal(got.float(), ref.float()), (got - ref).abs().max()
        if case in ("exact_rows", "st", "swiftkv_native", "by_type"):              # and the decode that follows
            ref_toks, _ = RK.greedy(ref_model, ids, rcache, ref, 4, ref_arm)
            from ridgefill_data_b200.engine.decode import greedy
            our_toks, _ = greedy(ours, ids, ocache, got, 4, our_arm)
            assert our_toks == ref_toks


def test_multiturn_harness_matches_reference():
    """The multi-turn set on mk4 prompts (turn plans, follow-up turns, repair by position and by question): the same
    generated tokens every turn and the same repair rows and costs as the reference's kva/multiturn.py."""
    import random as _random
    from kva import multiturn as RMT
    from ridgefill_data_b200.eval import multiturn as MT
    from ridgefill_data_b200.eval import text as TX
    tok = TX.CharTokenizer()
    words = ["alpha", "beta", "gamma", "delta", "omega", "river", "stone", "cloud", "north", "amber"]
    r = _random.Random(9)
    corpus = {"prose": " ".join(r.choice(words) for _ in range(4000))}
    p = TX.niah_prompts(tok, "raw", variant="mk4", text_of=corpus, lengths=(700,), sources=("prose",))[0]
    cfg = CONFIGS["qwen3.5-9b"]
    ref_model, _, _ = R.build(cfg, 4, 200, "cpu", MODS)
    ours = from_config(cfg, seed=0, device="cpu", dtype=torch.bfloat16)
    assert MT.plan(tok, p, 3) == RMT.plan(tok, p, 3)
    specs = [dict(name="id", split=4, tail=200, fill="identity"),
             dict(name="id-rep", split=4, tail=200, fill="identity", repair=1.0),
             dict(name="id-repq", split=4, tail=200, fill="identity", repair=0.5, repair_by="question")]
    RK = MODS[2]
    orec, rrec = dict(runs={}), dict(runs={})
    with torch.no_grad():
        MT.run_prompt(ours, tok, p, [Arm(s["name"], split=4, tail=200, fill="identity", meta=dict(s)) for s in specs],
                      orec, "raw", (2,), 4, None, 3)
        RMT.run_prompt(ref_model, tok, p, [RK.Arm(s["name"], split=4, tail=200, fill="identity", meta=dict(s))
                                           for s in specs], rrec, "raw", (2,), 4, None, 3)
    assert orec["turns"] == rrec["turns"] and orec["runs"].keys() == rrec["runs"].keys()
    for arm, o in orec["runs"].items():
        rr = rrec["runs"][arm]
        assert [t["gen"] for t in o["turns"]] == [t["gen"] for t in rr["turns"]], arm
        assert [t["correct"] for t in o["turns"]] == [t["correct"] for t in rr["turns"]], arm
        if "repair" in o:
            for k in ("rows", "macs", "layers", "row_layers", "hs_bytes"):
                assert o["repair"][k] == rr["repair"][k], (arm, k)


def test_decode_agreement_matches_reference():
    """The decode set's forced and free passes (engine/agree.py) against the reference's kva/agree.py."""
    from kva import agree as RA
    from ridgefill_data_b200.engine import agree as AG
    from ridgefill_data_b200.engine.decode import fork_cache
    from ridgefill_data_b200.engine.prefill import prefill
    cfg = CONFIGS["qwen3.5-9b"]
    RK = MODS[2]
    ref_model, _, ref_step = R.build(cfg, 4, 16, "cpu", MODS)
    ours = from_config(cfg, seed=0, device="cpu", dtype=torch.bfloat16)
    ids = uniform_prompt(64, cfg.vocab, seed=3)
    W, B = synthetic_maps(cfg.hidden, 4, cfg.n_layers, "cpu")
    with torch.no_grad():
        oex, ocache_ex, _ = prefill(ours, ids, Arm("exact"), keep=1)
        arm = Arm("rf", split=4, tail=16, fill="proj", projector=Projector(4, W, B))
        oarm_l, oarm_c, _ = prefill(ours, ids, arm, keep=1)
        fields, (y, lp) = AG.exact_record(ours, 64, fork_cache(ocache_ex), oex, 6, Arm("exact"))
        ours_cmp = AG.compare(ours, 64, oarm_c, oarm_l, 6, arm, y, lp)
        rex, rcache_ex = ref_model.forward_exact(ids, keep=torch.tensor([63]))
        ry, rlp = RA.decode(ref_model, 64, [dict(c) for c in rcache_ex], rex, 6, RK.Arm("exact"), logprobs=True)
        rarm = RK.Arm("rf", split=4, tail=16, fill="proj", projector=RK.Projector(4, W, B))
        hs, lower = RK.run_lower(ref_model, ids, [4])
        rl, rc, _ = RK.finish(ref_model, ids, hs[4], lower, rarm, 1)
        ref_cmp = RA.compare(ref_model, 64, rc, rl, 6, rarm, ry, rlp)
    assert y == ry and fields["gen"] == ry
    for k in ("gen", "first_divergence", "frac_identical", "forced_top1_agree"):
        assert ours_cmp[k] == ref_cmp[k], k
    assert ours_cmp["kl"] == ref_cmp["kl"] and ours_cmp["kl_mean"] == ref_cmp["kl_mean"]
