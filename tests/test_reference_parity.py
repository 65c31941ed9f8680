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
