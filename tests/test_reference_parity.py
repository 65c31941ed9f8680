"""Cross-implementation parity on the CPU: the reference's own RidgeFill (its kva package, installed unmodified in
baseline/_ref; run through kva.kva.run_lower / finish and Model.forward_exact) against this framework's engine on the
torch backend, with the same seeded weights and ridge maps, for every tiny model family. Both run bf16 weights on the
CPU, so the first-token logits must agree bitwise. Skipped where baseline/_ref is not installed."""
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
