"""The benchmark plan's CPU configuration end to end (fp32): tiny Llama-style decoder (8 layers, d 256,
4 q / 2 kv heads x 64, FFN 704, eps 1e-6, theta 1e4, vocab 4096, N(0, 0.02) weights from seed 0); split after
layer 4; 256 x 256 maps for layers 5-8 fitted in fp64 with lam = 1e-2 trace(X^T X) / d (uncentred); calibration
64 x 512 Zipf(1.1) ids (seed 1); one 2048-token uniform prompt (seed 2) with a 256-token exact tail; filled
K/V and last-token logits compared against full prefill, and against the identity fill."""
import torch

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.prefill import finish, run_lower
from ridgefill_data_b200.engine.scoring import kl
from ridgefill_data_b200.eval.data import uniform_prompt, zipf_docs
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.config import PRESETS
from ridgefill_data_b200.ridge import sweep


def test_tiny_config_end_to_end():
    cfg = PRESETS["tiny-llama"]
    m = from_config(cfg, seed=0, dtype=torch.float32, lazy=False)
    docs = zipf_docs(64, 512, cfg.vocab, s=1.1, seed=1)
    res = sweep.fit(m, docs, [4], lambdas=(1e-2,), center=False, solver="eigen", log=None)
    proj = res[4]["projector"]
    assert sorted(proj.W) == [4, 5, 6, 7] and proj.W[4].shape == (256, 256)
    ids = uniform_prompt(2048, cfg.vocab, seed=2)
    ref_logits, ref_cache = m.forward_exact(ids, keep=torch.tensor([2047]))
    hs, lower = run_lower(m, ids, [4])
    out = {}
    for fill in ("proj", "identity"):
        arm = Arm(fill, split=4, tail=256, fill=fill, projector=proj.to("cpu", torch.float32))
        out[fill] = finish(m, ids, hs[4], lower, arm, 1)
    P = 2048 - 256
    errs = {}
    for fill, (logits, cache, _) in out.items():
        e = []
        for i in range(4, 8):
            for part in ("k", "v"):
                a, b = cache[i][part][:, :P], ref_cache[i][part][:, :P]
                e.append(((a - b).norm() / b.norm()).item())
        errs[fill] = sum(e) / len(e)
    k_proj = float(kl(ref_logits, out["proj"][0]).mean())
    k_id = float(kl(ref_logits, out["identity"][0]).mean())
    assert errs["proj"] < errs["identity"], errs
    assert k_proj <= k_id + 1e-6 and k_proj < 0.05, (k_proj, k_id)
