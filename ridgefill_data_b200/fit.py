"""Fit CLI: one calibration capture, ridge maps for every split (ridge/sweep.py).

  python -m ridgefill_data_b200.fit MODEL S1,S2,... [--docs 64 --doc-len 512 | --calib ids.pt] [--held 4]
                                    [--out DIR] [--backend b200|torch] [--plain] [--lambdas 1e-3,0.01,...]

MODEL: a preset name (random-init weights of that shape, --seed) or a checkpoint directory. Calibration:
Zipf(1.1) synthetic documents (seeded) or a torch file holding a list of 1-D id tensors. --plain fits the
uncentred form W = (X^T X + lam trace(X^T X)/d I)^-1 X^T Y without a bias.
"""
import argparse
import sys

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("model")
    ap.add_argument("splits")
    ap.add_argument("--docs", type=int, default=64)
    ap.add_argument("--doc-len", type=int, default=512)
    ap.add_argument("--calib")
    ap.add_argument("--held", type=int, default=4)
    ap.add_argument("--out")
    ap.add_argument("--backend", default="b200" if torch.cuda.is_available() else "torch")
    ap.add_argument("--device", default="cuda" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--dtype", default="bf16", choices=("bf16", "fp32"))
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--plain", action="store_true")
    ap.add_argument("--lambdas")
    ap.add_argument("--solver", choices=("eigen", "cholesky"))
    ap.add_argument("--save-stats", action="store_true")
    a = ap.parse_args(argv)
    from .eval.data import zipf_docs
    from .models.base import from_config, load
    from .models.config import PRESETS
    from .ridge import sweep
    dtype = torch.bfloat16 if a.dtype == "bf16" else torch.float32
    if a.model in PRESETS:
        model = from_config(PRESETS[a.model], seed=a.seed, device=a.device, dtype=dtype, backend=a.backend)
    else:
        model = load(a.model, device=a.device, dtype=dtype, backend=a.backend)
    vocab = model.cfg.vocab
    if a.calib:
        docs = [dict(name=f"calib{j}", ids=t) for j, t in enumerate(torch.load(a.calib))]
    else:
        docs = zipf_docs(a.docs, a.doc_len, vocab, seed=1)
    held = zipf_docs(a.held, a.doc_len, vocab, seed=3) if a.held else None
    lams = tuple(float(x) for x in a.lambdas.split(",")) if a.lambdas else (
        (1e-2,) if a.plain else sweep.LAMBDAS)
    res = sweep.fit(model, docs, [int(s) for s in a.splits.split(",")], lams, held=held, out_dir=a.out,
                    solver=a.solver, center=not a.plain, save_stats=a.save_stats)
    for S, r in sorted(res.items()):
        print(f"split {S}: lambda* {r['lambda_star']}  maps for layers {S}..{model.n_layers - 1}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
