"""Fit CLI: one calibration capture, ridge maps for every split (ridge/sweep.py).

  python -m ridgefill_data_b200.fit MODEL S1,S2,... [--docs 64 --doc-len 512 | --calib ids.pt |
                                    --calib-set train --tokenizer DIR] [--held 4] [--out DIR] [--backend b200|torch]
                                    [--plain] [--lambdas 1e-3,0.01,...] [--weight qfp|sqrt|rank]
                                    [--save-stats] [--from-stats S.pt] [--list-docs S.pt] [--data-parallel]

MODEL: a preset name (random-init weights of that shape, --seed) or a checkpoint directory. Calibration:
Zipf(1.1) synthetic documents (seeded), a torch file holding a list of 1-D id tensors, or the text calibration
lists (--calib-set train; held-out documents from the 'held' list) tokenised for the model. --plain fits the
uncentred form W = (X^T X + lam trace(X^T X)/d I)^-1 X^T Y without a bias. --weight: the sensitivity-weighted
fit (ridge/wfit.py; one split). --from-stats refits saved sufficient statistics without a capture;
--list-docs prints the calibration documents a statistics file was captured from. --data-parallel (under
torchrun): documents sharded over the ranks, statistics summed once at the end.
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
    ap.add_argument("--calib-set", choices=("train", "held", "sterm"))
    ap.add_argument("--tokenizer")
    ap.add_argument("--weight", choices=("qfp", "sqrt", "rank"))
    ap.add_argument("--from-stats", nargs="+")
    ap.add_argument("--list-docs")
    ap.add_argument("--data-parallel", action="store_true")
    ap.add_argument("--unitrms", action="store_true",
                    help="also fit unit-RMS targets y / rms(y) (the raw fit becomes the control: -rawctl)")
    ap.add_argument("--kvfold", action="store_true",
                    help="also fit the K/V fold: late attention layers' pre-RoPE [k | v] from b / rms(b)")
    a = ap.parse_args(argv)
    if a.list_docs:
        st = torch.load(a.list_docs, map_location="cpu", weights_only=False)
        for name in st.get("docs", []):
            print(name)
        return 0
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
    splits = [int(s) for s in a.splits.split(",")]
    lams = tuple(float(x) for x in a.lambdas.split(",")) if a.lambdas else (
        (1e-2,) if a.plain else sweep.LAMBDAS)
    if a.from_stats:                                   # refit without a capture
        for path in a.from_stats:
            st = torch.load(path, map_location="cpu", weights_only=False)
            S = int(st["split"])
            maps = sweep.fit_split(st, S, model.n_layers, lams, a.solver or "eigen", not a.plain, model.device)
            print(f"{path}: split {S}, {len(maps)} lambdas, layers {S}..{model.n_layers - 1}")
        return 0
    if a.calib:
        docs = [dict(name=f"calib{j}", ids=t) for j, t in enumerate(torch.load(a.calib))]
        held = zipf_docs(a.held, a.doc_len, vocab, seed=3) if a.held else None
    elif a.calib_set:
        from .eval.text import calib_ids, tokenizer
        tok = tokenizer(a.tokenizer or a.model)
        docs = [dict(name=d["name"], ids=torch.as_tensor(d["ids"])) for d in calib_ids(tok, a.calib_set)]
        held = ([dict(name=d["name"], ids=torch.as_tensor(d["ids"])) for d in calib_ids(tok, "held", limit=a.held)]
                if a.held else None)
    else:
        docs = zipf_docs(a.docs, a.doc_len, vocab, seed=1)
        held = zipf_docs(a.held, a.doc_len, vocab, seed=3) if a.held else None
    group = None
    if a.data_parallel:
        import torch.distributed as dist
        if not dist.is_initialized():
            dist.init_process_group("nccl" if a.device.startswith("cuda") else "gloo")
        group = dist.group.WORLD
    if a.weight:
        from .ridge import wfit
        if len(splits) != 1:
            raise SystemExit("--weight fits one split at a time")
        st = wfit.capture_weighted(model, docs, splits[0], shape=a.weight).state()
        maps = sweep.fit_split(st, splits[0], model.n_layers, lams, a.solver or "eigen", not a.plain, model.device)
        if a.out:
            from pathlib import Path
            Path(a.out).mkdir(parents=True, exist_ok=True)
            torch.save(dict(st, weight=a.weight, docs=[d["name"] for d in docs]),
                       Path(a.out) / f"{model.cfg.name or 'model'}-w{a.weight}-s{splits[0]}.pt")
        print(f"weighted ({a.weight}) split {splits[0]}: {len(maps)} lambdas fitted")
        return 0
    res = sweep.fit(model, docs, splits, lams, held=held, out_dir=a.out, solver=a.solver, center=not a.plain,
                    save_stats=a.save_stats, group=group, unitrms=a.unitrms, kvfold=a.kvfold)
    for S, r in sorted(res.items()):
        extra = "".join(f"; {k} lambda* {r[k]['lambda_star']}" for k in ("unitrms", "kvfold") if k in r)
        print(f"split {S}: lambda* {r['lambda_star']}  maps for layers {S}..{model.n_layers - 1}{extra}")
    return 0


if __name__ == "__main__":
    sys.exit(main())
