"""Completion server CLI.

    python -m ridgefill_data_b200.serve --model qwen3.8-27b --synthetic-maps --port 8080          # random-init shape
    python -m ridgefill_data_b200.serve --checkpoint DIR --maps maps.safetensors --tokenizer DIR   # a real model
    python -m torch.distributed.run --nproc-per-node 2 --master-addr 127.0.0.1 -m ridgefill_data_b200.serve ...
                                                 # tensor parallel over 2 GPUs: rank 0 serves HTTP, all ranks compute

Modes per request (`ridgefill_mode`): "on" = RidgeFill (split / tail of the maps or the flags), "quality" = RidgeFill
with exact prefix rows (engine/quality.py: digit / special tokens, repeated spans of the prompt's end, the rows the
prompt's end attends to most; exact prefill below --min-prompt), "off" = exact prefill. Decoding is always exact and
greedy.

Under torchrun with several ranks the model is sharded over them (parallel/tp.py) and served in lockstep
(serve/lockstep.py): rank 0 runs the HTTP server and the scheduler, the other ranks run every model call with it.
"""
from __future__ import annotations

import argparse
import os
import sys


def build(args):
    import torch
    from ..engine.arm import Arm
    from ..models.base import from_config, load
    from ..models.config import PRESETS
    from ..ridge.projector import Projector
    device = torch.device(args.device)
    if args.checkpoint:
        model = load(args.checkpoint, device=device, backend=args.backend)
        name = args.checkpoint
    else:
        model = from_config(PRESETS[args.model], seed=0, device=device, backend=args.backend, std=0.02)
        name = args.model
    if args.maps:
        proj = Projector.load(args.maps, device)
        split = proj.split
    elif args.synthetic_maps:
        from ..eval.data import synthetic_maps
        split = args.split
        W, B = synthetic_maps(model.hidden, split, model.n_layers, device)
        proj = Projector(split, W, B)
    else:
        raise SystemExit("give --maps FILE (a fitted map file) or --synthetic-maps (benchmark shapes only)")
    tok, eos = None, ()
    if args.tokenizer:
        from ..eval.text import eos_ids, tokenizer
        tok = tokenizer(args.tokenizer)
        eos = eos_ids(args.tokenizer, tok) if args.tokenizer != "char" else (tok.eos_token_id,)
    from ..engine.quality import QualityMode, digit_ids_of, special_ids_of
    q = QualityMode()
    qmode = QualityMode(min_prompt=getattr(args, "min_prompt", q.min_prompt),
                        share=getattr(args, "quality_share", q.share),
                        qattn_share=getattr(args, "qattn_share", q.qattn_share),
                        qattn_window=getattr(args, "qattn_window", q.qattn_window),
                        lexical=bool(getattr(args, "lexical", q.lexical)),
                        digit_ids=digit_ids_of(tok), special_ids=special_ids_of(tok))
    arms = {"off": Arm("exact"), "on": Arm("ridgefill", split=split, tail=args.tail, fill="proj", projector=proj),
            "quality": Arm("quality", split=split, tail=args.tail, fill="proj", projector=proj,
                           meta={"quality": qmode})}
    if getattr(args, "kv_pages", 0):
        from ..models.kvpool import KVPool
        model.kv_pool = KVPool(model, args.kv_pages, getattr(args, "page_size", 128))
    vocab = model.cfg.vocab
    props = dict(model=str(name), n_layers=model.n_layers, vocab=vocab, split=split, tail=args.tail,
                 backend=args.backend, interleave=args.interleave)
    return model, arms, tok, eos, props


def main(argv=None):
    ap = argparse.ArgumentParser(description="RidgeFill completion server")
    ap.add_argument("--model", default="qwen3.8-27b", help="a preset shape (random init) when no --checkpoint")
    ap.add_argument("--checkpoint")
    ap.add_argument("--backend", default="b200", choices=("b200", "torch"))
    ap.add_argument("--device", default="cuda")
    ap.add_argument("--maps")
    ap.add_argument("--synthetic-maps", action="store_true")
    ap.add_argument("--split", type=int, default=32)
    ap.add_argument("--tail", type=int, default=4096)
    ap.add_argument("--tokenizer")
    ap.add_argument("--min-prompt", type=int, default=8192, help="quality mode: shorter prompts run exact")
    ap.add_argument("--quality-share", type=float, default=0.5, help="quality mode: cap on exact prefix rows")
    ap.add_argument("--qattn-share", type=float, default=0.2, help="quality mode: rows picked by window attention")
    ap.add_argument("--qattn-window", type=int, default=64)
    ap.add_argument("--lexical", type=int, default=1, help="quality mode: repeated-span rows (1 on, 0 off)")
    ap.add_argument("--kv-pages", type=int, default=0,
                    help="serve every request from one paged K/V pool of this many pages per attention layer "
                         "(0: a contiguous cache per request)")
    ap.add_argument("--page-size", type=int, default=128, help="rows per K/V page (a multiple of 128)")
    ap.add_argument("--interleave", type=int, default=4,
                    help="decode round every this many prefill layers (0: off; the period until --decode-gap-ms has "
                         "a measured prefill cost to work from)")
    ap.add_argument("--decode-graphs", type=int, default=1,
                    help="decode rounds as CUDA-graph replays while the running requests stay the same (1 on, 0 off)")
    ap.add_argument("--decode-gap-ms", type=float, default=100.0,
                    help="target gap between a running stream's tokens while a prompt is prefilled: each prefill's "
                         "decode-round period follows its size (0: every --interleave layers)")
    ap.add_argument("--tp-comm", default="nvls", choices=("nccl", "fused", "nvls"),
                    help="tensor parallel (under torchrun with several ranks): the all-reduce / all-gather kernels")
    ap.add_argument("--max-waiting", type=int, default=0,
                    help="refuse new requests with HTTP 503 while this many wait for a prefill (0: no limit)")
    ap.add_argument("--api-key", default=os.environ.get("RF_API_KEY"),
                    help="require `Authorization: Bearer KEY` on every endpoint but /health and /metrics "
                         "(default: $RF_API_KEY; unset: open)")
    ap.add_argument("--host", default="127.0.0.1")
    ap.add_argument("--port", type=int, default=8080)
    a = ap.parse_args(argv)
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        return main_tp(a)
    from .app import Server, create_app
    from .engine import Scheduler
    model, arms, tok, eos, props = build(a)
    sched = Scheduler(model, eos=eos, interleave=a.interleave, gap_ms=a.decode_gap_ms,
                      graphs=bool(a.decode_graphs), max_waiting=a.max_waiting).start()
    try:
        Server(create_app(sched, arms, tok, props, api_key=a.api_key), a.host, a.port, log_level="info").run()
    finally:
        sched.stop()
    return 0


def main_tp(a):
    """One rank of a tensor-parallel server (torchrun): the model sharded over the ranks, rank 0 serving HTTP."""
    from datetime import timedelta

    import torch
    import torch.distributed as dist

    from ..parallel.tp import TensorParallel, shard
    from .app import Server, create_app
    from .engine import Scheduler
    from .lockstep import Lockstep, serve_worker
    if a.kv_pages:
        raise SystemExit("--kv-pages serves one GPU; a tensor-parallel server keeps a K/V cache per request")
    rank, world, local = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"]), int(os.environ.get("LOCAL_RANK", 0))
    torch.cuda.set_device(local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    control = dist.new_group(backend="gloo")          # the lockstep commands: small host objects
    a.device = f"cuda:{local}"
    model, arms, tok, eos, props = build(a)
    try:
        tp = TensorParallel(mode=a.tp_comm, fill="rows" if world >= 8 else "columns")
    except Exception as e:                            # no NVSwitch multicast here: NCCL
        if a.tp_comm != "nvls":
            raise
        print(f"nvls unavailable ({e}); using nccl", file=sys.stderr)
        tp = TensorParallel(mode="nccl", fill="rows" if world >= 8 else "columns")
    shard(model, tp)
    lockstep = Lockstep(control, arms)
    try:
        if rank == 0:
            sched = Scheduler(model, eos=eos, interleave=0, graphs=False, lockstep=lockstep,
                              max_waiting=a.max_waiting).start()
            try:
                Server(create_app(sched, arms, tok, dict(props, tensor_parallel=world), api_key=a.api_key), a.host,
                       a.port, log_level="info").run()
            finally:
                sched.stop()
        else:
            serve_worker(model, lockstep)
    finally:
        tp.close()
        dist.destroy_process_group()
    return 0


if __name__ == "__main__":
    sys.exit(main())
