"""The reference arm of bench.py: the reference's own RidgeFill prefill (its `kva` package, installed unmodified in
baseline/_ref by install_reference.py) timed on the benchmark's model and prompt.

What runs is the reference's stock path: `kva.gpu.setup()` (one card per process, deterministic cuBLAS, TF32 off),
`kva.model.model_class(dir)(dir, device, bf16)` (its Llama / Qwen3 / Qwen3.5 classes), `kva.kva.Projector` and
`kva.kva.Arm`, and per step `kva.kva.run_lower` + `kva.kva.finish` (kva.py:282-300, 319-460) ending in the
first-token logits. There are no checkpoints on the GPU boxes, so the model directory holds only config.json (the
named shape) and the weights come from the same seeded generator as this framework's benchmark model
(RandomSource: the interface of the reference's Checkpoint class, `__contains__` and `get(key, device, dtype)`); the
one substitution is that class (kva/model.py:46-68), which reads safetensors files. The ridge maps are the same
synthetic maps. Nothing of this framework's models, kernels or engine is on the timed path.

Multi-GPU: the reference has no tensor parallelism; each rank runs its own prompt on its own card (data parallel,
weak scaling), and the step time is the max over ranks.
"""
from __future__ import annotations

import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path

REF = Path(__file__).resolve().parent / "_ref"


class Unavailable(RuntimeError):
    pass


def verify_install(root=REF):
    """The installed kva package, checked file by file against the hashes recorded at install time."""
    rec_path = root / "INSTALL.json"
    if not rec_path.is_file():
        raise Unavailable(f"the reference is not installed: no {rec_path} (run baseline/install_reference.py on "
                          "the reference checkout)")
    rec = json.loads(rec_path.read_text())
    if not rec.get("files"):
        raise Unavailable("baseline/_ref holds no copied kva package")
    for rel, digest in rec["files"].items():
        f = root / "kva" / rel
        if not f.is_file() or hashlib.sha256(f.read_bytes()).hexdigest() != digest:
            raise Unavailable(f"baseline/_ref/kva/{rel} differs from the reference as installed; refusing")
    return root


def import_reference(root=REF):
    verify_install(root)
    if str(root) not in sys.path:
        sys.path.insert(0, str(root))
    from kva import gpu as RG
    from kva import kva as RK
    from kva import model as RM
    return RG, RM, RK


def build(cfg, split, tail, device, modules=None, seed=0, std=0.02, map_seed=123):
    """(model, arm, step) of the reference for a ModelConfig; step(ids) -> first-token logits [1, V] fp32."""
    import torch
    from ridgefill_data_b200.eval.data import synthetic_maps
    from ridgefill_data_b200.models.checkpoint import RandomSource
    RG, RM, RK = modules or import_reference()
    if cfg.arch == "qwen3_5_moe":
        raise Unavailable("the reference has no forward pass for the MoE hybrid (its MoE model ran only in an "
                          "external vLLM fork)")
    tmp = Path(tempfile.mkdtemp(prefix="rf_ref_model_"))
    (tmp / "config.json").write_text(json.dumps(cfg.to_hf()))
    dev = torch.device(device)

    class DeviceDrawn(RandomSource):
        """Every tensor drawn on the benchmark device (the main arm's draws, bit for bit), then moved where the
        reference asks for it (its embedding table stays on the host): no host-side generation of a 2.5 GB table."""

        def get(self, key, device="cpu", dtype=None):
            return super().get(key, dev, dtype).to(device)

    stock = RM.Checkpoint
    RM.Checkpoint = lambda path: DeviceDrawn(cfg, seed=seed, std=std)
    try:
        model = RM.model_class(tmp)(tmp, device=device, dtype=torch.bfloat16)
    finally:
        RM.Checkpoint = stock
    W, B = synthetic_maps(cfg.hidden, split, cfg.n_layers, device, seed=map_seed)
    arm = RK.Arm("ridgefill", split=split, tail=tail, fill="proj", projector=RK.Projector(split, W, B))

    def step(ids):
        hs, lower = RK.run_lower(model, ids, [split])
        logits, _, _ = RK.finish(model, ids, hs[split], lower, arm, keep=1, keep_cache=False)
        return logits

    return model, arm, step


def run(args, metric, baseline_tok_s, clock_sampler):
    """bench.py --impl reference: prints one JSON line (rank 0)."""
    rank = int(os.environ.get("RANK", "0"))
    world = int(os.environ.get("WORLD_SIZE", "1"))
    local = int(os.environ.get("LOCAL_RANK", "0"))

    def unavailable(msg):
        if rank == 0:
            print(json.dumps(dict(impl="reference", unavailable=msg)), flush=True)

    try:
        RG, RM, RK = import_reference()
    except Unavailable as e:
        return unavailable(str(e))
    # the reference refuses anything but one visible card per process (kva/gpu.py:69-104): this rank's card only
    vis = [v for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    card = vis[local] if local < len(vis) else str(local)
    os.environ["CUDA_VISIBLE_DEVICES"] = card
    smi_index = int(card) if card.isdigit() else local
    os.environ.setdefault("KVA_GPU_VENDOR", "nvidia")
    os.environ.setdefault("KVA_GPU_NAME", "B200")
    import time

    import torch
    import torch.distributed as dist
    from ridgefill_data_b200.eval.data import uniform_prompt
    from ridgefill_data_b200.models.config import PRESETS
    if world > 1:
        from datetime import timedelta
        dist.init_process_group("gloo", timeout=timedelta(seconds=900))
    try:
        device, info = RG.setup()
    except SystemExit as e:
        unavailable(f"kva.gpu.setup refused: {e}")
        if world > 1:
            dist.destroy_process_group()
        return None
    cfg = PRESETS[args.model]
    try:
        model, arm, step = build(cfg, args.split, args.tail, device, (RG, RM, RK))
    except Unavailable as e:
        unavailable(str(e))
        if world > 1:
            dist.destroy_process_group()
        return None
    ids_host = uniform_prompt(args.seq, cfg.vocab, seed=2 + rank).pin_memory()
    ids_dev = ids_host.to(device)
    tok_host = torch.empty(1, dtype=torch.long).pin_memory()

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.no_grad():
        for _ in range(args.warmup):
            step(ids_dev)
        torch.cuda.synchronize()
        sampler = clock_sampler(smi_index)
        sampler.start()
        time.sleep(0.3)
        barrier()
        torch.cuda.synchronize()
        ev = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps + 1)]
        ev[0].record()
        for s in range(args.steps):
            step(ids_dev)
            ev[s + 1].record()
        torch.cuda.synchronize()
        barrier()
        clocks = sampler.stop()
        ms = ev[0].elapsed_time(ev[args.steps]) / args.steps
        per = sorted(ev[s].elapsed_time(ev[s + 1]) for s in range(args.steps))
        p50 = (per[(args.steps - 1) // 2] + per[args.steps // 2]) / 2
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(args.steps):
            ids = ids_host.to(device, non_blocking=True)
            logits = step(ids)
            tok_host.copy_(logits[-1].argmax().view(1), non_blocking=True)
            torch.cuda.current_stream().synchronize()
        e2e_ms = (time.perf_counter() - w0) * 1e3 / args.steps
    stats = torch.tensor([ms, e2e_ms, p50], dtype=torch.float64)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
        dist.destroy_process_group()
    ms_max, e2e_max, p50_max = stats.tolist()
    tokens = args.seq * world
    value = tokens / (ms_max / 1e3)
    base = baseline_tok_s.get(args.model, {}).get(args.seq)
    if rank == 0:
        print(json.dumps(dict(
            impl="reference", metric=metric, value=round(value, 1), unit="tokens/s", n_gpus=world, steps=args.steps,
            warmup=args.warmup, ms_per_step=round(ms_max, 3), higher_is_better=True, scaling="weak",
            vs_baseline=None, vs_published_other_hw=round(value / base, 3) if base else None, dtype="bf16",
            data="synthetic (seeded uniform prompt; the same random-init weights and ridge maps as the main arm)",
            config=dict(model=args.model, global_batch=world, seq_len=args.seq, split=args.split, tail=args.tail,
                        parallelism=f"dp{world}", deterministic=info.get("deterministic"),
                        l2="inputs larger than L2 (the weights, tens of GB, are streamed every step)"),
            clocks=clocks, gpu_launches=0,
            e2e=dict(value=round(tokens / (e2e_max / 1e3), 1), unit="tokens/s", ms_per_step=round(e2e_max, 3),
                     h2d_bytes_per_step=int(ids_host.numel() * ids_host.element_size()),
                     d2h_bytes_per_step=int(tok_host.numel() * tok_host.element_size())),
            ttft_ms=round(ms_max, 3), ttft_p50_ms=round(p50_max, 3),
            path="kva.gpu.setup + kva.model.model_class + kva.kva.run_lower/finish (unmodified, baseline/_ref)")),
            flush=True)
    return None
