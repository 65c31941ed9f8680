#!/usr/bin/env python3
"""Headline benchmark: RidgeFill prefill throughput (prompt tokens / TTFT) of the Qwen3.8-27B-shaped
hybrid (64 layers, every 4th full attention, Gated DeltaNet elsewhere; d 5120) on B200.

One step = one full prompt prefill through the public API (engine.prefill.run_lower + finish: layers
< split exact on all rows, every later layer filled from its ridge map on the prefix rows, the exact
tail through the full model) ending with the first-token logits. Random-init weights and maps of the
named shapes, a seeded uniform-random prompt.

  python bench.py [--gpus N] [--steps K] [--warmup W] [--seq 16384] [--tail 4096] [--split 32]
  python -m torch.distributed.run --nproc-per-node N ... bench.py --gpus N      (one rank per GPU)
  python bench.py --impl reference                                             (the reference arm)

Multi-GPU (--parallel): tp (default) shards every layer over the N ranks (tensor parallel: one prompt per
step, strong scaling; the reported value is prompt tokens / max-over-ranks step time); dp gives each rank its
own prompt (weak scaling; value = sum of tokens / max-over-ranks step time).
Timing: W untimed warm-up steps, then K steps bracketed by a barrier and torch.cuda.synchronize(),
CUDA events on the launching stream, max over ranks. The weights (54 GB) exceed L2 (126 MB), so every
step streams its inputs from HBM. SM clocks and throttle reasons are sampled with nvidia-smi during the
timed region. e2e: the same metric timed on the host around the user-facing call, including the
host->device copy of the prompt from pinned memory and the device->host read of the first token.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

# Published RidgeFill prompt times (other hardware and engines: the 27B hybrid on a llama.cpp fork, resident maps,
# split 16, tail 4096, one A100 40 GB; Flash-Next on a vLLM fork, TP2 on AMD R9700) -> tokens / s. BASELINE.json
# publishes no number for this metric on a B200, so the JSON line's vs_baseline stays null and the ratio to these
# published A100 / R9700 figures is reported under its own name (vs_published_other_hw).
BASELINE_TOK_S = {"qwen3.8-27b": {16384: 16384 / 10.380, 32768: 32768 / 21.112, 65536: 65536 / 46.284,
                                   122880: 122880 / 100.014},
                  # Flash-Next RidgeFill TTFT medians (vLLM fork, TP2 on 2x AMD R9700): 9K / 16K / 32K
                  "flash-next": {9216: 9216 / 10.178, 16384: 16384 / 16.463, 32768: 32768 / 31.180}}
METRIC = {"qwen3.8-27b": "prefill tok/s (RidgeFill TTFT), Qwen3.8-27B-shaped hybrid",
          "flash-next": "prefill tok/s (RidgeFill TTFT), Flash-Next-shaped MoE hybrid",
          "llama-3.1-8b": "prefill tok/s (RidgeFill TTFT), Llama-3.1-8B-shaped dense model",
          "qwen3-8b": "prefill tok/s (RidgeFill TTFT), Qwen3-8B-shaped dense model"}
# the benchmark plan's configurations: 27B split 32 / tail 4096; MoE split 24 / tail 2048; Llama-8B split 16 /
# tail 4096; Qwen3-8B split 18 (of its 12 / 18 / 24 sweep) / tail 4096
DEFAULT_SPLIT_TAIL = {"qwen3.8-27b": (32, 4096), "flash-next": (24, 2048), "llama-3.1-8b": (16, 4096),
                      "qwen3-8b": (18, 4096)}


class ClockSampler:
    """nvidia-smi samples (200 ms) of SM clock, max clock and throttle reasons while running."""

    FIELDS = ("clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
              "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
              "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index = index
        self.rows = []
        self.proc = None

    def start(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.FIELDS}",
                                          "--format=csv,noheader,nounits", "-lms", "200"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
            self.thread = threading.Thread(target=self._read, daemon=True)
            self.thread.start()
        except OSError:
            self.proc = None

    def _read(self):
        for line in self.proc.stdout:
            parts = [p.strip() for p in line.split(",")]
            if len(parts) == 7:
                self.rows.append(parts)

    def stop(self):
        if self.proc is None:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["nvidia-smi unavailable"])
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except subprocess.TimeoutExpired:
            self.proc.kill()
        rows = list(self.rows)
        if not rows:
            return dict(sm_mhz=None, sm_max_mhz=None, reasons=["no samples"])
        sm = [float(r[0]) for r in rows if r[0].replace(".", "").isdigit()]
        mx = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({n for r in rows for n, v in zip(names, r[3:]) if v.lower() == "active"})
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=max(mx) if mx else None,
                    reasons=reasons, samples=len(rows))


def reference_arm(args):
    """The reference's own RidgeFill prefill on the same model, prompt and maps (baseline/reference_arm.py)."""
    sys.path.insert(0, os.path.join(ROOT, "baseline"))
    import reference_arm as R
    return R.run(args, METRIC.get(args.model, f"prefill tok/s (RidgeFill TTFT), {args.model}"), BASELINE_TOK_S,
                 ClockSampler)


def measured_peaks():
    """Roofline denominators measured on this pool (MEASURED_PEAKS.json beside this file), else the stated fallback."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            d = json.load(f)
        return dict(bf16_tflops_sustained=float(d["bf16_tflops_sustained"]), bf16_tflops=float(d["bf16_tflops"]),
                    hbm_gbs=float(d["hbm_gbs"]), source="measured")
    except (OSError, KeyError, ValueError):
        return dict(bf16_tflops_sustained=1400.0, bf16_tflops=1590.0, hbm_gbs=6650.0, source="fallback")


def timed(fn, steps, nvtx=False):
    """Run fn() `steps` times back to back with one CUDA event between steps: (mean ms, p50 ms, per-step ms).
    nvtx: each step inside an NVTX range named "step" (for a profiler's range filter)."""
    import torch
    ev = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    ev[0].record()
    for s in range(steps):
        if nvtx:
            torch.cuda.nvtx.range_push("step")
        fn()
        if nvtx:
            torch.cuda.nvtx.range_pop()
        ev[s + 1].record()
    torch.cuda.synchronize()
    per = [ev[s].elapsed_time(ev[s + 1]) for s in range(steps)]
    return ev[0].elapsed_time(ev[steps]) / steps, statistics.median(per), per


def fit_bench(args):
    """bench.py --fit: the ridge fit at a model's full shape, timed by stage (capture with the fp64 Gram sums, the
    Cholesky solves over the lambda grid, the held-out lambda choice), against the reference's recorded 27B fit
    (capture 610 s, 90-137 s of eigen-fit per split, 26 min in all for 839,652 rows and splits 16 / 24 / 32 on one
    RTX 5090). Calibration rows are seeded Zipf(1.1) documents; data parallel over the ranks under torchrun."""
    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        from datetime import timedelta
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=1800), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)
    from ridgefill_data_b200.eval.data import zipf_docs
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.config import PRESETS
    from ridgefill_data_b200.ridge import sweep
    cfg = PRESETS[args.model]
    model = from_config(cfg, seed=0, device=device, backend="b200", std=0.02)
    splits = [int(s) for s in args.fit_splits.split(",")]
    n_docs = -(-args.fit_rows // args.fit_doc)
    docs = zipf_docs(n_docs, args.fit_doc, cfg.vocab, seed=1)
    held = zipf_docs(args.fit_held, args.fit_doc, cfg.vocab, seed=3)
    timings = {}
    t0 = time.perf_counter()
    res = sweep.fit(model, docs, splits, held=held, solver="cholesky", log=None, timings=timings,
                    group=dist.group.WORLD if world > 1 else None, lean=True)
    torch.cuda.synchronize()
    total = time.perf_counter() - t0
    stats = torch.tensor([total] + [timings[k] for k in sorted(timings)], dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    vals = stats.tolist()
    if rank == 0:
        print(json.dumps(dict(
            metric="ridge fit wall time (capture + fp64 Gram sums + Cholesky solves + lambda choice)",
            value=round(vals[0], 2), unit="s", higher_is_better=False, n_gpus=world, dtype="bf16 activations, fp64 sums",
            data="synthetic (seeded Zipf(1.1) calibration documents, random-init weights of the named shape)",
            config=dict(model=args.model, rows=n_docs * args.fit_doc, docs=n_docs, doc_len=args.fit_doc,
                        splits=splits, held_docs=args.fit_held, lambdas=len(sweep.LAMBDAS),
                        parallelism=f"dp{world}"),
            stages_s={k: round(v, 2) for k, v in zip(sorted(timings), vals[1:])},
            lambda_star={str(S): r["lambda_star"] for S, r in res.items()},
            hbm_peak_gib=round(torch.cuda.max_memory_allocated(device) / 2 ** 30, 2),
            reference_recorded=dict(capture_s=610, fit_s_per_split="90-137", total_min=26, rows=839652,
                                    hardware="1x RTX 5090, PyTorch fit_sweep.py --stream"))), flush=True)
    if world > 1:
        dist.destroy_process_group()


def decode_bench(args):
    """bench.py --decode 1,3,8: the greedy decode step of R sequences on one GPU, as the server runs it (one CUDA graph
    of the device-position step, engine/decode_graph.py), after a prefill of --decode-context tokens each; device
    time per step with CUDA events, 3 warm-up steps, then --steps timed, the RidgeFill 16K step untouched. One JSON
    line per R (tokens/s = R x steps per second), with the weight-read floor of the step (the model's bytes over the
    measured copy bandwidth)."""
    import torch
    from ridgefill_data_b200.engine.decode_graph import DecodeGraph
    from ridgefill_data_b200.engine.prefill import run_lower
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.config import PRESETS
    device = torch.device("cuda", 0)
    torch.cuda.set_device(device)
    cfg = PRESETS[args.model]
    model = from_config(cfg, seed=0, device=device, backend="b200", std=0.02)
    rs = sorted({int(r) for r in args.decode.split(",") if r})
    g = torch.Generator().manual_seed(0)
    caches, toks = [], []
    with torch.no_grad():
        for _ in range(max(rs)):
            ids = torch.randint(0, cfg.vocab, (args.decode_context,), generator=g).to(device)
            caches.append(run_lower(model, ids, [model.n_layers], reserve=args.steps + 64)[1])
            toks.append(int(ids[-1]))
    torch.cuda.synchronize()
    tensors = [t for w in model.W for t in w.values() if torch.is_tensor(t) and t.is_cuda]
    if torch.is_tensor(getattr(model, "lm_head", None)):
        tensors.append(model.lm_head)
    seen, weight_bytes = set(), 0          # every weight read once per step (views of one packed tensor counted once)
    for t in tensors:
        st = t.untyped_storage()
        if st.data_ptr() not in seen:
            seen.add(st.data_ptr())
            weight_bytes += st.nbytes()
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(os.path.dirname(os.path.abspath(__file__)), "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    for R in rs:
        with torch.no_grad():
            dg = DecodeGraph(model, caches[:R], headroom=args.steps + 8)
            for _ in range(3):
                dg.step(toks[:R])
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for _ in range(args.steps):
                dg.step(toks[:R])
            e1.record()
            torch.cuda.synchronize()
            ms = e0.elapsed_time(e1) / args.steps
            del dg
        print(json.dumps(dict(metric="greedy decode tokens/s (CUDA-graph step)", value=round(R * 1e3 / ms, 1),
                              unit="tokens/s", ms_per_step=round(ms, 3), sequences=R, steps=args.steps, warmup=3,
                              n_gpus=1, dtype="bf16", data="synthetic (seeded ids; random-init weights)",
                              config=dict(model=args.model, context=args.decode_context),
                              weight_floor_ms=round(weight_bytes / (peaks.get("hbm_gbs", 6540.5) * 1e6), 2))),
              flush=True)


def build_engine(args, device):
    from ridgefill_data_b200.engine.arm import Arm
    from ridgefill_data_b200.models.base import from_config
    from ridgefill_data_b200.models.config import PRESETS
    from ridgefill_data_b200.ridge.projector import Projector
    from ridgefill_data_b200.eval.data import synthetic_maps
    cfg = PRESETS[args.model]
    model = from_config(cfg, seed=0, device=device, backend="b200", std=0.02)
    W, B = synthetic_maps(cfg.hidden, args.split, cfg.n_layers, device)   # ridge maps near the identity
    if args.maps == "streamed":                 # pinned host maps streamed through a ring of device slots
        from ridgefill_data_b200.ridge.projector import StreamedProjector
        proj = StreamedProjector(args.split, W, B, slots=args.map_slots)
        del W, B
    else:
        proj = Projector(args.split, W, B)
    arm = Arm("ridgefill", split=args.split, tail=args.tail, fill="proj", projector=proj)
    return cfg, model, arm


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="ours", choices=("ours", "reference"))
    ap.add_argument("--model", default="qwen3.8-27b")
    ap.add_argument("--seq", type=int, default=16384)
    ap.add_argument("--tail", type=int)
    ap.add_argument("--split", type=int)
    ap.add_argument("--exact", dest="exact", action="store_true", default=True,
                    help="also time full (exact) prefill at every length for the speedup (the default)")
    ap.add_argument("--no-exact", dest="exact", action="store_false")
    ap.add_argument("--sweep", default="auto",
                    help="extra prompt lengths (comma-separated, or 'none') timed after the headline length: p50 "
                         "TTFT of RidgeFill and of full prefill at each; 'auto' = 32K, 64K and 128K for the 27B hybrid")
    ap.add_argument("--sweep-steps", type=int, default=5, help="timed steps per sweep length (p50 over them)")
    ap.add_argument("--arm", default="ridgefill", choices=("ridgefill", "quality"),
                    help="ridgefill (plain fill of every late prefix row) or quality (plus exact prefix rows chosen by "
                         "the lower layers' window attention mass, --qattn-share of the prompt)")
    ap.add_argument("--qattn-share", type=float, default=0.2)
    ap.add_argument("--maps", default="resident", choices=("resident", "streamed"),
                    help="ridge maps resident in HBM, or in pinned host memory streamed per prompt through "
                         "--map-slots device buffers (copies overlap the lower layers)")
    ap.add_argument("--map-slots", type=int, default=8)
    ap.add_argument("--fit", action="store_true", help="time the ridge fit instead of the prefill (see fit_bench)")
    ap.add_argument("--decode", default="", help="time the decode step of these numbers of sequences instead of the "
                                                 "prefill, e.g. 1,3,8 (see decode_bench)")
    ap.add_argument("--decode-context", type=int, default=1024, help="prompt tokens of each decoding sequence")
    ap.add_argument("--fit-rows", type=int, default=839652)
    ap.add_argument("--fit-doc", type=int, default=8192, help="calibration document length (tokens)")
    ap.add_argument("--fit-splits", default="16,24,32")
    ap.add_argument("--fit-held", type=int, default=2)
    ap.add_argument("--parallel", default="tp", choices=("tp", "dp"))
    ap.add_argument("--stages", action="store_true",
                    help="after the timed steps, one extra step with per-stage device times (lower layers, fill, "
                         "late layers) printed to stderr, max over ranks")
    ap.add_argument("--tp-comm", default="nvls", choices=("nccl", "fused", "nvls"),
                    help="tensor-parallel collectives: nvls (fused GEMM + NVSwitch multicast kernels; falls back to "
                         "nccl where the GPUs offer no multicast), nccl (baseline), fused (peer stores)")
    ap.add_argument("--tp-fill", default="auto", choices=("auto", "columns", "rows"),
                    help="tensor-parallel map fill: columns (each rank a column slice of every map, then the fused "
                         "NVLS gather), rows (each rank a block of prefix rows through the whole map, then an "
                         "all-to-all of the heads' projections: parallel/rowfill.py), or auto: rows from 8 ranks on "
                         "(measured 144.4 vs 150.1 ms at TP 8, 16K), columns below (349.1 vs 366.0 ms at TP 2)")
    ap.add_argument("--tp-overlap", type=int, default=1,
                    help="nvls row-parallel products in this many row chunks, each chunk's GEMM beside the previous "
                         "chunk's all-reduce on a second stream (1: the fused GEMM + all-reduce kernel)")
    args = ap.parse_args()
    dsplit, dtail = DEFAULT_SPLIT_TAIL.get(args.model, (32, 4096))
    args.split = dsplit if args.split is None else args.split
    args.tail = dtail if args.tail is None else args.tail
    args.warmup = max(3, args.warmup)
    if args.impl == "reference":
        return reference_arm(args)
    if args.fit:
        return fit_bench(args)
    if args.decode:
        return decode_bench(args)

    import torch
    import torch.distributed as dist
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world > 1:
        torch.cuda.set_device(local)
        from datetime import timedelta
        dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=torch.device("cuda", local))
    device = torch.device("cuda", local)
    torch.cuda.set_device(device)

    from ridgefill_data_b200.engine.prefill import finish, run_lower
    from ridgefill_data_b200.eval.data import uniform_prompt
    from ridgefill_data_b200.ops._ext import check_errors, ext

    cfg, model, arm = build_engine(args, device)
    tp_mode = world > 1 and args.parallel == "tp"
    tp = None
    if tp_mode and args.tp_fill == "auto":
        args.tp_fill = "rows" if world >= 8 else "columns"
    if tp_mode:
        from ridgefill_data_b200.parallel.tp import TensorParallel, shard
        try:
            tp = TensorParallel(mode=args.tp_comm, fill=args.tp_fill, overlap=args.tp_overlap)
        except Exception as e:                       # no NVSwitch multicast here: the NCCL baseline
            if args.tp_comm != "nvls":
                raise
            print(f"nvls unavailable ({e}); using nccl", file=sys.stderr)
            args.tp_comm = "nccl"
            tp = TensorParallel(mode="nccl", fill=args.tp_fill)
        shard(model, tp)
    ids_host = uniform_prompt(args.seq, cfg.vocab, seed=2 + (0 if tp_mode else rank)).pin_memory()
    ids_dev = ids_host.to(device)
    tok_host = torch.empty(1, dtype=torch.long).pin_memory()

    def step(ids):
        if args.arm == "quality":
            return quality_step(ids)
        hs, lower = run_lower(model, ids, [arm.split], maps=arm.projector)
        logits, _, _ = finish(model, ids, hs[arm.split], lower, arm, keep=1, keep_cache=False)
        return logits

    from ridgefill_data_b200.engine.quality import QualityMode, prefill_quality
    qmode = QualityMode(qattn_share=args.qattn_share)

    def quality_step(ids):
        """The quality mode (engine/quality.py): exact prefix rows (rule tokens, repeated spans of the prompt's end,
        and the rows the last 64 prompt rows attend to most in the exact lower layers) recomputed exactly through
        every late layer over the filled rows. Synthetic token ids have no digit or special tokens."""
        return prefill_quality(model, ids, arm, qmode, keep=1, keep_cache=False)[0]

    def barrier():
        if world > 1:
            dist.barrier()

    with torch.no_grad():
        for _ in range(args.warmup):
            step(ids_dev)
        torch.cuda.synchronize()
        check_errors(device)

        # ---- device-timed region
        sampler = ClockSampler(local)
        sampler.start()
        time.sleep(0.3)
        barrier()
        torch.cuda.synchronize()
        launches0 = ext().launch_count()
        ms, p50_ms, step_ms = timed(lambda: step(ids_dev), args.steps, nvtx=os.environ.get("RF_NVTX") == "1")
        barrier()
        launches = ext().launch_count() - launches0
        clocks = sampler.stop()

        if args.stages:                          # diagnostics outside the timed region
            from ridgefill_data_b200.utils.trace import StageTimer
            timer = StageTimer()
            with timer.stage("lower"):
                hs, lower = run_lower(model, ids_dev, [arm.split])
            with timer.stage("late"):
                finish(model, ids_dev, hs[arm.split], lower, arm, keep=1, keep_cache=False, timer=timer)
            del hs, lower
            rep = timer.report()
            if rank == 0:
                print(json.dumps(dict(stages_ms={k: round(v, 3) for k, v in rep.items()})), file=sys.stderr)

        # ---- end to end through the public API: pinned H2D of the prompt, prefill, D2H of the first token
        barrier()
        torch.cuda.synchronize()
        w0 = time.perf_counter()
        for _ in range(args.steps):
            ids = ids_host.to(device, non_blocking=True)
            logits = step(ids)
            tok_host.copy_(logits[-1].argmax().view(1), non_blocking=True)
            torch.cuda.current_stream().synchronize()
        e2e_ms = (time.perf_counter() - w0) * 1e3 / args.steps
        barrier()

        def exact_p50(ids, steps):
            keep = torch.arange(ids.shape[0] - 1, ids.shape[0], device=device)
            model.forward_exact(ids, keep=keep)                     # warm-up at this length
            torch.cuda.synchronize()
            barrier()
            return timed(lambda: model.forward_exact(ids, keep=keep), steps)[1]

        exact_ms = exact_p50(ids_dev, max(3, min(10, args.steps // 2))) if args.exact else None

        # ---- the other prompt lengths of the metric (outside the headline timed region): p50 TTFT of RidgeFill
        # and of full prefill at each
        sweep = []
        lengths = [] if args.sweep == "none" else (
            [32768, 65536, 131072] if args.sweep == "auto" and args.model == "qwen3.8-27b" else
            [] if args.sweep == "auto" else [int(x) for x in args.sweep.split(",") if x.strip()])
        for L in [x for x in lengths if x != args.seq and x > args.tail]:
            ids_l = uniform_prompt(L, cfg.vocab, seed=2 + (0 if tp_mode else rank)).to(device)
            step(ids_l)                                               # warm-up at this length
            torch.cuda.synchronize()
            barrier()
            _, rf50, _ = timed(lambda: step(ids_l), args.sweep_steps)
            ex50 = exact_p50(ids_l, max(2, args.sweep_steps // 2 + 1)) if args.exact else 0.0
            sweep.append((L, rf50, ex50))
            del ids_l
            torch.cuda.empty_cache()
        check_errors(device)

    flat = [ms, e2e_ms, exact_ms or 0.0, p50_ms] + [v for s in sweep for v in s[1:]]
    stats = torch.tensor(flat, dtype=torch.float64, device=device)
    if world > 1:
        dist.all_reduce(stats, op=dist.ReduceOp.MAX)
    vals = stats.tolist()
    ms_max, e2e_max, exact_max, p50_max = vals[:4]
    tokens = args.seq * (1 if tp_mode else world)
    value = tokens / (ms_max / 1e3)
    e2e_value = tokens / (e2e_max / 1e3)
    base = BASELINE_TOK_S.get(args.model, {}).get(args.seq)
    from ridgefill_data_b200.eval.cost import CostModel
    cost = CostModel(cfg)
    macs = (cost.bypass(args.seq, args.split, args.tail, round(args.qattn_share * args.seq), select="qattn")
            if args.arm == "quality" else cost.ridgefill(args.seq, args.split, args.tail))
    flops = 2 * macs * (1 if tp_mode else world)
    peaks = measured_peaks()
    tflops = flops / (ms_max / 1e3) / 1e12
    by_len = {str(args.seq): dict(ttft_p50_ms=round(p50_max, 3),
                                  exact_p50_ms=round(exact_max, 3) if exact_ms else None,
                                  speedup_vs_exact=round(exact_max / p50_max, 3) if exact_ms else None)}
    for j, (L, _, _) in enumerate(sweep):
        rf50, ex50 = vals[4 + 2 * j], vals[5 + 2 * j]
        by_len[str(L)] = dict(ttft_p50_ms=round(rf50, 3), exact_p50_ms=round(ex50, 3) if args.exact else None,
                              speedup_vs_exact=round(ex50 / rf50, 3) if args.exact else None,
                              tok_s=round(L * (1 if tp_mode else world) / (rf50 / 1e3), 1))
    if rank == 0:
        line = dict(metric=METRIC.get(args.model, f"prefill tok/s (RidgeFill TTFT), {args.model}"), value=round(value, 1), unit="tokens/s", n_gpus=world, steps=args.steps,
                    warmup=args.warmup, ms_per_step=round(ms_max, 3), higher_is_better=True,
                    scaling="strong" if tp_mode else "weak", vs_baseline=None,
                    vs_published_other_hw=round(value / base, 3) if base else None, dtype="bf16",
                    data="synthetic (seeded uniform prompt; random-init weights and ridge maps of the named shapes)",
                    config=dict(model=args.model, global_batch=1 if tp_mode else world, seq_len=args.seq,
                                split=args.split, tail=args.tail, arm=args.arm, maps=args.maps,
                                **({"map_slots": args.map_slots} if args.maps == "streamed" else {}),
                                **({"qattn_share": args.qattn_share, "qattn_window": 64} if args.arm == "quality"
                                   else {}),
                                parallelism=(f"tp{world}" + ("" if args.tp_comm == "nccl" else f"-{args.tp_comm}")
                                             + ("-rowfill" if args.tp_fill == "rows" else "")
                                             + (f"-overlap{args.tp_overlap}" if args.tp_overlap > 1
                                                and args.tp_comm == "nvls" else "")) if tp_mode
                                else f"dp{world}",
                                l2="inputs larger than L2 (the weights, tens of GB, are streamed every step)"),
                    clocks=clocks, gpu_launches=int(launches),
                    e2e=dict(value=round(e2e_value, 1), unit="tokens/s", ms_per_step=round(e2e_max, 3),
                             h2d_bytes_per_step=int(ids_host.numel() * ids_host.element_size()),
                             d2h_bytes_per_step=int(tok_host.numel() * tok_host.element_size())),
                    ttft_ms=round(ms_max, 3), ttft_p50_ms=round(p50_max, 3),
                    flops_per_step=round(flops), tflops=round(tflops, 1),
                    frac_of_sustained_bf16=round(tflops / (peaks["bf16_tflops_sustained"] * world), 3),
                    peaks_source=peaks["source"], ttft_by_len=by_len,
                    hbm_peak_gib=round(torch.cuda.max_memory_allocated(device) / 2 ** 30, 2),
                    steps_ms_rank0=[round(x, 2) for x in step_ms])
        if exact_ms:
            line.update(exact_prefill_ms=round(exact_max, 3), speedup_vs_exact=round(exact_max / p50_max, 3))
        print(json.dumps(line), flush=True)
    if tp is not None:
        torch.cuda.synchronize()
        dist.barrier()
        tp.close()
    if world > 1:
        dist.destroy_process_group()


if __name__ == "__main__":
    main()
