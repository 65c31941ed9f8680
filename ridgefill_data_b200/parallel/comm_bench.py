"""Collective microbenchmarks at the 27B hybrid's tensor-parallel shapes (one rank per GPU, launched by torchrun):
NCCL vs the NVSwitch-multicast kernels for the row-parallel all-reduce (alone and after its GEMM) and for the map
fill's column all-gather. Device time with CUDA events after warm-up, max over ranks; prints one JSON line per
case on rank 0 with the achieved bus bandwidth and the fraction of the NVLink roofline.

    torchrun --nproc-per-node 8 --master-addr 127.0.0.1 -m ridgefill_data_b200.parallel.comm_bench

Roofline (per GPU, 770 GB/s per direction measured for a peer copy on this pool):
  all-reduce        NVLS: S bytes must leave and S enter each GPU once -> S / 770 GB/s
  GEMM + all-reduce max(GEMM FLOPs / 1414 TFLOP/s (measured sustained bf16), S / 770 GB/s)
  column all-gather (N - 1) / N S must enter each GPU -> that / 770 GB/s
"""
from __future__ import annotations

import argparse
import json
import os
from datetime import timedelta

import torch
import torch.distributed as dist

LINK_GBS = 770.0
GEMM_TFLOPS = 1414.3


def _time(fn, warmup=3, iters=10):
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    dist.barrier()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    ms = torch.tensor([s.elapsed_time(e) / iters], device="cuda")
    dist.all_reduce(ms, op=dist.ReduceOp.MAX)
    return float(ms)


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--rows", type=int, nargs="+", default=[16384, 4096])
    ap.add_argument("--d", type=int, default=5120)
    ap.add_argument("--k", type=int, default=3072, help="row-parallel GEMM K per rank (down_proj: 17408 / N)")
    ap.add_argument("--sweep", action="store_true", help="all-reduce only: CTA count x switch accumulation sweep")
    a = ap.parse_args(argv)
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(int(os.environ.get("LOCAL_RANK", rank)))
    dist.init_process_group("nccl", timeout=timedelta(seconds=60), device_id=torch.device("cuda", torch.cuda.current_device()))
    from ..ops import gemm as G
    from ..ops._ext import check_errors
    from .nvls import NvlsMapFill, NvlsRowParallel
    g = torch.Generator(device="cuda").manual_seed(rank)
    rp, mf = NvlsRowParallel(), NvlsMapFill()
    out = []
    d = a.d
    if a.sweep:
        for rows in a.rows:
            S = rows * d * 2
            part = rp.partial_view(rows, d)
            part.copy_(torch.randn(rows, d, device="cuda", generator=g).bfloat16())
            dst = torch.empty(rows, d, dtype=torch.bfloat16, device="cuda")
            for acc in (True, False):
                for ctas in (16, 32, 64, 148):
                    for copy in (False, True):
                        rp.max_ctas, rp.acc32 = ctas, acc
                        t = _time(lambda: rp.allreduce_(rows, d, dst if copy else None))
                        out.append(dict(case="allreduce_sweep", rows=rows, world=world, acc32=acc, ctas=ctas,
                                        copy=copy, ms=round(t, 4), frac_of_roofline=round(S / (LINK_GBS * 1e9) * 1e3 / t, 3)))
            rp.max_ctas, rp.acc32 = 0, True
            x = part.clone()
            t = _time(lambda: dist.all_reduce(x))
            out.append(dict(case="nccl_allreduce", rows=rows, world=world, ms=round(t, 4)))
        if rank == 0:
            for r in out:
                print(json.dumps(r), flush=True)
        rp.close()
        mf.close()
        dist.barrier()
        dist.destroy_process_group()
        return
    for rows in a.rows:
        S = rows * d * 2
        x = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
        y = torch.randn(rows, a.k, device="cuda", generator=g).bfloat16()
        w = (torch.randn(d, a.k, device="cuda", generator=g) * 0.02).bfloat16()
        h = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
        part = rp.partial_view(rows, d)
        part.copy_(x)
        dst = torch.empty_like(x)
        ref = x.float().clone()
        dist.all_reduce(ref)
        rp.allreduce_(rows, d, dst)
        torch.cuda.synchronize()
        check_errors()
        err = float((dst.float() - ref).abs().max() / ref.abs().max())
        t_nccl = _time(lambda: dist.all_reduce(x))
        t_nvls = _time(lambda: rp.allreduce_(rows, d, dst))
        roof = S / (LINK_GBS * 1e9) * 1e3
        bus = lambda ms: S * 2 * (world - 1) / world / (ms * 1e-3) / 1e9  # noqa: E731
        out.append(dict(case="allreduce", rows=rows, d=d, world=world, bytes=S, nccl_ms=round(t_nccl, 4),
                        nvls_ms=round(t_nvls, 4), nccl_busbw_gbs=round(bus(t_nccl), 1),
                        nvls_busbw_gbs=round(bus(t_nvls), 1), roofline_ms=round(roof, 4),
                        nvls_frac_of_roofline=round(roof / t_nvls, 3), max_rel_err_vs_nccl_fp32=err))

        def nccl_gemm_ar():
            o = G.linear(y, w, residual=h if rank == 0 else None)
            dist.all_reduce(o)
        t1 = _time(nccl_gemm_ar)
        rp.fused_gemm = False
        t2s = _time(lambda: rp(y, w, h))
        rp.fused_gemm = True
        want = rp(y, w, h).float()
        rp.fused_gemm = False
        got_split = rp(y, w, h).float()
        rp.fused_gemm = True
        torch.cuda.synchronize()
        check_errors()
        ferr = float((want - got_split).abs().max() / got_split.abs().max())
        t2 = _time(lambda: rp(y, w, h))
        rp.comm_off = True
        t2_gemm_part = _time(lambda: rp(y, w, h))
        rp.comm_off = False
        dedicated = {}
        for cc in (32, 64):
            rp.comm_ctas = cc
            dedicated[cc] = round(_time(lambda: rp(y, w, h)), 4)
            torch.cuda.synchronize()
            check_errors()
            assert torch.equal(rp(y, w, h).float(), want), "dedicated comm CTAs changed the result"
        rp.comm_ctas = 0
        overlapped = {}
        rp.fused_gemm = False
        for k in (2, 4, 8):
            rp.overlap, rp.overlap_min_rows = k, 1024
            overlapped[k] = round(_time(lambda: rp(y, w, h)), 4)
            torch.cuda.synchronize()
            check_errors()
            assert torch.equal(rp(y, w, h).float(), got_split), "the overlapped chunks changed the result"
        rp.overlap, rp.overlap_min_rows = 1, NvlsRowParallel.overlap_min_rows
        rp.fused_gemm = True
        t_gemm_symm = _time(lambda: G.linear(y, w, out=part))
        t_gemm = _time(lambda: G.linear(y, w))
        flops = 2 * rows * d * a.k
        roof2 = max(flops / (GEMM_TFLOPS * 1e12), S / (LINK_GBS * 1e9)) * 1e3
        out.append(dict(case="gemm+allreduce", rows=rows, d=d, k=a.k, world=world, gemm_ms=round(t_gemm, 4),
                        gemm_into_symmetric_ms=round(t_gemm_symm, 4), fused_comm_off_ms=round(t2_gemm_part, 4),
                        fused_dedicated_comm_ctas_ms=dedicated, overlapped_chunks_ms=overlapped,
                        nccl_ms=round(t1, 4), nvls_two_kernels_ms=round(t2s, 4), nvls_fused_ms=round(t2, 4),
                        fused_vs_two_kernel_max_rel_diff=ferr, roofline_ms=round(roof2, 4),
                        nvls_fused_frac_of_roofline=round(roof2 / t2, 3)))

        cols = d // world
        b = torch.randn(rows, d, device="cuda", generator=g).bfloat16()
        wl = (torch.randn(cols, d, device="cuda", generator=g) * 0.02).bfloat16()
        bl = torch.zeros(cols, device="cuda", dtype=torch.bfloat16)

        def nccl_fill():
            part = G.linear(b, wl, bias=bl)
            full = torch.empty(world * rows, cols, dtype=part.dtype, device=part.device)
            dist.all_gather_into_tensor(full, part)
            return full.view(world, rows, cols).permute(1, 0, 2).reshape(rows, d)
        got = mf(b, wl, bl, d).clone()
        want = nccl_fill()
        mf.fused_gemm = False
        got2 = mf(b, wl, bl, d).clone()
        mf.fused_gemm = True
        torch.cuda.synchronize()
        check_errors()
        same = bool(torch.equal(got, want)) and bool(torch.equal(got2, want))
        t3 = _time(nccl_fill)
        mf.fused_gemm = False
        t4s = _time(lambda: mf(b, wl, bl, d))
        mf.fused_gemm = True
        t4 = _time(lambda: mf(b, wl, bl, d))
        flops3 = 2 * rows * d * cols
        roof3 = max(flops3 / (GEMM_TFLOPS * 1e12), S * (world - 1) / world / (LINK_GBS * 1e9)) * 1e3
        out.append(dict(case="map_fill", rows=rows, d=d, world=world, nccl_ms=round(t3, 4),
                        nvls_two_kernels_ms=round(t4s, 4), nvls_ms=round(t4, 4),
                        bitwise_equal=same, roofline_ms=round(roof3, 4), nvls_frac_of_roofline=round(roof3 / t4, 3)))
    if rank == 0:
        for r in out:
            print(json.dumps(r), flush=True)
    rp.close()
    mf.close()
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
