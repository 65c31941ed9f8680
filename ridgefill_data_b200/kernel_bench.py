"""Single-kernel workloads at the 27B hybrid / MoE shapes, for timing (CUDA events) and for ncu captures.

    python -m ridgefill_data_b200.kernel_bench gemm              # two launches, no timing (ncu target)
    python -m ridgefill_data_b200.kernel_bench attn --time 10    # 3 warm-up launches, then 10 timed
    python -m ridgefill_data_b200.kernel_bench decode_attn --m 8 --n 16384 --time 10   # 8 sequences at 16K

Each workload is sized so its inputs exceed the 126 MB L2 where that is the point (GEMM, MoE) and stays a
few GB on the device, so an ncu capture of one launch ends in seconds. Timing prints ms per launch and the
achieved TFLOP/s and, for the decode workloads (bound by what they read), GB/s, with the algorithmic counts next
to each workload.
"""
from __future__ import annotations

import argparse
import json

import torch


def _gemm(dev, a):
    from .ops import gemm as G
    m, n, k = a.m or 8192, a.n or 16384, a.k or 5120
    x = torch.randn(m, k, device=dev).bfloat16()
    w = torch.randn(n, k, device=dev).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    return (lambda: G.linear(x, w, out=out)), dict(flops=2 * m * n * k, shape=[m, n, k])


def _attn(dev, a):
    from .ops import kernels as K
    hq, hkv, hd, n = 24, 4, a.hd or 256, a.n or 8192
    q = torch.randn(hq, n, hd, device=dev).bfloat16()
    k = torch.randn(hkv, n, hd, device=dev).bfloat16()
    v = torch.randn_like(k)
    out = torch.empty(n, hq * hd, device=dev, dtype=torch.bfloat16)
    flops = 4 * hq * hd * n * (n + 1) / 2     # causal QK^T + PV
    return (lambda: K.attention(q, k, v, n, hd ** -0.5, out, impl=a.impl)), dict(flops=flops, shape=[hq, hkv, hd, n])


def _gdn(dev, a):
    from .ops import kernels as K
    nv = a.nv or 48
    n, nk, dk, dv = a.n or 16384, max(1, nv // 3), 128, 128
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(n, C + 2 * nv, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, 4, device=dev) / 2).bfloat16()
    A_log = torch.rand(nv, device=dev) * 2.7
    dt = torch.randn(nv, device=dev) * 0.1
    q, kk, v, beta, g = K.gdn_prep(proj, C, C + nv, conv_w, None, A_log, dt, nk, nv, dk, dv)
    st = torch.zeros(nv, dk, dv, device=dev)
    out = torch.empty(n, nv * dv, device=dev, dtype=torch.bfloat16)
    fill = a.fill

    groups = a.groups or None

    def run():
        st.zero_()
        K.gdn_scan(None if fill else q, kk, v, beta, g, st, None if fill else out, groups=groups)
    # the recurrence's 4 nv dk dv MACs per token (the chunked form does more)
    return run, dict(flops=2 * 4 * nv * dk * dv * n, shape=[n, nk, nv, dk, dv], fill=fill, groups=groups or "auto")


def _moe(dev, a):
    from .ops import moe as MO
    n, E, k, d, F = a.n or 16384, 512, 10, 2048, 512
    x = torch.randn(n, d, device=dev).bfloat16()
    idx, _ = MO.router_topk(torch.randn(n, E, device=dev), E, k)
    xp, pos, seg, tiles = MO.align(idx, E, x)
    if a.down:
        y = torch.randn(n * k, F, device=dev).bfloat16()
        w = (torch.randn(E, d, F, device=dev) * 0.02).bfloat16()
        return (lambda: MO.grouped(y, w, seg, tiles, swiglu=False)), dict(flops=2 * n * k * d * F, shape=[n, E, k, d, F])
    w = (torch.randn(E, 2 * F, d, device=dev) * 0.02).bfloat16()
    return (lambda: MO.grouped(xp, w, seg, tiles, swiglu=True)), dict(flops=2 * n * k * 2 * F * d, shape=[n, E, k, d, F])


def _gemv(dev, a):
    """Decode-size products: m rows (1-16) against an n x k weight (the 27B MLP down projection by default)."""
    from .ops import gemm as G
    m, n, k = a.m or 8, a.n or 5120, a.k or 17408
    x = torch.randn(m, k, device=dev).bfloat16()
    w = (torch.randn(n, k, device=dev) * 0.02).bfloat16()
    out = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
    return (lambda: G.linear(x, w, out=out)), dict(flops=2 * m * n * k, bytes=2 * (n * k + m * k + m * n),
                                                   shape=[m, n, k])


def _decode_attn(dev, a):
    """One decode row of a 27B attention layer for m sequences at position n (contiguous caches of n + 64 rows)."""
    from .ops import kernels as K
    R, n = a.m or 8, a.n or 16384
    hq, hkv, hd, rot = 24, 4, a.hd or 256, 64
    rows = n + 64
    qkv = torch.randn(R, hq * 2 * hd + 2 * hkv * hd, device=dev).bfloat16()
    kb = [torch.randn(hkv, rows, hd, device=dev).bfloat16() for _ in range(R)]
    vb = [torch.randn(hkv, rows, hd, device=dev).bfloat16() for _ in range(R)]
    pos = torch.full((R,), n, dtype=torch.int32, device=dev)
    qn = (torch.randn(hd, device=dev) * 0.1).bfloat16()
    kn = (torch.randn(hd, device=dev) * 0.1).bfloat16()
    inv_freq = 1.0 / (1e7 ** (torch.arange(0, rot, 2, dtype=torch.float32) / rot))
    tables = K.rope_tables(inv_freq, rows, dev)
    out = torch.empty(R, hq * hd, device=dev, dtype=torch.bfloat16)
    run = lambda: K.decode_attention(qkv, pos, kb, vb, [], [rows] * R, [rows * hd] * R, 0, 0, hq, hkv,  # noqa: E731
                                     hd, True, qn, kn, 1, 1e-6, tables, rot, hd ** -0.5, out)
    return run, dict(flops=R * 4 * hq * hd * (n + 1), bytes=R * 2 * hkv * (n + 1) * hd * 2, shape=[R, n, hq, hkv, hd])


def _gdn_decode(dev, a):
    """One decode row of a 27B GDN layer (48 value heads of 128 x 128 fp32 state) for m sequences."""
    from .ops import kernels as K
    R, nv = a.m or 8, a.nv or 48
    nk, dk, dv = max(1, nv // 3), 128, 128
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(R, C + 2 * nv, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, 4, device=dev) / 2).bfloat16()
    A_log = torch.rand(nv, device=dev) * 2.7
    dt = torch.randn(nv, device=dev) * 0.1
    conv = [torch.randn(3, C, device=dev).bfloat16() for _ in range(R)]
    rec = [torch.zeros(nv, dk, dv, device=dev) for _ in range(R)]
    out = torch.empty(R, nv * dv, device=dev, dtype=torch.bfloat16)
    run = lambda: K.gdn_decode_step(proj, conv_w, A_log, dt, conv, conv, rec, rec, out, nk, nv, dk, dv,  # noqa: E731
                                    C, C + nv)
    return run, dict(flops=R * 2 * 4 * nv * dk * dv, bytes=R * nv * dk * dv * 4 * 2, shape=[R, nk, nv, dk, dv])


WORKLOADS = {"gemm": _gemm, "attn": _attn, "gdn": _gdn, "moe": _moe, "gemv": _gemv, "decode_attn": _decode_attn,
             "gdn_decode": _gdn_decode}


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("workload", choices=sorted(WORKLOADS))
    ap.add_argument("--time", type=int, default=0, help="timed launches (0: two untimed launches only)")
    ap.add_argument("--m", type=int, default=0, help="rows (gemm, gemv) or sequences (decode_attn, gdn_decode)")
    ap.add_argument("--n", type=int, default=0, help="columns (gemm, gemv), tokens, or the decode position")
    ap.add_argument("--k", type=int, default=0)
    ap.add_argument("--hd", type=int, default=0)
    ap.add_argument("--impl", default="auto", help="attention: auto | mma | tcgen05")
    ap.add_argument("--fill", action="store_true", help="gdn: state-only (fill) mode")
    ap.add_argument("--down", action="store_true", help="moe: the down projection instead of gate/up")
    ap.add_argument("--nv", type=int, default=0, help="gdn: value heads (48 = the 27B on one GPU, 6 = its TP 8 share)")
    ap.add_argument("--groups", type=int, default=0, help="gdn: chunk groups of the two-level scan (0: automatic)")
    a = ap.parse_args(argv)
    dev = torch.device("cuda", 0)
    fn, info = WORKLOADS[a.workload](dev, a)
    if a.time <= 0:
        for _ in range(2):
            fn()
        torch.cuda.synchronize()
        print(json.dumps(dict(workload=a.workload, ok=True, **info)))
        return
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dev)     # 256 MB > L2
    for _ in range(3):
        fn()
    ms = []
    for _ in range(a.time):
        flush.zero_()
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        ms.append(s.elapsed_time(e))
    ms.sort()
    med = ms[len(ms) // 2]
    rate = dict(tflops=round(info["flops"] / med / 1e9, 1))
    if "bytes" in info:
        rate["gbs"] = round(info["bytes"] / med / 1e6, 1)
    print(json.dumps(dict(workload=a.workload, ms_median=round(med, 4), ms_min=round(ms[0], 4), **rate,
                          l2="flushed (256 MB write) before each launch", **info)))


if __name__ == "__main__":
    main()
