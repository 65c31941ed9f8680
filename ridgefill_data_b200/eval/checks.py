"""Reproducibility gates (the role of code/qwen38-27b-kit/checks.py:83-160 CHECK-A/B, the exact-vs-exact rescore
diff of code/kva/evaluate.py:572-574 and the kit's TIMING-WARM rule).

  dump_logits / same_dump   logits rows written as raw little-endian fp32 with a sha256 sidecar; two dumps pass when
                            their bytes are identical (CHECK-A: a run against itself; CHECK-B: two builds or hosts)
  rerun_bitwise             runs a logits-producing callable twice and compares the results bit for bit
  warm_timed                device timing (CUDA events) only after `warmup` untimed calls, max over `repeats`
"""
from __future__ import annotations

import hashlib
from pathlib import Path

import numpy as np
import torch

from ..utils import atomic


def dump_logits(path, logits):
    data = logits.detach().float().cpu().contiguous().numpy().astype("<f4").tobytes()
    atomic.write_bytes(path, data)
    digest = hashlib.sha256(data).hexdigest()
    atomic.write_bytes(f"{path}.sha256", atomic.sidecar_line(path, digest).encode())
    return digest


def same_dump(a, b):
    """(identical, first differing fp32 index or None, max abs difference)."""
    x = np.frombuffer(Path(a).read_bytes(), "<f4")
    y = np.frombuffer(Path(b).read_bytes(), "<f4")
    if x.shape != y.shape:
        return False, 0, float("inf")
    diff = np.flatnonzero(x.view("<u4") != y.view("<u4"))
    if not len(diff):
        return True, None, 0.0
    return False, int(diff[0]), float(np.abs(x.astype(np.float64) - y).max())


def rerun_bitwise(fn):
    """fn() -> tensor; returns (identical, sha256 of the first run's bytes)."""
    a = fn().detach().float().cpu().contiguous()
    b = fn().detach().float().cpu().contiguous()
    same = bool(torch.equal(a.view(torch.int32), b.view(torch.int32)))
    return same, hashlib.sha256(a.numpy().tobytes()).hexdigest()


def warm_timed(fn, warmup=3, repeats=5):
    """Milliseconds per call (the max of `repeats` CUDA-event timings) after `warmup` untimed calls."""
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    times = []
    for _ in range(repeats):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        fn()
        e.record()
        torch.cuda.synchronize()
        times.append(s.elapsed_time(e))
    return max(times)
