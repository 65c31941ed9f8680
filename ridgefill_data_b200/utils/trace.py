"""Stage timing: named regions timed on the device with CUDA events (wall clock on the CPU), summed per name, and
reported as the max over ranks (the slowest rank decides a collective step). The reference records per-arm wall
times and memory peaks (code/scripts/evaluate.py:594-600); this is the device-side equivalent.

    timer = StageTimer()
    with timer.stage("lower"):
        ...
    timer.report(group)      # {"lower": ms, ...} (synchronizes)
"""
from __future__ import annotations

import time
from contextlib import contextmanager

import torch


class StageTimer:
    def __init__(self, enabled=True, device=None):
        self.enabled = enabled
        self.cuda = torch.cuda.is_available() if device is None else torch.device(device).type == "cuda"
        self.events = {}      # name -> [(start, end)] CUDA events
        self.wall = {}        # name -> seconds (CPU)

    @contextmanager
    def stage(self, name):
        if not self.enabled:
            yield
            return
        if self.cuda:
            s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            s.record()
            try:
                yield
            finally:
                e.record()
                self.events.setdefault(name, []).append((s, e))
        else:
            t0 = time.perf_counter()
            try:
                yield
            finally:
                self.wall[name] = self.wall.get(name, 0.0) + time.perf_counter() - t0

    def totals(self):
        """{name: ms} on this rank."""
        if self.cuda:
            torch.cuda.synchronize()
            return {n: sum(s.elapsed_time(e) for s, e in pairs) for n, pairs in self.events.items()}
        return {n: 1e3 * v for n, v in self.wall.items()}

    def report(self, group=None):
        """{name: ms}, the max over the ranks of `group` when torch.distributed is initialised."""
        tot = self.totals()
        import torch.distributed as dist
        if dist.is_available() and dist.is_initialized() and dist.get_world_size(group) > 1:
            names = sorted(tot)
            gathered = [None] * dist.get_world_size(group)
            dist.all_gather_object(gathered, tot, group=group)
            names = sorted({n for g in gathered for n in g})
            tot = {n: max(g.get(n, 0.0) for g in gathered) for n in names}
        return tot

    def reset(self):
        self.events.clear()
        self.wall.clear()
