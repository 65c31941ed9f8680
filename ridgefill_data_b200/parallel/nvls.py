"""Tensor-parallel collectives through NVSwitch multicast (csrc/nvls.cu), on symmetric buffers bound to one
multicast object (allocated and exchanged with torch's symmetric-memory plumbing).

NvlsRowParallel  h + sum_r y_r w_r^T: the tcgen05 GEMM writes this rank's partial (the residual added on rank 0)
                 into its symmetric buffer; one kernel then barriers the ranks, reduces its own 1/N of the rows in
                 the switch (multimem.ld_reduce, fp32 accumulation), multicasts the sums to every rank
                 (multimem.st) and barriers again. The result is a view of one of OUT_BUFFERS rotating symmetric
                 output buffers: valid until OUT_BUFFERS further reductions (the model's stable() clones a tensor
                 that must live longer, e.g. the split state).
                 With fused_gemm (the default) the GEMM and the reduction are one kernel (csrc/gemm.cu kEpiNvlsAR):
                 comm warps reduce each 128-row block as soon as every rank's epilogues have written it, while the
                 tensor cores work on later blocks.
NvlsMapFill      the column-sharded ridge-map fill: this rank's slice x_l[:, cols_r] from the GEMM (bias epilogue)
                 is multicast into every rank's copy of x_l (one store per 16 bytes, the switch fans it out), then a
                 barrier; buffers alternate by layer parity. With fused_gemm (the default) the epilogue itself
                 issues the multicast stores and the barrier closes the same kernel (csrc/gemm.cu kEpiNvlsAG).
Every wait is bounded; a timeout sets the device error word (ops._ext.check_errors raises).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops import gemm as G
from ..ops._ext import ext

SLOT_AR_IN, SLOT_AR_OUT, SLOT_AG, SLOT_BAR = 0, 1, 2, 3
OUT_BUFFERS = 4
COUNTER_AR, COUNTER_AG = 56, 57
FLAG_WORDS = 64


class NvlsUnavailable(RuntimeError):
    """The GPUs or the driver offer no multicast objects (no NVSwitch multicast)."""


def _group_name(group):
    return (group if group is not None else dist.group.WORLD).group_name


class _Symm:
    """One symmetric allocation: local tensor, every rank's unicast pointer and the multicast pointer."""

    def __init__(self, numel, dtype, group, need_multicast=True):
        import torch.distributed._symmetric_memory as symm
        name = _group_name(group)
        self.t = symm.empty(numel, dtype=dtype, device=torch.device("cuda", torch.cuda.current_device()))
        self.h = symm.rendezvous(self.t, name)
        self.ptrs = [int(p) for p in self.h.buffer_ptrs]
        self.mc = int(self.h.multicast_ptr)
        if need_multicast and self.mc == 0:
            raise NvlsUnavailable("symmetric memory has no multicast address (NVLS unsupported here)")


class _NvlsBase:
    def __init__(self, group):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        # the flag words need no multicast address, but asking for one fails here (at construction) on GPUs
        # without NVSwitch multicast, so callers can fall back before any layer runs
        self.flags = _Symm(FLAG_WORDS, torch.int32, group, need_multicast=True)
        self.flags.t.zero_()
        torch.cuda.synchronize()
        dist.barrier(group=group)
        self.flag_local = self.flags.ptrs[self.rank]
        self.epoch = 0
        self.err = ext().error_word(torch.cuda.current_device())

    def counter(self, idx):
        return self.flag_local + 4 * idx

    def close(self):
        """Drop this object's symmetric buffers (call before destroy_process_group)."""
        torch.cuda.synchronize()
        for name in ("flags", "part", "buf", "ar_flags"):
            if hasattr(self, name):
                setattr(self, name, None)
        if hasattr(self, "outs"):
            self.outs = []
        self.cap = 0


class NvlsRowParallel(_NvlsBase):
    max_ctas = 32          # the all-reduce saturates the switch with 32 CTAs of 512 threads (measured at TP 2 / 8)
    acc32 = True
    fused_gemm = True      # one kernel: GEMM tiles + per-row-block reduction by the comm warps (kEpiNvlsAR)
    comm_off = False       # diagnostics only: the fused kernel moves no data (times its GEMM part)
    comm_ctas = 0          # > 0: CTAs dedicated to the reduction (the rest compute tiles); 0: every CTA does both
    # overlap > 1: the rows go in up to `overlap` chunks; chunk j's GEMM (on all but max_ctas SMs) runs while chunk
    # j - 1's all-reduce (max_ctas CTAs) runs beside it on a second stream. Neither kernel waits on the other, so
    # they need not be co-resident; the reduction kernels of different ranks wait on each other as before.
    overlap = 1
    overlap_min_rows = 2048

    def __init__(self, group=None):
        super().__init__(group)
        self.cap = 0
        self.d = None
        self.part = None
        self.outs = []
        self.turn = 0
        self.ar_flags = None
        self.ar_epoch = 0

    def _ensure(self, rows, d):
        if rows <= self.cap and d == self.d:
            return
        cap = 1 << (max(rows, 1024) - 1).bit_length()
        self.part = _Symm(cap * d, torch.bfloat16, self.group)
        self.outs = [_Symm(cap * d, torch.bfloat16, self.group) for _ in range(OUT_BUFFERS)]
        self.cap, self.d = cap, d
        self.max_mb = cap // 128
        if self.ar_flags is None or self.ar_flags.t.numel() < self.max_mb * 8 + 64:
            self.ar_flags = _Symm(self.max_mb * 8 + 64, torch.int32, self.group, need_multicast=False)
            self.ar_flags.t.zero_()
            self.ar_epoch = 0
        self.counters = torch.zeros(self.max_mb + 1, dtype=torch.int32, device=self.part.t.device)
        torch.cuda.synchronize()
        dist.barrier(group=self.group)

    def owns(self, t):
        base = t.untyped_storage().data_ptr()
        return any(base == o.t.untyped_storage().data_ptr() for o in self.outs)

    def allreduce_(self, rows, d, dst=None):
        """Sum over ranks of this rank's partial rows (already in the symmetric partial buffer): into dst, or
        (dst None) a view of the next rotating symmetric output buffer."""
        self.epoch += 1
        chunk = -(-rows // self.world)
        r0, r1 = min(rows, self.rank * chunk), min(rows, (self.rank + 1) * chunk)
        out = self.outs[self.turn]
        self.turn = (self.turn + 1) % len(self.outs)
        ext().nvls_allreduce(self.part.mc, out.mc, out.ptrs[self.rank], dst, rows, d, r0, r1,
                             self.flag_local, self.flags.ptrs, self.rank, SLOT_AR_IN, SLOT_AR_OUT, self.epoch,
                             self.counter(COUNTER_AR), self.err, self.max_ctas, self.acc32)
        return dst if dst is not None else out.t[:rows * d].view(rows, d)

    def partial_view(self, rows, d):
        self._ensure(rows, d)
        return self.part.t[:rows * d].view(rows, d)

    def _chunks(self, rows):
        k = min(self.overlap, rows // self.overlap_min_rows) if self.overlap > 1 else 1
        if k <= 1:
            return [(0, rows)]
        step = -(-rows // k)
        step = -(-step // 128) * 128                   # whole 128-row blocks per chunk
        return [(a, min(rows, a + step)) for a in range(0, rows, step)]

    def _overlapped(self, y, w, h, chunks):
        rows, d = y.shape[0], w.shape[0]
        part = self.partial_view(rows, d)
        out = self.outs[self.turn]
        self.turn = (self.turn + 1) % len(self.outs)
        main = torch.cuda.current_stream()
        if getattr(self, "comm_stream", None) is None:
            self.comm_stream = torch.cuda.Stream()
        comm = self.comm_stream
        sms = torch.cuda.get_device_properties(torch.cuda.current_device()).multi_processor_count
        gemm_ctas = max(2, sms - self.max_ctas)
        for a, b in chunks:
            G.linear(y[a:b], w, residual=h[a:b] if self.rank == 0 else None, out=part[a:b], max_ctas=gemm_ctas)
            ev = torch.cuda.Event()
            ev.record(main)
            comm.wait_event(ev)
            m = b - a
            share = -(-m // self.world)
            r0, r1 = min(m, self.rank * share), min(m, (self.rank + 1) * share)
            off = 2 * a * d
            self.epoch += 1
            with torch.cuda.stream(comm):
                ext().nvls_allreduce(self.part.mc + off, out.mc + off, out.ptrs[self.rank] + off, None, m, d, r0, r1,
                                     self.flag_local, self.flags.ptrs, self.rank, SLOT_AR_IN, SLOT_AR_OUT, self.epoch,
                                     self.counter(COUNTER_AR), self.err, self.max_ctas, self.acc32)
        done = torch.cuda.Event()
        done.record(comm)
        main.wait_event(done)
        return out.t[:rows * d].view(rows, d)

    def __call__(self, y, w, h):
        rows, d = y.shape[0], w.shape[0]
        chunks = self._chunks(rows)
        if len(chunks) > 1:
            return self._overlapped(y, w, h, chunks)
        part = self.partial_view(rows, d)
        if not self.fused_gemm:
            G.linear(y, w, residual=h if self.rank == 0 else None, out=part)
            return self.allreduce_(rows, d)
        self.ar_epoch += 1
        out = self.outs[self.turn]
        self.turn = (self.turn + 1) % len(self.outs)
        ext().gemm_nvls_ar(y, w, h if self.rank == 0 else None, part, self.part.mc, out.mc,
                           self.ar_flags.ptrs[self.rank], self.ar_flags.ptrs, self.rank, self.ar_epoch, self.counters,
                           self.max_mb, 256 if d % 256 == 0 else 128, 0, self.err, self.comm_off, self.comm_ctas)
        return out.t[:rows * d].view(rows, d)


class NvlsMapFill(_NvlsBase):
    fused_gemm = True      # one kernel: the GEMM epilogue stores each tile through the multicast address (kEpiNvlsAG)

    def __init__(self, group=None):
        super().__init__(group)
        self.cap = 0
        self.d = None
        self.buf = None
        self.done = torch.zeros(4, dtype=torch.int32, device=torch.device("cuda", torch.cuda.current_device()))

    def _ensure(self, rows, d):
        if rows <= self.cap and d == self.d:
            return
        cap = 1 << (max(rows, 1024) - 1).bit_length()
        self.buf = _Symm(2 * cap * d, torch.bfloat16, self.group)
        self.cap, self.d = cap, d

    def __call__(self, b, w_local, bias_local, d):
        """Full x = b W^T + c [rows, d] on every rank from this rank's column slice (w_local [d / N, H])."""
        P = b.shape[0]
        self._ensure(P, d)
        self.epoch += 1
        par = self.epoch & 1
        cols = w_local.shape[0]
        off = par * self.cap * d
        if self.fused_gemm and cols % 64 == 0:
            ext().gemm_nvls_ag(b, w_local, bias_local, self.buf.mc + 2 * off, d, self.rank * cols, self.flag_local,
                               self.flags.ptrs, self.rank, self.epoch, self.done, 256 if cols % 256 == 0 else 128,
                               self.err)
        else:
            part = G.linear(b, w_local, bias=bias_local)
            ext().nvls_allgather(part, self.buf.mc + 2 * off, d, self.rank * cols, self.flag_local, self.flags.ptrs,
                                 self.rank, SLOT_AG, self.epoch, self.counter(COUNTER_AG), self.err)
        return self.buf.t[off:off + P * d].view(P, d)


class NvlsF64Reducer(_NvlsBase):
    """In-place sum over ranks of fp64 tensors (the ridge fit's sufficient statistics) through NVSwitch multicast:
    each tensor is staged in chunks of `chunk` elements into a symmetric buffer, every rank reduces its share of the
    chunk in the switch (exact fp64 adds, multimem.ld_reduce) and multicasts the sums, and the chunk is copied
    back. Replaces the NCCL all-reduce at the end of a data-parallel capture."""

    COUNTER = 58

    def __init__(self, group=None, chunk=1 << 25):
        super().__init__(group)
        self.chunk = int(chunk)
        self.buf_in = _Symm(self.chunk, torch.float64, group)
        self.buf_out = _Symm(self.chunk, torch.float64, group)
        torch.cuda.synchronize()
        dist.barrier(group=group)

    def allreduce_(self, tensors):
        for t in tensors:
            flat = t.view(-1)
            for s in range(0, flat.numel(), self.chunk):
                m = min(self.chunk, flat.numel() - s)
                self.buf_in.t[:m].copy_(flat[s:s + m])
                self.epoch += 1
                ext().nvls_allreduce_f64(self.buf_in.mc, self.buf_out.mc, m, self.flag_local, self.flags.ptrs,
                                         self.rank, SLOT_AR_IN, SLOT_AR_OUT, self.epoch, self.counter(self.COUNTER),
                                         self.err)
                flat[s:s + m].copy_(self.buf_out.t[:m])
        return tensors

    def close(self):
        super().close()
        self.buf_in = self.buf_out = None


def nccl_allreduce_reference(x, group=None):
    y = x.clone()
    dist.all_reduce(y, group=group)
    return y
