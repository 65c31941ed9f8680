"""Fused compute + collective operators over NVLink peer memory (tensor parallelism, one rank per GPU).

FusedRowParallel   h + sum_r y_r w_r^T (row-parallel o_proj / out_proj / down_proj). The tcgen05 GEMM epilogue
                   stores every partial tile straight into the receive slot of the rank that owns those rows
                   (the reduce-scatter's transfer overlaps the MMAs tile by tile); the owner sums the slots in fp32
                   with the residual (reduce_rows), then every rank pulls the reduced row blocks into its fresh
                   output (gather_rows). Flags are epoch-stamped; every wait is bounded.
FusedMapFill       the ridge-map fill under tensor parallelism: each rank holds a column slice of every map
                   W_l; the GEMM epilogue (bias added) broadcasts its column tiles into every rank's copy of
                   x_l = h_S W_l^T + c_l, so after one flag wait each rank has the full predicted layer input
                   (double-buffered by layer parity).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import check_errors, ext
from .symm import SymmetricBuffer

ARRIVE, REDUCED, GATHERED, COUNTER = 0, 8, 16, 63
FLAG_WORDS = 64


class _Flags:
    def __init__(self, group):
        self.buf = SymmetricBuffer(FLAG_WORDS * 4, group)
        self.ptrs = list(self.buf.ptrs)
        self.local = self.buf.ptrs[self.buf.rank]

    def close(self):
        self.buf.close()


class FusedRowParallel:
    def __init__(self, group=None, max_rows=16384, d=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.flags = _Flags(group)
        self.epoch = 0
        self.cap_rows = 0
        self.d = d
        self.recv = self.red = None
        self.err = ext().error_word(torch.cuda.current_device())

    def _ensure(self, rows, d):
        if rows <= self.cap_rows and d == self.d:
            return
        self._free_buffers()
        cap = max(rows, 1024)
        cap = 1 << (cap - 1).bit_length()
        chunk = -(-cap // self.world)
        self.recv = SymmetricBuffer(self.world * chunk * d * 2, self.group)
        self.red = SymmetricBuffer(chunk * d * 2, self.group)
        self.cap_rows, self.d, self.chunk_cap = cap, d, chunk

    def _free_buffers(self):
        for b in (self.recv, self.red):
            if b is not None:
                b.close()
        self.recv = self.red = None

    def __call__(self, y, w, h):
        M, d = y.shape[0], w.shape[0]
        self._ensure(M, d)
        self.epoch += 1
        e = self.epoch
        chunk = -(-M // self.world)
        slot_stride = self.chunk_cap * d
        x = ext()
        x.gemm_peer(y, w, None, list(self.recv.ptrs), 0, self.rank, chunk, slot_stride, d, 0,
                    256 if d % 256 == 0 else 128, self.err)
        x.comm_signal(self.flags.ptrs, ARRIVE + self.rank, e)
        r0, r1 = self.rank * chunk, min(M, (self.rank + 1) * chunk)
        rows = max(0, r1 - r0)
        res = h[r0:r1] if rows > 0 else None
        x.comm_reduce_rows(self.recv.ptrs[self.rank], slot_stride, res, self.red.ptrs[self.rank], rows, d,
                           self.world, self.rank, self.flags.local, ARRIVE, REDUCED, e,
                           self.flags.local + COUNTER * 4, self.flags.ptrs, self.err)
        out = torch.empty(M, d, dtype=torch.bfloat16, device=y.device)
        x.comm_gather_rows(list(self.red.ptrs), chunk, M, d, out, self.flags.local, REDUCED, e, self.err)
        return out

    def close(self):
        self._free_buffers()
        self.flags.close()


class FusedMapFill:
    def __init__(self, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.flags = _Flags(group)
        self.epoch = 0
        self.buf = None
        self.cap_rows = 0
        self.d = None
        self.err = ext().error_word(torch.cuda.current_device())

    def _ensure(self, rows, d):
        if rows <= self.cap_rows and d == self.d:
            return
        if self.buf is not None:
            self.buf.close()
        cap = 1 << (max(rows, 1024) - 1).bit_length()
        self.buf = SymmetricBuffer(2 * cap * d * 2, self.group)
        self.cap_rows, self.d = cap, d

    def __call__(self, b, w_local, bias_local, d):
        """Full x = b W^T + c [rows, d] on every rank from this rank's column slice (w_local [d / N, H])."""
        P = b.shape[0]
        self._ensure(P, d)
        self.epoch += 1
        e = self.epoch
        par = e & 1
        off = par * self.cap_rows * d * 2
        cols = w_local.shape[0]
        peers = [p + off for p in self.buf.ptrs]
        x = ext()
        x.gemm_peer(b, w_local, bias_local, peers, 1, 0, 0, 0, d, self.rank * cols,
                    256 if cols % 256 == 0 else 128, self.err)
        x.comm_signal(self.flags.ptrs, GATHERED + self.rank, e)
        x.comm_wait(self.flags.local, GATHERED, self.world, e, self.err)
        return self.buf.view((P, d), torch.bfloat16, offset=off)

    def close(self):
        if self.buf is not None:
            self.buf.close()
        self.flags.close()


def check(device=None):
    check_errors(device)
