"""Symmetric device buffers over CUDA IPC: every rank allocates the same-size buffer; the handles are exchanged
over the process group and opened, so each rank holds device pointers to every peer's buffer (NVLink P2P).

The buffers come from cudaMalloc (not the caching allocator) so an IPC handle covers exactly the buffer. They
are freed and unmapped by close() (call before destroy_process_group)."""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..ops._ext import ext

DTYPE_CODE = {torch.bfloat16: 0, torch.float32: 1, torch.int32: 2, torch.float64: 3}


class SymmetricBuffer:
    def __init__(self, nbytes, group=None):
        self.group = group
        self.rank = dist.get_rank(group)
        self.world = dist.get_world_size(group)
        self.nbytes = int(nbytes)
        self.device = torch.cuda.current_device()
        self.local = ext().ipc_malloc(self.nbytes)
        handles = [None] * self.world
        dist.all_gather_object(handles, ext().ipc_handle(self.local), group=group)
        self.ptrs = []
        self._opened = []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local)
            else:
                p = ext().ipc_open(h)
                self._opened.append(p)
                self.ptrs.append(p)
        dist.barrier(group=group)

    def view(self, shape, dtype, offset=0, rank=None):
        """A non-owning tensor over this rank's buffer (or a peer's mapping when rank is given)."""
        base = self.ptrs[self.rank if rank is None else rank] + offset
        return ext().tensor_at(base, list(shape), DTYPE_CODE[dtype], self.device)

    def close(self):
        for p in self._opened:
            ext().ipc_close(p)
        self._opened = []
        if self.local:
            ext().ipc_free(self.local)
            self.local = 0
