"""Paged K/V storage for serving several sequences from one memory budget (the unified KV of a multi-user server).

Each attention layer owns a pool of `pages` pages, K and V each [pages, kv_heads, page_size, head_dim] bf16; a
sequence's cache entry for that layer holds the ids of the pages it has taken (host list `pages`, and the same ids
as an int32 device tensor `pages_dev` for the kernels) and its row count `n`. Row r of the sequence lives in page
pages[r // page_size] at row r % page_size. The B200 model writes K/V straight into the pages (head_norm_rope with a
page table) and its tcgen05 attention reads the key tiles through the page table (a 4-D TMA map over the pool; a
page holds a whole number of key tiles). Pages are taken as a sequence grows and returned by release() when it ends.

Attach with model.kv_pool = KVPool(model, pages); every cache the model creates after that is paged. The pool is
zero-filled once, so the unused rows of a sequence's last page (read by a key tile, masked in the softmax) are never
NaN. Paged caches serve prefill, exact rows and decode; the diagnostic paths that read a layer's whole K/V as one
tensor (multi-turn repair, selector signals over cached keys, impact analysis) need the contiguous caches.
"""
from __future__ import annotations

import threading

import torch


class PoolExhausted(RuntimeError):
    """No free pages left for a growing sequence."""


class KVPool:
    def __init__(self, model, pages, page_size=128):
        if page_size % 128:
            raise ValueError(f"page_size {page_size}: a multiple of 128 (the attention kernel's key tile)")
        if model.head_dim not in (128, 256):
            raise ValueError(f"paged K/V needs head_dim 128 or 256 (the tcgen05 attention), not {model.head_dim}")
        self.pages, self.page_size = int(pages), int(page_size)
        self.n_kv, self.head_dim = model.n_kv, model.head_dim
        self.layers = [i for i, t in enumerate(model.layer_types) if t == "attn"]
        shape = (self.pages, self.n_kv, self.page_size, self.head_dim)
        dev, dt = model.device, model.dtype
        self.k = {i: torch.zeros(shape, dtype=dt, device=dev) for i in self.layers}
        self.v = {i: torch.zeros(shape, dtype=dt, device=dev) for i in self.layers}
        self._free = {i: list(range(self.pages - 1, -1, -1)) for i in self.layers}
        self._owner = {i: [None] * self.pages for i in self.layers}   # who holds each page (None: free)
        self._lock = threading.Lock()
        self.owner = "default"      # the scheduler names the request a prefill or decode step works for

    @property
    def page_stride(self):
        return self.n_kv * self.page_size * self.head_dim

    def free_pages(self, layer=None):
        layer = self.layers[0] if layer is None else layer
        with self._lock:
            return len(self._free[layer])

    def bytes(self):
        return sum(t.numel() * t.element_size() for t in list(self.k.values()) + list(self.v.values()))

    def grow(self, layer, entry, rows, device):
        """Make the cache entry of `layer` hold at least `rows` rows (taking pages from the pool)."""
        have = entry.setdefault("pages", [])
        need = -(-int(rows) // self.page_size)
        if need <= len(have):
            return
        with self._lock:
            free = self._free[layer]
            if need - len(have) > len(free):
                raise PoolExhausted(f"KV pool: layer {layer} needs {need - len(have)} more pages, {len(free)} free")
            for _ in range(need - len(have)):
                p = free.pop()
                self._owner[layer][p] = self.owner
                have.append(p)
        entry["pages_dev"] = torch.tensor(have, dtype=torch.int32).to(device, non_blocking=False)

    def release(self, cache):
        """Return every page of a cache (a list of per-layer entries) to the pool. Entries copied from one another
        share their page lists; a page is returned once."""
        with self._lock:
            for i, entry in enumerate(cache):
                pages = entry.get("pages") if isinstance(entry, dict) else None
                if not pages or i not in self._free:
                    continue
                for p in pages:
                    if self._owner[i][p] is not None:
                        self._owner[i][p] = None
                        self._free[i].append(p)

    def release_owner(self, owner):
        """Return every page still held for `owner` (a request that failed before its cache was handed back)."""
        with self._lock:
            for i in self.layers:
                for p, o in enumerate(self._owner[i]):
                    if o == owner:
                        self._owner[i][p] = None
                        self._free[i].append(p)
