"""Greedy decode of a fixed set of sequences as one CUDA graph per step.

Eager decode is bound by the host: a 27B step launches ~700 kernels for one sequence (~2,500 for eight), and
Python's enqueue time (19.5 ms for one sequence against an 8 ms weight-read floor on a B200) sets the step time.
DecodeGraph captures model.decode_step_dev once for the sequences it is given: that call reads every token id and
position from device buffers, writes K/V at the position read on the device and bounds attention by it, and updates
the GDN states in place. Each step then copies the tokens and positions into those buffers, replays the graph, and
does the host bookkeeping (cache lengths) the captured call cannot do.

A graph is tied to its sequences and to the room their caches had when it was captured (`headroom` more tokens);
step() refuses to go past it. The scheduler (serve/engine.py) captures a new graph when the set of running requests
changes. Models with routed experts or tensor parallelism keep the eager path (decode_step_dev raises
NotImplementedError for them).
"""
from __future__ import annotations

import torch


def _length(model, cache):
    """Tokens a sequence's cache holds (its first attention layer's rows, or a GDN layer's length)."""
    for i, t in enumerate(model.layer_types):
        if t == "attn":
            return int(cache[i].get("n", 0))
    return int(cache[0].get("len", 0))


class DecodeGraph:
    def __init__(self, model, caches, headroom, pool=None):
        if not hasattr(model, "decode_step_dev"):
            raise NotImplementedError("the model has no device-position decode step")
        self.model = model
        self.caches = list(caches)
        self.lengths = [_length(model, c) for c in self.caches]
        self.limit = [n + int(headroom) for n in self.lengths]
        dev = model.device
        # room for `headroom` more rows in every attention cache before capture: the graph keeps the buffers (or the
        # page table) it was captured with
        for c in self.caches:
            for i, t in enumerate(model.layer_types):
                if t == "attn":
                    model._kv_reserve(c[i], int(headroom), i)
        model.rope(max(self.limit) + 1)
        R = len(self.caches)
        self.tok = torch.zeros(R, dtype=torch.long, device=dev)
        self.pos = torch.zeros(R, dtype=torch.int32, device=dev)
        self._tok_host = torch.zeros(R, dtype=torch.long).pin_memory()
        self._pos_host = torch.zeros(R, dtype=torch.int32).pin_memory()
        self._copied = None          # the previous step's host -> device copies (the pinned buffers are reused)
        self.graph = torch.cuda.CUDAGraph()
        # pool: a memory pool shared with earlier graphs (torch.cuda.graph_pool_handle()), so a new capture reuses
        # their blocks instead of allocating device memory; only one of them may be replayed at a time
        # thread-local capture: other threads of the process (a server's request threads) may use CUDA meanwhile
        with torch.no_grad(), torch.cuda.graph(self.graph, pool=pool, capture_error_mode="thread_local"):
            self.logits = model.decode_step_dev(self.tok, self.pos, self.caches)

    def room(self):
        """Steps left before a sequence reaches the room its cache had at capture."""
        return min(lim - n for lim, n in zip(self.limit, self.lengths))

    def step(self, toks):
        """Advance every sequence by its token toks[r] (at its current length); returns the logits [R, V] (a buffer
        the next step overwrites)."""
        if self.room() <= 0:
            raise RuntimeError("decode graph: a sequence reached the cache room it was captured with")
        if self._copied is not None:
            self._copied.synchronize()
        self._tok_host.copy_(torch.as_tensor(list(toks), dtype=torch.long))
        self._pos_host.copy_(torch.as_tensor(self.lengths, dtype=torch.int32))
        self.tok.copy_(self._tok_host, non_blocking=True)
        self.pos.copy_(self._pos_host, non_blocking=True)
        self._copied = torch.cuda.Event()
        self._copied.record()
        self.graph.replay()
        m = self.model
        for r, c in enumerate(self.caches):
            n = self.lengths[r] + 1
            for i, t in enumerate(m.layer_types):
                if t == "attn":
                    m._commit_kv(c[i], n)
                else:
                    c[i]["len"] = c[i].get("len", 0) + 1
            self.lengths[r] = n
        return self.logits
