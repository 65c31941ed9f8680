"""Request scheduler for serving one model on one device.

One worker thread owns the model. Requests wait in a FIFO queue; the worker takes one at a time for prefill and
keeps every started request in the decode set until it has produced its tokens. Each decode round advances every
active request by one greedy token (an exact full-model step over its own cache); the requests of a round go
through the model together (`decode_batch`: one pass over the weights, per-sequence attention and recurrent
state), which is what makes concurrent streams cheap on a weight-bandwidth-bound decode. A long prefill does not stall
the running streams: the engine's layer loop calls `tick(i)` before every layer, and every k layers the worker
runs one decode round for the other requests, so their inter-token gap during a prefill is bounded by k layers of
that prefill instead of all of it (the quantity the fixed-arrival mix measures). k is `interleave`, or with
`gap_ms` it is sized to the prefill: gap_ms / (rows x the per-row, per-layer cost learned from large prefills that
ran alone), so a short prompt runs uninterrupted and a long one yields about every gap_ms. Under
tensor parallelism the layer outputs live in rotating collective buffers, so interleaving is off there; a
tensor-parallel model is served by this scheduler on rank 0 with `lockstep` (serve/lockstep.py), which has every
other rank make the same model calls.

Events are plain dicts handed to the request's `emit` callback from the worker thread, in the field layout of the
llama.cpp server's `/completion` stream (kept alike so the 27B kit's clients read them unchanged):
  token:  {"tokens": [id], "content": str, "tokens_predicted": k, "stop": false}
  final:  {"tokens": [], "content": "", "stop": true, "stop_type": "eos" | "limit", "tokens_predicted": k,
           "tokens_evaluated": n_prompt, "truncated": false, "timings": {prompt_n, prompt_ms, prompt_per_second,
           predicted_n, predicted_ms, predicted_per_second, prompt_filled_n, cache_n, ridgefill: {...}}}
  error:  {"error": message, "stop": true}
"""
from __future__ import annotations

import collections
import itertools
import logging
import queue
import threading
import time
from dataclasses import dataclass, field

import torch

from ..engine import decode as D
from ..engine.arm import Arm
from ..engine.prefill import finish, run_lower


_log = logging.getLogger("ridgefill_data_b200.serve")

LATENCY_WINDOW = 10000      # latency samples kept per /metrics summary
MAX_SCORED_ROWS = 4096      # prompt positions a request can have scored (prompt_logprobs): the last ones


def prefill_request(model, ids, arm, n_predict, tick=None, keep=1):
    """The model work of one request's prefill (every rank of a lockstep group runs it alike): (logits [k, V] of the
    last k <= keep prompt rows, the last one giving the first token; cache; prompt rows filled from the maps). A
    RidgeFill arm has logits only for its tail rows (the rows run through every layer), so k is at most the tail."""
    quality = arm.meta.get("quality")
    n = int(ids.numel())
    if quality is not None:
        from ..engine.quality import prefill_quality
        if n >= quality.min_prompt and arm.split is not None:
            keep = max(1, min(keep, n - arm.prefix_len(n)))
        logits, cache, P, rows = prefill_quality(model, ids, arm, quality, keep=keep, reserve=n_predict + 64,
                                                 tick=tick)
        return logits, cache, int(P) - len(rows)
    if arm.fill == "exact" or arm.split is None:
        hs, cache = run_lower(model, ids, [model.n_layers], tick=tick, reserve=n_predict + 64)
        return model.logits(hs[model.n_layers][-keep:]), cache, 0
    keep = max(1, min(keep, n - arm.prefix_len(n)))
    hs, lower = run_lower(model, ids, [arm.split], tick=tick, reserve=n_predict + 64, maps=arm.projector)
    logits, cache, P = finish(model, ids, hs[arm.split], lower, arm, keep=keep, tick=tick)
    return logits, cache, int(P)


def score_prompt(logits, ids, top=0, chunk=256):
    """Teacher-forced scores of the prompt positions that `logits` (the last k rows' logits) predict: row j scores
    prompt token n - k + 1 + j. Returns (first scored position, [(logprob, rank, [(id, logprob)] * top)]); rank is
    1 + the number of tokens the row gives a higher log-prob (the vLLM prompt_logprobs fields)."""
    n, k = int(ids.numel()), int(logits.shape[0])
    m = k - 1
    out = []
    tgt_all = ids[n - m:].to(logits.device)
    for c0 in range(0, m, chunk):
        lp = logits[c0:min(m, c0 + chunk)].float().log_softmax(-1)
        tgt = tgt_all[c0:c0 + lp.shape[0]]
        tl = lp.gather(1, tgt[:, None])[:, 0]
        rank = (lp > tl[:, None]).sum(-1) + 1
        alts = lp.topk(top, -1) if top > 0 else None
        tl, rank = tl.tolist(), rank.tolist()
        av = (alts.values.tolist(), alts.indices.tolist()) if alts is not None else None
        for j in range(lp.shape[0]):
            out.append((tl[j], int(rank[j]),
                        list(zip(av[1][j], av[0][j])) if av is not None else []))
    return n - m, out


def score_next(logits, top=0):
    """(greedy token, its log-prob, [(id, logprob)] * top) of the last row: the first generated token's score."""
    lp = logits[-1].float().log_softmax(-1)
    tok = int(lp.argmax())
    alts = lp.topk(top) if top > 0 else None
    return (tok, float(lp[tok]),
            list(zip(alts.indices.tolist(), alts.values.tolist())) if alts is not None else [])


class ServerBusy(RuntimeError):
    """The waiting queue is full (max_waiting): the client should retry later."""


@dataclass
class Request:
    ids: torch.Tensor                       # [n] int64 prompt ids (host)
    n_predict: int
    arm: Arm                                # the prefill arm (exact, or a RidgeFill arm)
    emit: object                            # callable(event dict), called from the worker thread
    ignore_eos: bool = False
    rid: str = ""
    detok: object = None                    # callable([id]) -> str, optional
    t_submit: float = 0.0
    # runtime state
    cache: list = None
    position: int = 0
    tok: int = -1
    produced: list = field(default_factory=list)
    t_prefill0: float = 0.0
    t_first: float = 0.0
    t_last: float = 0.0
    filled: int = 0
    cancelled: bool = False
    prompt_logprobs: int = -1               # >= 0: score the prompt (that many top alternatives per position)
    stop_ids: frozenset = frozenset()       # token ids that end this request (beside the server's eos ids)
    prompt_scores: object = None            # (first scored position, [(logprob, rank, alternatives)])
    next_score: object = None               # (first generated token, its logprob, alternatives) when scored


class Scheduler:
    def __init__(self, model, eos=(), interleave=4, max_active=64, max_batch=32, sync=None, gap_ms=0.0,
                 sample_rows=4096, graphs=True, graph_min_tokens=8, lockstep=None, max_waiting=0):
        self.model = model
        # lockstep: a serve.lockstep.Lockstep when the model is sharded over ranks (this scheduler runs on rank 0
        # and every model call is mirrored on the others)
        self.lockstep = lockstep
        self.eos = frozenset(int(e) for e in eos)
        self.interleave = int(interleave)
        # gap_ms > 0: the decode-round period of a prefill follows its size, so that the running streams wait about
        # gap_ms between tokens: period = gap_ms / (rows x the measured ms per row and layer of prefills of at least
        # sample_rows rows that ran with no decode round inside; shorter ones are dominated by fixed costs). Until
        # one such prefill is measured, `interleave` layers.
        self.gap_ms = float(gap_ms)
        self.sample_rows = int(sample_rows)
        self._row_layer_ms = None
        # decode rounds as CUDA-graph replays (engine/decode_graph.py) while the set of running requests stays the
        # same; a new graph is captured when it changes and every request has graph_min_tokens or more to go
        self.graphs = bool(graphs) and model.device.type == "cuda" and lockstep is None
        self.graph_min_tokens = int(graph_min_tokens)
        self._graph = None
        self._graph_key = None
        self._graph_pool = None
        self._seen_key = None        # the previous round's set: a graph is captured once a set repeats
        self.max_active = int(max_active)
        self.max_waiting = int(max_waiting)      # > 0: requests refused (ServerBusy) while this many wait
        self.failed = None                       # why the worker stopped serving (a broken lockstep group)
        self._held = None                        # the queue's head while the K/V pool cannot hold it yet
        self.max_batch = int(max_batch)
        self.waiting = queue.Queue()
        self.active = []
        self._stop = threading.Event()
        self._wake = threading.Event()
        self._thread = None
        self._ids = itertools.count()
        self.sync = sync if sync is not None else (torch.cuda.synchronize if model.device.type == "cuda"
                                                  else (lambda: None))
        self.stats = dict(requests=0, completed=0, errors=0, prompt_tokens=0, predicted_tokens=0,
                          filled_tokens=0, interleaved_rounds=0, decode_batches=0, graph_captures=0, graph_steps=0,
                          cancelled=0, refused_busy=0)
        # latency samples for /metrics: quantiles over the last LATENCY_WINDOW, count and sum over all time
        self.ttft_ms, self.prompt_ms, self.decode_round_ms = (collections.deque(maxlen=LATENCY_WINDOW)
                                                              for _ in range(3))
        self._lat_total = {k: [0, 0.0] for k in ("ttft_ms", "prompt_ms", "decode_round_ms")}
        self._lock = threading.Lock()

    # ---- control
    def start(self):
        if self._thread is None:
            self._thread = threading.Thread(target=self._loop, name="rf-scheduler", daemon=True)
            self._thread.start()
        return self

    def stop(self, timeout=30):
        self._stop.set()
        self._wake.set()
        if self._thread is not None:
            self._thread.join(timeout)
            self._thread = None

    def submit(self, req: Request):
        if req.n_predict < 1 and not (req.n_predict == 0 and req.prompt_logprobs >= 0):
            raise ValueError("n_predict must be at least 1 (0 only for a request that scores its prompt)")
        if req.ids.dim() != 1 or req.ids.numel() == 0:
            raise ValueError("the prompt must be a non-empty 1-D id sequence")
        limit = getattr(self.model, "max_positions", None)
        if limit and req.ids.numel() + req.n_predict > limit:
            raise ValueError(f"{req.ids.numel()} prompt ids + {req.n_predict} new tokens exceed the model's "
                             f"{limit} positions")
        vocab = getattr(getattr(self.model, "cfg", None), "vocab", None)
        if vocab and (int(req.ids.min()) < 0 or int(req.ids.max()) >= vocab):
            raise ValueError(f"prompt ids outside the vocabulary [0, {vocab})")
        if self.failed is not None:
            raise ServerBusy(f"the server stopped: {self.failed}")
        if self.max_waiting > 0 and self.waiting.qsize() >= self.max_waiting:
            with self._lock:
                self.stats["refused_busy"] += 1
            raise ServerBusy(f"{self.waiting.qsize()} requests are waiting (the server's limit); retry later")
        req.rid = req.rid or f"req-{next(self._ids)}"
        req.t_submit = time.perf_counter()
        with self._lock:
            self.stats["requests"] += 1
        self.waiting.put(req)
        self._wake.set()
        return req.rid

    @property
    def load(self):
        return dict(waiting=self.waiting.qsize() + (self._held is not None), active=len(self.active))

    # ---- worker
    def _loop(self):
        try:
            self._serve()
        except Exception as e:          # a broken lockstep group (a rank gone): fail every request, serve no more
            self._fail(e)
            return
        if self.lockstep is not None:
            self.lockstep.command("stop")

    def _fail(self, err):
        self.failed = f"{type(err).__name__}: {err}"
        _log.error("scheduler stopped: %s", self.failed)
        reqs = list(self.active) + ([self._held] if self._held is not None else [])
        self.active, self._held = [], None
        while True:
            try:
                reqs.append(self.waiting.get_nowait())
            except queue.Empty:
                break
        for req in reqs:
            with self._lock:
                self.stats["errors"] += 1
            self._emit(req, {"error": f"the server stopped: {self.failed}", "stop": True})

    def _admission(self, req):
        """"ok" when the paged K/V pool (if any) can hold the request's rows for its whole life on top of what the
        running requests will still take, "wait" when it can once some of them end, "never" when the pool is too
        small for it."""
        pool = getattr(self.model, "kv_pool", None)
        if pool is None:
            return "ok"
        ps, layer = pool.page_size, pool.layers[0]
        need = -(-(int(req.ids.numel()) + req.n_predict) // ps)
        if need > pool.pages:
            return "never"
        growth = 0                     # pages the running requests will still take as they decode
        for r in self.active:
            final = -(-(r.position + max(0, r.n_predict - len(r.produced))) // ps)
            have = len((r.cache[layer] if r.cache else {}).get("pages", []))
            growth += max(0, final - have)
        return "ok" if pool.free_pages(layer) - growth >= need else "wait"

    def _next_request(self):
        """The request to prefill now, or None: the queue's head unless the K/V pool cannot hold it yet (it then
        stays at the head, ahead of later arrivals, until running requests end)."""
        req = self._held
        self._held = None
        if req is None:
            try:
                req = self.waiting.get_nowait()
            except queue.Empty:
                return None
        if req.cancelled:                            # its client left while it waited: never prefilled
            with self._lock:
                self.stats["cancelled"] += 1
            return None
        verdict = self._admission(req)
        if verdict == "wait" and self.active:
            self._held = req
            return None
        if verdict != "ok":
            pool = self.model.kv_pool
            with self._lock:
                self.stats["errors"] += 1
            why = (f"more K/V pages than the pool's {pool.pages} x {pool.page_size} rows" if verdict == "never" else
                   "more K/V pages than the pool has free with nothing else running")
            self._emit(req, {"error": f"the prompt and its tokens need {why}", "stop": True})
            return None
        return req

    def _serve(self):
        while not self._stop.is_set():
            started = False
            if len(self.active) < self.max_active:
                req = self._next_request()
                if req is not None:
                    started = True
                    self._prefill(req)
            if self.active:
                self._decode_round()
            elif not started:
                self._wake.wait(0.05)
                self._wake.clear()

    def period_for(self, rows):
        """Prefill layers between decode rounds for a prompt of `rows` tokens."""
        if self.gap_ms > 0 and self._row_layer_ms:
            return max(1, int(self.gap_ms / max(1e-9, rows * self._row_layer_ms)))
        return self.interleave

    def _tick_for(self, owner):
        """tick(i) for the prefill of `owner`: a decode round of the running streams every period_for(rows) layers."""
        if self.interleave <= 0 or getattr(self.model, "tp", None) is not None or self.lockstep is not None:
            return None
        count = itertools.count(1)
        period = self.period_for(int(owner.ids.numel()))

        def tick(i):                      # the owner joins the decode set only after its prefill
            if next(count) % period == 0 and self.active:
                self.stats["interleaved_rounds"] += 1
                self._decode_round()
        return tick

    def _emit(self, req, ev):
        try:
            req.emit(ev)
        except Exception:            # a closed client must not stop the worker
            req.cancelled = True

    @torch.no_grad()
    def _prefill(self, req: Request):
        model, arm = self.model, req.arm
        n = int(req.ids.numel())
        req.t_prefill0 = time.perf_counter()
        rounds0 = self.stats["interleaved_rounds"]
        tick = self._tick_for(req)
        pool = getattr(model, "kv_pool", None)
        if pool is not None:
            pool.owner = req.rid                       # pages taken during this prefill belong to the request
        err, sent = None, False
        keep = 1 if req.prompt_logprobs < 0 else min(n, MAX_SCORED_ROWS + 1)
        try:
            if self.lockstep is not None:
                key = self.lockstep.key_of(arm)        # before the command: an unknown arm reaches no rank
                self.lockstep.command("prefill", req.rid, req.ids, req.n_predict, key, keep)
                sent = True
            logits, cache, req.filled = prefill_request(model, req.ids.to(model.device), arm, req.n_predict, tick,
                                                        keep=keep)
            tok = int(D.check_finite(logits[-1], f"{req.rid} first token").argmax())
            if req.prompt_logprobs >= 0:
                req.prompt_scores = score_prompt(logits, req.ids, req.prompt_logprobs)
                req.next_score = score_next(logits, req.prompt_logprobs)
            del logits
        except Exception as e:                         # report, drop the request, keep serving
            err = e
        if sent and not self.lockstep.agree(err is None) and err is None:
            err = RuntimeError("the prefill failed on another rank")
        if err is not None:
            self.stats["errors"] += 1
            if pool is not None:
                pool.release_owner(req.rid)
            if sent:
                self.lockstep.command("release", req.rid)
            self._emit(req, {"error": f"{type(err).__name__}: {err}", "stop": True})
            return
        now = time.perf_counter()
        req.cache, req.position, req.t_first, req.t_last = cache, n, now, now
        prompt_ms = 1e3 * (now - req.t_prefill0)
        self._observe("prompt_ms", prompt_ms)
        if self.stats["interleaved_rounds"] == rounds0 and n >= self.sample_rows:   # a clean per-row cost sample
            x = prompt_ms / (n * max(1, getattr(model, "n_layers", 1)))
            self._row_layer_ms = x if self._row_layer_ms is None else 0.7 * self._row_layer_ms + 0.3 * x
        self._observe("ttft_ms", 1e3 * (now - req.t_submit))
        self.stats["prompt_tokens"] += n
        self.stats["filled_tokens"] += req.filled
        if req.n_predict == 0:                         # a scoring request: the prompt's log-probs, no token
            self._final(req)
            return
        self._deliver(req, tok)
        if not self._done(req):
            self.active.append(req)
        else:
            self._final(req)

    def _deliver(self, req, tok):
        req.produced.append(tok)
        req.tok = tok
        self.stats["predicted_tokens"] += 1
        self._emit(req, {"tokens": [tok], "content": req.detok([tok]) if req.detok else "",
                         "tokens_predicted": len(req.produced), "stop": False})

    def _done(self, req):
        return (req.cancelled or len(req.produced) >= req.n_predict
                or (not req.ignore_eos and req.tok in self.eos) or req.tok in req.stop_ids)

    @torch.no_grad()
    def _decode_round(self):
        """One token for every active request: the plain ones together through model.decode_batch (one pass over
        the weights for all of them, up to max_batch rows at a time), SwiftKV-native ones alone (their late layers
        run a different path)."""
        pool = getattr(self.model, "kv_pool", None)
        saved = pool.owner if pool is not None else None
        if pool is not None:       # pages a decode step takes are released with the cache that holds them
            pool.owner = "decode"
        t0 = time.perf_counter()
        try:
            self._decode_round_inner()
        finally:
            if pool is not None:
                pool.owner = saved
        self._observe("decode_round_ms", 1e3 * (time.perf_counter() - t0))

    def _observe(self, name, ms):
        getattr(self, name).append(ms)
        tot = self._lat_total[name]
        tot[0] += 1
        tot[1] += ms

    def _graph_for(self, grp):
        """The decode graph of this group of requests (reused, or captured now), or None for an eager round."""
        if not self.graphs or len(grp) > self.max_batch:
            return None
        key = tuple(id(r) for r in grp)
        g = self._graph
        if g is not None and self._graph_key == key and g.room() > 0 and g.lengths == [r.position for r in grp]:
            return g
        self._graph = self._graph_key = None
        seen, self._seen_key = self._seen_key, key
        left = min(r.n_predict - len(r.produced) for r in grp)
        if left < self.graph_min_tokens or seen != key:   # capture only for a set that held for a round
            return None
        from ..engine.decode_graph import DecodeGraph
        if self._graph_pool is None:
            self._graph_pool = torch.cuda.graph_pool_handle()
        try:
            g = DecodeGraph(self.model, [r.cache for r in grp],
                            headroom=max(r.n_predict - len(r.produced) for r in grp), pool=self._graph_pool)
        except NotImplementedError:        # no device-position decode for this model: eager rounds from now on
            self.graphs = False
            return None
        except Exception as e:             # a capture that failed: report once, decode eagerly from now on
            self.graphs = False
            import sys
            print(f"decode graphs off: capture failed ({type(e).__name__}: {e})", file=sys.stderr)
            return None
        self._graph, self._graph_key = g, key
        self.stats["graph_captures"] += 1
        return g

    def _decode_round_inner(self):
        reqs = list(self.active)
        plain = [r for r in reqs if r.arm.fill != "swiftkv_native"]
        toks = {}
        for j in range(0, len(plain), self.max_batch):
            grp = plain[j:j + self.max_batch]
            if self.lockstep is not None:
                self.lockstep.command("decode", [r.rid for r in grp], [r.tok for r in grp], [r.position for r in grp])
            err = None
            try:
                g = self._graph_for(grp) if len(plain) <= self.max_batch else None
                if g is not None:
                    logits = g.step([r.tok for r in grp])
                    self.stats["graph_steps"] += 1
                else:
                    logits = self.model.decode_batch([r.tok for r in grp], [r.position for r in grp],
                                                     [r.cache for r in grp])
                self.stats["decode_batches"] += 1
            except Exception as e:          # a failed batch may have appended to some caches: end its requests
                err = e
            if self.lockstep is not None and not self.lockstep.agree(err is None) and err is None:
                err = RuntimeError("the decode batch failed on another rank")
            for j, r in enumerate(grp):
                toks[id(r)] = err if err is not None else logits[j]
        for r in reqs:
            if r.arm.fill == "swiftkv_native":
                if self.lockstep is not None:
                    self.lockstep.command("step", r.rid, r.tok, r.position, self.lockstep.key_of(r.arm))
                err = None
                try:
                    toks[id(r)] = D.step(self.model, r.tok, r.position, r.cache, r.arm)[-1]
                except Exception as e:
                    err = e
                if self.lockstep is not None and not self.lockstep.agree(err is None) and err is None:
                    err = RuntimeError("the decode step failed on another rank")
                if err is not None:
                    toks[id(r)] = err
        keep = []
        for req in reqs:
            row = toks[id(req)]
            try:
                if isinstance(row, Exception):
                    raise row
                tok = int(D.check_finite(row, f"{req.rid} decode").argmax())
            except Exception as e:
                self.stats["errors"] += 1
                self._emit(req, {"error": f"{type(e).__name__}: {e}", "stop": True})
                self._release(req)
                continue
            req.position += 1
            req.t_last = time.perf_counter()
            self._deliver(req, tok)
            if self._done(req):
                self._final(req)
            else:
                keep.append(req)
        self.active = keep
        if self._graph is not None and len(keep) != len(reqs):   # a request of the graph ended: its caches go
            self._graph = self._graph_key = None

    def _release(self, req):
        """Drop the request's cache; with a paged KV pool its pages go back to the pool."""
        pool = getattr(self.model, "kv_pool", None)
        if pool is not None and req.cache is not None:
            pool.release(req.cache)
            pool.release_owner(req.rid)
        req.cache = None
        if self.lockstep is not None:
            self.lockstep.command("release", req.rid)

    def _final(self, req):
        n = int(req.ids.numel())
        prompt_ms = 1e3 * (req.t_first - req.t_prefill0)
        pred = len(req.produced)
        pred_ms = 1e3 * (req.t_last - req.t_first)
        stop_type = ("eos" if (req.tok in self.eos and not req.ignore_eos) or req.tok in req.stop_ids else "limit")
        arm = req.arm
        timings = dict(prompt_n=n, prompt_ms=round(prompt_ms, 3),
                       prompt_per_second=round(n / max(prompt_ms, 1e-9) * 1e3, 3),
                       predicted_n=pred, predicted_ms=round(pred_ms, 3),
                       predicted_per_second=round((pred - 1) / (pred_ms / 1e3), 3) if pred > 1 and pred_ms > 0
                       else None,
                       prompt_filled_n=req.filled, cache_n=0,
                       queue_ms=round(1e3 * (req.t_prefill0 - req.t_submit), 3))
        if req.filled:
            timings["ridgefill"] = dict(n_filled=req.filled, split=arm.split, tail=arm.tail, fill=arm.fill,
                                        n_cached_exact_prefix=0)
            # the real tail of every request, one log line each (the record a protocol audit reads)
            _log.info("request %s: %d of %d prompt tokens approximated from layer %s", req.rid, req.filled, n,
                      arm.split)
        self._release(req)
        with self._lock:
            self.stats["completed"] += 1
            if req.cancelled:
                self.stats["cancelled"] += 1
        final = {"tokens": [], "content": "", "stop": True, "stop_type": stop_type, "tokens_predicted": pred,
                 "tokens_evaluated": n, "truncated": False, "id": req.rid, "timings": timings}
        if req.prompt_scores is not None:
            final["prompt_scores"] = req.prompt_scores
            if req.produced:
                final["next_score"] = req.next_score
        self._emit(req, final)

    # ---- metrics (Prometheus text exposition)
    def metrics_text(self):
        s = dict(self.stats, **self.load)
        lines = []
        for k, v in sorted(s.items()):
            name = f"ridgefill_{k}" + ("_total" if k not in ("waiting", "active") else "")
            kind = "gauge" if k in ("waiting", "active") else "counter"
            lines += [f"# TYPE {name} {kind}", f"{name} {v}"]
        dev = getattr(self.model, "device", None)
        if dev is not None and getattr(dev, "type", "") == "cuda":
            import torch
            lines += ["# TYPE ridgefill_hbm_peak_gib gauge",
                      f"ridgefill_hbm_peak_gib {torch.cuda.max_memory_allocated(dev) / 2 ** 30:.3f}"]
        pool = getattr(self.model, "kv_pool", None)
        if pool is not None:
            lines += ["# TYPE ridgefill_kv_pages_free gauge", f"ridgefill_kv_pages_free {pool.free_pages()}"]
        for key in ("ttft_ms", "prompt_ms", "decode_round_ms"):
            name, xs = f"ridgefill_{key}", sorted(getattr(self, key))
            lines.append(f"# TYPE {name} summary")
            for q in (0.5, 0.9, 0.99):
                v = xs[min(len(xs) - 1, int(q * len(xs)))] if xs else float("nan")
                lines.append(f'{name}{{quantile="{q}"}} {v:.3f}')
            count, total = self._lat_total[key]
            lines += [f"{name}_count {count}", f"{name}_sum {total:.3f}"]
        return "\n".join(lines) + "\n"
