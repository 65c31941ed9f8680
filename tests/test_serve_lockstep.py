"""Serving a sharded model in lockstep (serve/lockstep.py), on two gloo ranks on the CPU: rank 0 runs the scheduler,
rank 1 the worker loop; every model call does a collective (an all-reduce in the model's logits, as the sharded
model's own collectives would), so a call that one rank skipped or reordered would hang until the group's timeout.
The streams equal the single-process greedy decode, the worker received rank 0's commands in rank 0's order, and
an arm that is not one of the server's is refused before any rank is told."""
import os
import socket
import threading
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ridgefill_data_b200.engine.arm import Arm
from ridgefill_data_b200.engine.decode import greedy
from ridgefill_data_b200.engine.prefill import prefill
from ridgefill_data_b200.eval.data import synthetic_maps, uniform_prompt
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.tiny import tiny_configs
from ridgefill_data_b200.ridge.projector import Projector

CFG = tiny_configs(8, 64)["qwen3.5-9b"]
SPLIT, TAIL = 4, 16
JOBS = [(40, 5, "on"), (23, 3, "off"), (57, 4, "on"), (31, 6, "off")]


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _setup():
    model = from_config(CFG, seed=0, device="cpu", dtype=torch.float32)
    W, B = synthetic_maps(CFG.hidden, SPLIT, CFG.n_layers, "cpu", dtype=torch.float32)
    arms = {"off": Arm("exact"), "on": Arm("ridgefill", split=SPLIT, tail=TAIL, fill="proj",
                                            projector=Projector(SPLIT, W, B))}
    return model, arms


def _rank(rank, world, port, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    from ridgefill_data_b200.serve.engine import Request, Scheduler
    from ridgefill_data_b200.serve.lockstep import Lockstep, serve_worker
    model, arms = _setup()
    calls = []
    plain_logits = model.logits

    def logits(h):                      # a collective in every model call, like a sharded model's
        t = torch.ones(1)
        dist.all_reduce(t)
        calls.append(int(t.item()))
        return plain_logits(h)
    model.logits = logits
    ls = Lockstep(None, arms)
    if rank == 0:
        sent = []
        plain_command = ls.command

        def command(*cmd):
            sent.append((cmd[0], cmd[1] if len(cmd) > 1 else None))
            plain_command(*cmd)
        ls.command = command
        sched = Scheduler(model, interleave=2, lockstep=ls).start()
        streams, refused = [], None
        for j, (n, n_pred, mode) in enumerate(JOBS):
            evs, done = [], threading.Event()

            def emit(ev, evs=evs, done=done):
                evs.append(ev)
                if ev.get("stop"):
                    done.set()
            sched.submit(Request(ids=uniform_prompt(n, CFG.vocab, seed=j), n_predict=n_pred, arm=arms[mode],
                                 emit=emit, ignore_eos=True))
            streams.append((evs, done))
        for _, done in streams:
            done.wait(60)
        scored, sdone = [], threading.Event()            # a scoring request: prompt log-probs, no token
        sched.submit(Request(ids=uniform_prompt(30, CFG.vocab, seed=8), n_predict=0, arm=arms["off"],
                             prompt_logprobs=1, emit=lambda ev: (scored.append(ev), sdone.set() if ev.get("stop")
                                                                 else None)))
        sdone.wait(60)
        evs, done = [], threading.Event()
        sched.submit(Request(ids=uniform_prompt(20, CFG.vocab, seed=9), n_predict=2, arm=Arm("exact"),
                             emit=lambda ev: (evs.append(ev), done.set() if ev.get("stop") else None), ignore_eos=True))
        done.wait(60)
        refused = evs[-1].get("error") if evs else None
        sched.stop()
        toks = [[ev["tokens"][0] for ev in e if ev.get("tokens")] for e, _ in streams]
        first, vals = scored[-1]["prompt_scores"]
        out.put((0, dict(toks=toks, log=sent, calls=len(calls), refused=refused, scored=(first, len(vals)))))
    else:
        log = []
        serve_worker(model, ls, log=log)
        out.put((1, dict(log=log, calls=len(calls))))
    dist.destroy_process_group()


def test_lockstep_serving_mirrors_every_model_call():
    ctx = mp.get_context("spawn")
    out = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    res = dict(out.get(timeout=240) for _ in procs)
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    model, arms = _setup()
    for (n, n_pred, mode), got in zip(JOBS, res[0]["toks"]):
        ids = uniform_prompt(n, CFG.vocab, seed=JOBS.index((n, n_pred, mode)))
        logits, cache, _ = prefill(model, ids, arms[mode], keep=1)
        want, _ = greedy(model, ids, cache, logits, n_pred, arms[mode])
        assert got == list(want), (n, mode)
    assert res[1]["log"] == res[0]["log"]
    assert res[0]["log"][-1] == ("stop", None)
    ops = [op for op, _ in res[0]["log"]]
    assert ops.count("prefill") == len(JOBS) + 1 and ops.count("release") == len(JOBS) + 1 and "decode" in ops
    assert res[0]["scored"] == (1, 29)                   # every position after the first, exact
    assert res[0]["calls"] == res[1]["calls"] > 0                 # every model call met its peer's collective
    assert res[0]["refused"] and "not one of the server's arms" in res[0]["refused"]
