"""Serving a tensor-parallel model: rank 0 schedules, every rank makes the same model calls in the same order.

The HTTP front end and the scheduler (serve/engine.py) run on rank 0 only. Every call that touches the sharded
model (a request's prefill, a decode batch, a single SwiftKV-native step) is first broadcast to the other ranks as a
small command over a CPU (gloo) process group and then run on every rank, so the model's own collectives (NCCL or
the NVSwitch kernels) line up: same calls, same order, same inputs. Rank 0's tokens drive the decode: a command
carries the tokens and positions of its batch, so the workers never pick a token themselves. After each model call
the ranks agree on its outcome (an all-reduce of a failure flag): a request that fails on every rank alike (an input
the engine refuses before the model's collectives) is dropped on all of them and its caches are released everywhere.
A failure on one rank inside the model's collectives leaves the others waiting in a collective, and the process
group's timeout ends the job (the host-side failure detection of parallel/health.py covers that case). Caches stay
where they are made; a worker keeps them by request id.

Commands, all from the scheduler's one worker thread:
  ("prefill", rid, ids, n_predict, arm_key, keep)   then agree   (keep: prompt rows whose logits are computed)
  ("decode", [rid], [tok], [position])        then agree
  ("step", rid, tok, position, arm_key)       then agree   (SwiftKV-native requests)
  ("release", rid)
  ("stop",)

Decode rounds are not interleaved into a prefill here (the scheduler turns the tick off under lockstep) and decode
graphs stay off (a graph holds one rank's pointers only).
"""
from __future__ import annotations

import torch
import torch.distributed as dist

from ..engine import decode as D


class Lockstep:
    """Commands and outcome agreement over `group` (a gloo group of the serving ranks; None: the default group,
    which must then be gloo). `arms` maps the request modes to the arms every rank built alike; a command names an
    arm by its key."""

    def __init__(self, group=None, arms=None, src=0):
        self.group = group
        self.src = int(src)
        self.arms = dict(arms or {})
        self.rank = dist.get_rank()
        self.world = dist.get_world_size(group)

    def key_of(self, arm):
        for k, a in self.arms.items():
            if a is arm:
                return k
        raise ValueError("the request's arm is not one of the server's arms, so the other ranks cannot run it")

    def command(self, *cmd):
        dist.broadcast_object_list([cmd], src=self.src, group=self.group)

    def receive(self):
        box = [None]
        dist.broadcast_object_list(box, src=self.src, group=self.group)
        return box[0]

    def agree(self, ok):
        """True when the call succeeded on every rank."""
        flag = torch.tensor([0 if ok else 1], dtype=torch.int32)
        dist.all_reduce(flag, group=self.group)
        return int(flag.item()) == 0


def serve_worker(model, lockstep, log=None):
    """The loop of a rank other than 0: run each command as rank 0 does, until ("stop",). `log`: a list that gets
    (op, rid or rids) for every command (tests compare it with rank 0's)."""
    from .engine import prefill_request
    caches = {}
    pool = getattr(model, "kv_pool", None)
    arms = lockstep.arms
    while True:
        cmd = lockstep.receive()
        op = cmd[0]
        if log is not None:
            log.append((op, cmd[1] if len(cmd) > 1 else None))
        if op == "stop":
            return
        if op == "release":
            cache = caches.pop(cmd[1], None)
            if pool is not None:
                if cache is not None:
                    pool.release(cache)
                pool.release_owner(cmd[1])
            continue
        ok = True
        try:
            with torch.no_grad():
                if op == "prefill":
                    _, rid, ids, n_predict, key, keep = cmd
                    if pool is not None:
                        pool.owner = rid
                    _, cache, _ = prefill_request(model, ids.to(model.device), arms[key], n_predict, keep=keep)
                    caches[rid] = cache
                elif op == "decode":
                    _, rids, toks, positions = cmd
                    if pool is not None:
                        pool.owner = "decode"
                    model.decode_batch(list(toks), list(positions), [caches[r] for r in rids])
                elif op == "step":
                    _, rid, tok, position, key = cmd
                    if pool is not None:
                        pool.owner = "decode"
                    D.step(model, tok, position, caches[rid], arms[key])
                else:
                    raise ValueError(f"lockstep command {op!r}")
        except Exception:            # the outcome is agreed below; rank 0 reports it
            ok = False
            if op == "prefill" and pool is not None:
                pool.release_owner(cmd[1])
        lockstep.agree(ok)
