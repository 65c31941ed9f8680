"""Shard driver: run N disjoint worker processes (one per GPU) and stop every worker's process group on the first
failure (code/qwen38-27b-kit/drive.py:12-51).

Each worker runs in its own session (its own process group), gets --shard r --shards N (and CUDA_VISIBLE_DEVICES=r
when gpus is set), and logs to <out>/workers/<name>-<r>.log. The driver polls; the first non-zero exit code makes
it send SIGTERM to every worker's process group, then SIGKILL to any group still alive after `grace` seconds.
Only the process groups this driver started are signalled.

    python -m ridgefill_data_b200.utils.drive OUT --shards 4 [--gpus] -- python -m some.module ARGS
"""
from __future__ import annotations

import argparse
import os
import signal
import subprocess
import sys
import time
from pathlib import Path


class WorkerFailed(RuntimeError):
    pass


def _stop(procs, grace):
    for p in procs:
        try:
            os.killpg(p.pid, signal.SIGTERM)
        except ProcessLookupError:
            pass
    deadline = time.time() + grace
    for p in procs:
        try:
            p.wait(timeout=max(0.0, deadline - time.time()))
        except subprocess.TimeoutExpired:
            try:
                os.killpg(p.pid, signal.SIGKILL)
            except ProcessLookupError:
                pass
            p.wait()


def run_shards(cmd, shards, out, gpus=False, poll=0.2, grace=15.0, env=None, name="worker"):
    """Run cmd + ['--shard', r, '--shards', N] for r < N; returns the exit codes (all 0) or raises WorkerFailed
    naming the first failed shard after stopping every worker."""
    out = Path(out)
    (out / "workers").mkdir(parents=True, exist_ok=True)
    procs, logs = [], []
    try:
        for r in range(shards):
            e = dict(os.environ if env is None else env)
            if gpus:
                e["CUDA_VISIBLE_DEVICES"] = str(r)
            log = (out / "workers" / f"{name}-{r}.log").open("w")
            logs.append(log)
            procs.append(subprocess.Popen(list(cmd) + ["--shard", str(r), "--shards", str(shards)], stdout=log,
                                          stderr=subprocess.STDOUT, start_new_session=True, env=e))
        while True:
            codes = [p.poll() for p in procs]
            bad = [(r, c) for r, c in enumerate(codes) if c not in (None, 0)]
            if bad:
                r, c = bad[0]
                raise WorkerFailed(f"shard {r} exited with {c}; stopped every worker (logs in {out / 'workers'})")
            if all(c == 0 for c in codes):
                return codes
            time.sleep(poll)
    finally:
        _stop(procs, grace)
        for log in logs:
            log.close()


def main(argv=None):
    argv = sys.argv[1:] if argv is None else argv
    if "--" not in argv:
        raise SystemExit("usage: drive OUT --shards N [--gpus] -- CMD ...")
    i = argv.index("--")
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("out")
    ap.add_argument("--shards", type=int, required=True)
    ap.add_argument("--gpus", action="store_true")
    a = ap.parse_args(argv[:i])

    def on_term(signum, frame):
        raise SystemExit(128 + signum)
    signal.signal(signal.SIGTERM, on_term)
    run_shards(argv[i + 1:], a.shards, a.out, a.gpus)


if __name__ == "__main__":
    main()
