"""Failure detection on the host (no GPU is faulted): gloo ranks on the CPU where one rank raises, announces and
leaves, or stops beating; the shard driver stopping every worker on the first failure; the kernel-log watchdog on
a fake log; atomic results and the cell runner's resume / host rules."""
import json
import os
import socket
import sys
import time
from datetime import timedelta

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from ridgefill_data_b200.eval import runner as RN
from ridgefill_data_b200.parallel.health import Heartbeat, PeerLost
from ridgefill_data_b200.utils import atomic, drive, watch


def _port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, mode, out):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    store = dist.distributed_c10d._get_default_store()
    hb = Heartbeat(store, rank, world, stale=2.0)
    x = torch.ones(4)
    dist.all_reduce(x)                                     # step 0: everybody present
    dist.barrier()
    result = "ok"
    try:
        if rank == 1:
            if mode == "announce":
                try:
                    raise ValueError("bad input on rank 1")
                except ValueError as e:
                    hb.fail(e)
                    return
            if mode == "silent":
                return                                     # leaves between steps without a word
            if mode == "skip_collective":
                time.sleep(8)
                return
        if mode == "silent":
            time.sleep(3)                                  # past the stale limit
        elif mode == "announce":
            time.sleep(1)
        if mode == "skip_collective":
            try:
                dist.all_reduce(x)                         # rank 1 never joins: the group timeout ends it
                result = "joined"
            except Exception as e:                          # noqa: BLE001
                result = f"collective error: {type(e).__name__}"
        else:
            try:
                hb.check()
                result = "no failure seen"
            except PeerLost as e:
                result = f"lost: {e}"
    finally:
        if rank == 0:
            with open(out, "w") as f:
                f.write(result)
    dist.destroy_process_group()


@pytest.mark.parametrize("mode,want", [("announce", "lost: rank 1 failed: bad input"), ("silent", "lost: rank 1: no heartbeat"),
                                       ("skip_collective", "collective error")])
def test_rank_failure_seen_on_host(tmp_path, mode, want):
    out = tmp_path / "r0.txt"
    ctx = mp.get_context("spawn")
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, mode, str(out))) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert out.read_text().startswith(want), out.read_text()


def test_drive_stops_every_worker_on_first_failure(tmp_path):
    code = ("import sys, time\n"
            "r = int(sys.argv[sys.argv.index('--shard') + 1])\n"
            "time.sleep(0.5)\n"
            "sys.exit(3) if r == 1 else time.sleep(60)\n")
    t0 = time.time()
    with pytest.raises(drive.WorkerFailed, match="shard 1 exited with 3"):
        drive.run_shards([sys.executable, "-c", code], 3, tmp_path, grace=5)
    assert time.time() - t0 < 30
    ok = drive.run_shards([sys.executable, "-c", "import sys; sys.exit(0)"], 2, tmp_path)
    assert ok == [0, 0]


def test_watchdog_classifies_and_fires(tmp_path):
    lines = [["NVRM: Xid (PCI:0000:1b:00): 13, pid=1, Graphics Exception"],
             ["kernel: something else", "NVRM: Xid (PCI:0000:1b:00): 79, pid=1, GPU has fallen off the bus."]]
    fired = []
    wd = watch.Watchdog(tmp_path, source=lambda: lines.pop(0) if lines else [], on_alert=fired.append)
    assert wd.check_once() == [] and len(wd.logged) == 1
    assert len(wd.check_once()) == 1 and fired
    assert (tmp_path / watch.ALERT).exists()
    with pytest.raises(SystemExit):
        watch.refuse_if_alert(tmp_path)
    assert watch.classify("NVRM: Xid (PCI:0000:1b:00): 109, ...")[0] == "fatal"
    assert watch.classify("no xid here") is None


def test_memory_sampler():
    with watch.MemorySampler(period=0.05) as m:
        time.sleep(0.2)
    assert len(m.samples) >= 2


def test_atomic_results(tmp_path):
    p = tmp_path / "a" / "r.json"
    digest = atomic.write_result(p, dict(x=1))
    assert atomic.finished(p) and atomic.read_sidecar(p) == digest
    p.write_text(p.read_text().replace("1", "2"))
    assert not atomic.finished(p)
    atomic.refresh_sidecar(p)
    assert atomic.finished(p)
    h1 = atomic.treehash(tmp_path)
    (tmp_path / "a" / "s.json").write_text("{}")
    assert atomic.treehash(tmp_path) != h1
    assert atomic.main(["check", str(p)]) == 0


def test_cell_runner_resume_and_host(tmp_path):
    ledger = tmp_path / "ledger.jsonl"
    ledger.write_text(json.dumps(dict(type="hypothesis", id="FINAL-X")) + "\n")
    cell = dict(name="c1", registration="FINAL-X", samples=["s1", "s2", "s3"], arms=["exact", "kva"])
    calls = []

    def harness(c, sid):
        calls.append(sid)
        return RN.mock_harness(c, sid)
    host = dict(host="h1", gpu_name="B200", driver="580")
    RN.run_cell(cell, tmp_path / "res", harness, ledger, info=host)
    assert calls == ["s1", "s2", "s3"]
    (tmp_path / "res" / "c1" / "samples" / "s2.json").unlink()
    RN.run_cell(cell, tmp_path / "res", harness, ledger, info=host)
    assert calls[3:] == ["s2"]                                             # resumes the missing sample only
    with pytest.raises(SystemExit, match="does not resume on another host"):
        RN.run_cell(cell, tmp_path / "res", harness, ledger, info=dict(host, host="h2"))
    RN.run_cell(cell, tmp_path / "res", harness, ledger, info=dict(host, host="h2"), new_host=True)
    assert any(p.name.startswith("c1.abandoned-") for p in (tmp_path / "res").iterdir())
    with pytest.raises(SystemExit, match="differs"):
        RN.run_cell(dict(cell, arms=["exact"]), tmp_path / "res", harness, ledger, info=dict(host, host="h2"))
    with pytest.raises(SystemExit, match="FINAL-TBD|not a declared"):
        RN.run_cell(dict(cell, registration="FINAL-TBD"), tmp_path / "res", harness, ledger, info=host)
