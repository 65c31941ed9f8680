"""Run watchdog and memory sampler (code/c5/watchdog.sh, code/evaluate.py:219-232 KVA_MEMLOG role).

Watchdog: every `period` seconds it reads new kernel-log lines from a source (default: `journalctl -k` since the
start, when readable; tests pass a fake) and classifies NVIDIA Xid reports:
  fatal (stop the run)   Xid 48 (double-bit ECC), 74 (NVLink error), 79 (fallen off the bus), 94/95 (contained /
                         uncontained ECC), 109 (context-switch timeout), 119/120 (GSP errors), 140 (ECC unrecovered)
  logged only            every other Xid (e.g. 13 graphics engine exception, 31 MMU fault, 43 channel reset)
On a fatal line it writes <dir>/KERNEL-ALERT (reason and lines), sends SIGTERM to the watched process (or calls
`on_alert`), and stops. refuse_if_alert(dir) makes a launcher refuse to start while an alert is present.
Nothing here touches a GPU or its settings: it reads logs and memory counters only.

MemorySampler: a background thread recording torch's allocated / reserved bytes (and the device's used bytes)
every `period` seconds into a list (and optionally a JSON-lines file).
"""
from __future__ import annotations

import json
import os
import re
import signal
import subprocess
import threading
import time
from pathlib import Path

XID = re.compile(r"NVRM: Xid \(([^)]*)\): (\d+)")
FATAL_XIDS = {48, 74, 79, 94, 95, 109, 119, 120, 140}
ALERT = "KERNEL-ALERT"


def classify(line):
    """('fatal' | 'logged', xid, device) for an Xid line, else None."""
    m = XID.search(line)
    if not m:
        return None
    xid = int(m.group(2))
    return ("fatal" if xid in FATAL_XIDS else "logged"), xid, m.group(1)


def journal_source(since=None):
    """A callable returning kernel-log lines newer than the last call (empty when journalctl is unreadable)."""
    since = since or time.strftime("%Y-%m-%d %H:%M:%S")
    seen = [0]

    def read():
        try:
            out = subprocess.run(["journalctl", "-k", "--since", since, "-o", "short-iso", "--no-pager"],
                                 capture_output=True, text=True, timeout=10).stdout.splitlines()
        except (OSError, subprocess.TimeoutExpired):
            return []
        new = out[seen[0]:]
        seen[0] = len(out)
        return new
    return read


def refuse_if_alert(directory):
    alert = Path(directory) / ALERT
    if alert.exists():
        raise SystemExit(f"{alert} exists: a previous run hit an unrecoverable GPU fault; inspect and remove it first")


class Watchdog:
    def __init__(self, directory, pid=None, source=None, period=5.0, on_alert=None):
        self.dir = Path(directory)
        self.dir.mkdir(parents=True, exist_ok=True)
        self.pid, self.period, self.on_alert = pid, period, on_alert
        self.source = source or journal_source()
        self.logged, self.fired = [], None
        self._stop = threading.Event()
        self._thread = None

    def check_once(self):
        """Read new lines; returns the fatal lines (and acts on them) or []."""
        fatal = []
        for line in self.source():
            c = classify(line)
            if c is None:
                continue
            (fatal if c[0] == "fatal" else self.logged).append(line)
        if fatal and self.fired is None:
            self.fired = fatal
            (self.dir / ALERT).write_text(f"KERNEL ALERT at {time.strftime('%Y-%m-%dT%H:%M:%S')}\n" + "\n".join(fatal) + "\n")
            if self.on_alert is not None:
                self.on_alert(fatal)
            elif self.pid is not None:
                try:
                    os.kill(self.pid, signal.SIGTERM)
                except ProcessLookupError:
                    pass
        with (self.dir / "watchdog.log").open("a") as f:
            for line in fatal:
                f.write(f"fatal {line}\n")
        return fatal

    def _loop(self):
        while not self._stop.is_set() and self.fired is None:
            self.check_once()
            self._stop.wait(self.period)

    def start(self):
        self._thread = threading.Thread(target=self._loop, name="rf-watchdog", daemon=True)
        self._thread.start()
        return self

    def stop(self):
        self._stop.set()
        if self._thread is not None:
            self._thread.join(timeout=self.period + 5)


class MemorySampler:
    def __init__(self, device=None, period=0.5, path=None):
        self.device, self.period, self.path = device, period, path
        self.samples = []
        self._stop = threading.Event()
        self._thread = None

    def sample(self):
        import torch
        rec = dict(t=time.time())
        if torch.cuda.is_available():
            dev = self.device if self.device is not None else torch.cuda.current_device()
            free, total = torch.cuda.mem_get_info(dev)
            rec.update(allocated=torch.cuda.memory_allocated(dev), reserved=torch.cuda.memory_reserved(dev),
                       device_used=total - free)
        self.samples.append(rec)
        if self.path:
            with open(self.path, "a") as f:
                f.write(json.dumps(rec) + "\n")
        return rec

    def _loop(self):
        while not self._stop.is_set():
            self.sample()
            self._stop.wait(self.period)

    def __enter__(self):
        self._thread = threading.Thread(target=self._loop, name="rf-memlog", daemon=True)
        self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._thread.join(timeout=self.period + 5)
        return False

    def peak(self, key="reserved"):
        return max((s.get(key, 0) for s in self.samples), default=0)
