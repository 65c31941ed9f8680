"""Provenance blocks and crash-safe JSON records (the record keeping of code/kva/prov.py:52-100).

write_json never leaves a partial record behind: the JSON goes to a temporary file next to the target, is synced,
then read back from the disk (around the page cache) and compared with the object. One failed comparison is
retried; a second one is an IntegrityError. Only a verified temporary file is renamed over the target, and the
directory is synced after the rename.
"""
from __future__ import annotations

import hashlib
import json
import os
import platform
import subprocess
import sys
import time
from pathlib import Path

from . import integrity

REPO = Path(__file__).resolve().parents[2]


def _git(*args):
    """Output of a git command in this checkout ('' when git or the checkout is unavailable)."""
    try:
        done = subprocess.run(["git", "-C", str(REPO), *args], capture_output=True, text=True, timeout=10)
    except (OSError, subprocess.SubprocessError):
        return ""
    return done.stdout.strip()


# the code state when this process imported the package (later edits do not change what already runs)
COMMIT_AT_START = _git("rev-parse", "HEAD")
DIRTY_AT_START = _git("status", "--porcelain", "--", "ridgefill_data_b200") != ""


def sha256(path):
    with open(path, "rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def gpu_info():
    """Name, architecture, SM count, memory and device count of the current GPU (None without one)."""
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        props = torch.cuda.get_device_properties(torch.cuda.current_device())
        return {"name": props.name, "arch": f"sm_{props.major}{props.minor}", "sms": props.multi_processor_count,
                "total_gib": round(props.total_memory / 2 ** 30, 2), "count": torch.cuda.device_count()}
    except Exception:                        # a probe of the device never fails the run it describes
        return None


def provenance(model=None, config=None, gpu=None):
    """Who, where, what code and what software produced a record."""
    import torch
    return {
        "time_utc": time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()),
        "host": platform.node(),
        "code_commit": COMMIT_AT_START,
        "code_dirty": DIRTY_AT_START,
        "model": None if model is None else str(model),
        "torch": torch.__version__,
        "cuda": torch.version.cuda,
        "python": platform.python_version(),
        "command": " ".join([sys.executable, *sys.argv]),
        "gpu": gpu_info() if gpu is None else gpu,
        "config": config,
    }


def _matches(path, obj):
    """The file, read around the page cache, parses to the same JSON as obj."""
    try:
        on_disk = json.loads(integrity.read_direct(path))
    except ValueError:
        return False
    return json.dumps(on_disk) == json.dumps(obj)


def _sync_dir(folder):
    fd = os.open(folder, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)


def write_json(path, obj):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.parent / f"{path.name}.{os.getpid()}.tmp"
    payload = json.dumps(obj).encode()
    attempts = 2
    for _ in range(attempts):
        with open(tmp, "wb") as f:
            f.write(payload)
            f.flush()
            os.fsync(f.fileno())
        if _matches(tmp, obj):
            break
    else:
        tmp.unlink()
        raise integrity.IntegrityError(f"{path}: the JSON read back differently after {attempts} writes")
    os.replace(tmp, path)
    _sync_dir(path.parent)
