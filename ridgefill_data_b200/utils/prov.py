"""Provenance blocks and crash-safe JSON records (code/kva/prov.py:52-100).

write_json never leaves a partial file: bytes go to a temporary file beside the target, are
fsynced, read back around the page cache and compared, then renamed over the target and the
directory fsynced.
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
    try:
        return subprocess.run(["git", "-C", str(REPO), *args], capture_output=True, text=True,
                              timeout=10).stdout.strip()
    except Exception:
        return ""


COMMIT_AT_START = _git("rev-parse", "HEAD")
DIRTY_AT_START = bool(_git("status", "--porcelain", "--", "ridgefill_data_b200"))


def sha256(path):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while chunk := f.read(1 << 20):
            h.update(chunk)
    return h.hexdigest()


def gpu_info():
    try:
        import torch
        if not torch.cuda.is_available():
            return None
        p = torch.cuda.get_device_properties(torch.cuda.current_device())
        return dict(name=p.name, arch=f"sm_{p.major}{p.minor}", sms=p.multi_processor_count,
                    total_gib=round(p.total_memory / 2**30, 2), count=torch.cuda.device_count())
    except Exception:
        return None


def provenance(model=None, config=None, gpu=None):
    import torch
    return dict(time_utc=time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime()), host=platform.node(),
                code_commit=COMMIT_AT_START, code_dirty=DIRTY_AT_START,
                model=str(model) if model is not None else None, torch=torch.__version__,
                cuda=torch.version.cuda, python=sys.version.split()[0],
                command=" ".join([sys.executable] + sys.argv), gpu=gpu if gpu is not None else gpu_info(),
                config=config)


def _reads_back(path, obj):
    try:
        return json.dumps(json.loads(integrity.read_direct(path))) == json.dumps(obj)
    except ValueError:
        return False


def write_json(path, obj):
    path = Path(path)
    path.parent.mkdir(parents=True, exist_ok=True)
    tmp = path.with_name(f"{path.name}.{os.getpid()}.tmp")
    for _ in (1, 2):
        with open(tmp, "wb") as f:
            f.write(json.dumps(obj).encode())
            f.flush()
            os.fsync(f.fileno())
        if _reads_back(tmp, obj):
            break
    else:
        tmp.unlink()
        raise integrity.IntegrityError(f"{path}: the written JSON read back different twice")
    tmp.replace(path)
    fd = os.open(path.parent, os.O_RDONLY)
    try:
        os.fsync(fd)
    finally:
        os.close(fd)
