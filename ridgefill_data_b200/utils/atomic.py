"""Atomic result files with sha256 sidecars and a results-tree hash (code/finals/lib/atomic.py).

write_result(path, obj): JSON to a temporary file beside the target, fsync, read back (the bytes must match what
was written), rename, fsync the directory; then the same for '<path>.sha256' in `sha256sum -c` format. A file is
finished only when it and a matching sidecar exist. treehash(root): sha256 over the sorted '<relpath> <sha256>'
lines of every regular file (hidden files and sidecars excluded), for receipts naming exactly which bytes moved.

    python -m ridgefill_data_b200.utils.atomic treehash DIR | sidecar FILE | check FILE...
"""
from __future__ import annotations

import argparse
import hashlib
import json
import os
import sys
import tempfile
from pathlib import Path


class AtomicWriteError(RuntimeError):
    """The bytes did not read back as written."""


def sha256_file(path, bufsize=1 << 20):
    digest = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(bufsize), b""):
            digest.update(block)
    return digest.hexdigest()


def write_bytes(path, data):
    path = Path(path)
    folder = path.parent
    folder.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix="." + path.name + ".", dir=folder)
    try:
        with os.fdopen(fd, "wb") as f:
            f.write(data)
            f.flush()
            os.fsync(f.fileno())
        with open(tmp, "rb") as f:
            if f.read() != data:
                raise AtomicWriteError(f"{path}: read-back differs from the written bytes")
        os.replace(tmp, path)
    except BaseException:
        if os.path.exists(tmp):
            os.unlink(tmp)
        raise
    dfd = os.open(path.parent, os.O_RDONLY)
    try:
        os.fsync(dfd)
    finally:
        os.close(dfd)


def sidecar_line(path, digest):
    return f"{digest}  {Path(path).name}\n"


def write_result(path, obj):
    """JSON + sidecar, atomically; returns the sha256."""
    data = (json.dumps(obj, sort_keys=True, indent=1) + "\n").encode()
    write_bytes(path, data)
    digest = hashlib.sha256(data).hexdigest()
    write_bytes(f"{path}.sha256", sidecar_line(path, digest).encode())
    return digest


def read_sidecar(path):
    """The sha256 a sidecar records for path, or None (missing or malformed)."""
    sc = Path(f"{path}.sha256")
    if not sc.exists():
        return None
    try:
        digest, name = sc.read_text().splitlines()[0].split("  ", 1)
    except (ValueError, IndexError):
        return None
    if name != Path(path).name or len(digest) != 64 or set(digest) - set("0123456789abcdef"):
        return None
    return digest


def finished(path):
    p = Path(path)
    return p.exists() and read_sidecar(p) is not None and read_sidecar(p) == sha256_file(p)


def refresh_sidecar(path):
    write_bytes(f"{path}.sha256", sidecar_line(path, sha256_file(path)).encode())


def treehash(root):
    root = Path(root)
    lines = []
    for p in sorted(root.rglob("*")):
        hidden_or_sidecar = p.name.startswith(".") or p.name.endswith(".sha256")
        if p.is_file() and not hidden_or_sidecar:
            lines.append(f"{p.relative_to(root).as_posix()} {sha256_file(p)}\n")
    return hashlib.sha256("".join(lines).encode()).hexdigest()


def main(argv=None):
    ap = argparse.ArgumentParser(prog="ridgefill_data_b200.utils.atomic", description="atomic result files")
    sub = ap.add_subparsers(required=True, dest="cmd")
    for name in ("treehash", "sidecar"):
        sub.add_parser(name).add_argument("path")
    sub.add_parser("check").add_argument("paths", nargs="+")
    a = ap.parse_args(argv)
    if a.cmd == "treehash":
        print(treehash(a.path))
    elif a.cmd == "sidecar":
        refresh_sidecar(a.path)
    else:
        bad = [p for p in a.paths if not finished(p)]
        for p in bad:
            print(f"MISMATCH {p}: no sidecar or it does not match", file=sys.stderr)
        return 2 if bad else 0
    return 0


if __name__ == "__main__":
    sys.exit(main())
