"""Result files that are either complete or absent, each with a sha256 sidecar, and a hash over a results tree
(the file discipline of code/finals/lib/atomic.py).

write_result(path, obj) writes the JSON through write_bytes: a temporary file in the target's folder, synced, read
back and compared byte for byte, renamed over the target, then the folder synced. '<path>.sha256' (sha256sum
format) is written the same way afterwards, so a file counts as finished only when both exist and agree.
treehash(root) hashes the sorted '<relative path> <sha256>' lines of every regular file under root (hidden files
and sidecars left out), so that a receipt can name exactly which bytes moved.

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

_HEX = frozenset("0123456789abcdef")


class AtomicWriteError(RuntimeError):
    """What was written did not read back identically."""


def sha256_file(path, bufsize=1 << 20):
    digest = hashlib.sha256()
    with open(path, "rb") as f:
        for block in iter(lambda: f.read(bufsize), b""):
            digest.update(block)
    return digest.hexdigest()


def _fsync_folder(folder):
    handle = os.open(folder, os.O_RDONLY)
    try:
        os.fsync(handle)
    finally:
        os.close(handle)


def _write_checked(tmp, data, target):
    with open(tmp, "wb") as out:
        out.write(data)
        out.flush()
        os.fsync(out.fileno())
    if Path(tmp).read_bytes() != data:
        raise AtomicWriteError(f"{target}: the temporary file did not read back as written")


def write_bytes(path, data):
    """Replace `path` with `data` so that readers see the old file or the new one, never a mix."""
    path = Path(path)
    folder = path.parent
    folder.mkdir(parents=True, exist_ok=True)
    fd, tmp = tempfile.mkstemp(prefix="." + path.name + ".", dir=folder)
    os.close(fd)
    try:
        _write_checked(tmp, data, path)
        os.replace(tmp, path)
    except BaseException:
        Path(tmp).unlink(missing_ok=True)
        raise
    _fsync_folder(folder)


def sidecar_line(path, digest):
    return f"{digest}  {Path(path).name}\n"


def _sidecar(path):
    return Path(f"{path}.sha256")


def write_result(path, obj):
    """The JSON of obj and its sidecar, each written atomically; returns the sha256."""
    data = (json.dumps(obj, sort_keys=True, indent=1) + "\n").encode()
    write_bytes(path, data)
    digest = hashlib.sha256(data).hexdigest()
    write_bytes(_sidecar(path), sidecar_line(path, digest).encode())
    return digest


def read_sidecar(path):
    """The sha256 that the sidecar of `path` records, or None when it is missing or malformed."""
    side = _sidecar(path)
    if not side.exists():
        return None
    lines = side.read_text().splitlines()
    if not lines or "  " not in lines[0]:
        return None
    digest, _, name = lines[0].partition("  ")
    well_formed = len(digest) == 64 and set(digest) <= _HEX and name == Path(path).name
    return digest if well_formed else None


def finished(path):
    """The file exists and its sidecar records its current sha256."""
    path = Path(path)
    if not path.exists():
        return False
    recorded = read_sidecar(path)
    return recorded is not None and recorded == sha256_file(path)


def refresh_sidecar(path):
    write_bytes(_sidecar(path), sidecar_line(path, sha256_file(path)).encode())


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
    sub.add_parser("treehash").add_argument("path")
    sub.add_parser("sidecar").add_argument("path")
    sub.add_parser("check").add_argument("paths", nargs="+")
    a = ap.parse_args(argv)
    if a.cmd == "treehash":
        print(treehash(a.path))
        return 0
    if a.cmd == "sidecar":
        refresh_sidecar(a.path)
        return 0
    unfinished = [p for p in a.paths if not finished(p)]
    for p in unfinished:
        print(f"MISMATCH {p}: no sidecar or it does not match", file=sys.stderr)
    return 2 if unfinished else 0


if __name__ == "__main__":
    sys.exit(main())
