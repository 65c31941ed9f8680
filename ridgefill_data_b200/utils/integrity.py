"""Load-time integrity checks (the checks of code/kva/integrity.py:1-179): file hashes compared with a recorded
reference, and a second read from the disk that separates corrupted host memory (bad page-cache pages over an
intact file) from a file that really changed.

A model directory carries SHA256SUMS in sha256sum's format, listing exactly its top-level *.safetensors and *.json
files. When it is missing it is written from reads that bypass the page cache (O_DIRECT, or a dropped cache where
the filesystem refuses O_DIRECT). Other files (maps, predictors) are checked against the sha256 recorded when they
were written.
"""
from __future__ import annotations

import errno
import hashlib
import json
import mmap
import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CHUNK = 1 << 24
THREADS = 4
MANIFEST = "SHA256SUMS"


class IntegrityError(RuntimeError):
    """A file differs from its reference on the disk as well, or is still wrong after a reload."""


def _evict(fd):
    os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)


class _Uncached:
    """Iterate over a file's bytes in CHUNK blocks without serving them from the page cache. O_DIRECT is tried
    first; a filesystem that refuses it (at open, or at the first read) gets a plain descriptor whose cached pages
    are dropped first."""

    def __init__(self, path):
        self.path = path

    def _plain(self):
        fd = os.open(self.path, os.O_RDONLY)
        _evict(fd)
        return fd

    def __iter__(self):
        try:
            fd = os.open(self.path, os.O_RDONLY | os.O_DIRECT)
            direct = True
        except OSError as e:
            if e.errno != errno.EINVAL:
                raise
            fd, direct = self._plain(), False
        block = mmap.mmap(-1, CHUNK)            # page aligned, as O_DIRECT requires
        done = 0
        try:
            while True:
                try:
                    got = os.readv(fd, [block])
                except OSError as e:
                    if e.errno != errno.EINVAL or not direct:
                        raise
                    os.close(fd)
                    fd, direct = self._plain(), False
                    os.lseek(fd, done, os.SEEK_SET)
                    continue
                if got == 0:
                    return
                done += got
                yield block[:got]
        finally:
            os.close(fd)
            block.close()


def read_direct(path):
    return b"".join(_Uncached(path))


def file_sha256(path, direct=False):
    digest = hashlib.sha256()
    if direct:
        for piece in _Uncached(path):
            digest.update(piece)
    else:
        with open(path, "rb") as f:
            for piece in iter(lambda: f.read(CHUNK), b""):
                digest.update(piece)
    return digest.hexdigest()


def drop_cache(path):
    """Evict the file's clean cached pages, so that the next read comes from the disk."""
    fd = os.open(path, os.O_RDONLY)
    try:
        _evict(fd)
    finally:
        os.close(fd)


def _hash_all(paths, direct=False):
    paths = list(paths)
    with ThreadPoolExecutor(THREADS) as pool:
        sums = list(pool.map(file_sha256, paths, [direct] * len(paths)))
    return dict(zip(paths, sums))


def model_files(model_dir):
    return sorted(p for p in Path(model_dir).iterdir() if p.is_file() and p.suffix in (".safetensors", ".json"))


def _parse_sums(text):
    sums = {}
    for line in text.splitlines():
        if line:
            sha, name = line.split(None, 1)
            sums[name.strip()] = sha
    return sums


def model_manifest(model_dir, create=True):
    """{file name: sha256} from SHA256SUMS, which has to list exactly the model's files (a truncated list is an
    error, not a shorter check). Written atomically from uncached reads when absent (unless create is off)."""
    model_dir = Path(model_dir)
    path = model_dir / MANIFEST
    names = {p.name for p in model_files(model_dir)}
    if path.exists():
        sums = _parse_sums(path.read_text())
        if set(sums) != names:
            raise IntegrityError(f"{path} must list exactly the model's files; mismatched: "
                                 f"{sorted(set(sums).symmetric_difference(names))}")
        return sums
    if not create:
        return None
    sums = {p.name: sha for p, sha in _hash_all(model_files(model_dir), direct=True).items()}
    tmp = path.parent / f"{MANIFEST}.{os.getpid()}.tmp"
    with open(tmp, "w") as f:
        for name, sha in sums.items():
            f.write(f"{sha}  {name}\n")
        f.flush()
        os.fsync(f.fileno())
    os.replace(tmp, path)
    return sums


def verify_model(model_dir):
    """Hash the model's files as this process reads them and compare them with SHA256SUMS. Returns the names of
    files that are wrong in memory but intact on the disk (the caller drops and reloads them); raises
    IntegrityError when a file is wrong on the disk too."""
    model_dir = Path(model_dir)
    want = model_manifest(model_dir)
    seen = _hash_all(model_dir / name for name in want)
    wrong = [p.name for p, sha in seen.items() if want[p.name] != sha]
    for name in wrong:
        on_disk = file_sha256(model_dir / name, direct=True)
        if on_disk != want[name]:
            raise IntegrityError(f"{model_dir / name} hashes to {on_disk} on the disk; {MANIFEST} records "
                                 f"{want[name]}")
    return wrong


def _pins(obj, name):
    """sha256 strings recorded beside a value naming the file `name` anywhere in a JSON object: key X with X_sha256
    next to it, or path with sha256 next to it."""
    stack = [obj]
    while stack:
        o = stack.pop()
        if isinstance(o, list):
            stack.extend(o)
        elif isinstance(o, dict):
            for k, v in o.items():
                if isinstance(v, str) and Path(v).name == name:
                    sha = o.get("sha256" if k == "path" else f"{k}_sha256")
                    if isinstance(sha, str):
                        yield sha
                stack.append(v)


def recorded_sha256(path, results):
    """The sha256 that the JSON records in directory `results` give for a file of this name, or None when no
    record names it or the records disagree (then one of them hashed a bad read, and none is trusted)."""
    results = Path(results)
    if not results.is_dir():
        return None
    name = Path(path).name
    found = set()
    for f in sorted(results.glob("*.json")):
        try:
            found.update(_pins(json.loads(f.read_text()), name))
        except (OSError, ValueError):
            continue
    return next(iter(found)) if len(found) == 1 else None


def read_verified(path, ref=None):
    """(bytes, sha256) of a file, read normally and compared with ref (default: the hash of an uncached read).
    On a mismatch the bytes are read again from the disk; IntegrityError if those differ from ref as well."""
    path = Path(path)
    if ref is None:
        ref = file_sha256(path, direct=True)
    data = path.read_bytes()
    sha = hashlib.sha256(data).hexdigest()
    if sha == ref:
        return data, sha
    data = read_direct(path)
    sha = hashlib.sha256(data).hexdigest()
    if sha != ref:
        raise IntegrityError(f"{path} hashes to {sha} on the disk; the reference is {ref}")
    drop_cache(path)
    return data, sha
