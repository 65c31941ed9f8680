"""Load-time integrity checks: file hashes against a recorded reference, with a disk re-read that
tells host-RAM corruption (bad page-cache pages, file intact on disk) from a changed file
(code/kva/integrity.py:1-179).

Models: <model dir>/SHA256SUMS (sha256sum format) lists exactly the top-level *.safetensors and
*.json files; it is written on first use from reads that bypass the page cache (O_DIRECT, or a
dropped cache where O_DIRECT is unsupported). Maps and other files: a sha256 recorded when the
file was written.
"""
from __future__ import annotations

import errno
import hashlib
import mmap
import os
from concurrent.futures import ThreadPoolExecutor
from pathlib import Path

CHUNK = 1 << 24
THREADS = 4
MANIFEST = "SHA256SUMS"


class IntegrityError(RuntimeError):
    """A file differs from its reference on disk too, or stays corrupted after a reload."""


def _direct_chunks(path):
    """Yield the file's bytes read around the page cache."""
    try:
        fd = os.open(path, os.O_RDONLY | os.O_DIRECT)
    except OSError as e:
        if e.errno != errno.EINVAL:
            raise
        fd = os.open(path, os.O_RDONLY)
        os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
    buf = mmap.mmap(-1, CHUNK)
    try:
        while True:
            try:
                n = os.readv(fd, [buf])
            except OSError as e:       # some filesystems accept O_DIRECT at open but refuse the read
                if e.errno != errno.EINVAL:
                    raise
                os.close(fd)
                fd = os.open(path, os.O_RDONLY)
                os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
                n = os.readv(fd, [buf])
            if not n:
                break
            with memoryview(buf) as view:
                yield bytes(view[:n])
    finally:
        os.close(fd)
        buf.close()


def read_direct(path):
    return b"".join(_direct_chunks(path))


def file_sha256(path, direct=False):
    h = hashlib.sha256()
    if direct:
        for c in _direct_chunks(path):
            h.update(c)
        return h.hexdigest()
    with open(path, "rb") as f:
        while chunk := f.read(CHUNK):
            h.update(chunk)
    return h.hexdigest()


def drop_cache(path):
    """Drop the file's clean cached pages so the next read comes from the disk."""
    fd = os.open(path, os.O_RDONLY)
    try:
        os.posix_fadvise(fd, 0, 0, os.POSIX_FADV_DONTNEED)
    finally:
        os.close(fd)


def _hash_all(paths, direct=False):
    with ThreadPoolExecutor(THREADS) as pool:
        return dict(zip(paths, pool.map(lambda p: file_sha256(p, direct), paths)))


def model_files(model_dir):
    return sorted(p for p in Path(model_dir).iterdir() if p.suffix in (".safetensors", ".json") and p.is_file())


def model_manifest(model_dir, create=True):
    """{file name: sha256} from SHA256SUMS, which must list exactly the model's files (a truncated
    manifest never passes as a short one). Written atomically from direct reads when absent."""
    model_dir = Path(model_dir)
    path = model_dir / MANIFEST
    files = model_files(model_dir)
    if path.exists():
        sums = {name.strip(): sha for sha, name in (ln.split(None, 1) for ln in path.read_text().splitlines() if ln)}
        if set(sums) != {p.name for p in files}:
            raise IntegrityError(f"{path} does not list exactly the model's files "
                                 f"(differences: {sorted(set(sums) ^ {p.name for p in files})})")
        return sums
    if not create:
        return None
    sums = {p.name: sha for p, sha in _hash_all(files, direct=True).items()}
    tmp = path.with_name(f"{MANIFEST}.{os.getpid()}.tmp")
    with open(tmp, "w") as f:
        f.write("".join(f"{sha}  {name}\n" for name, sha in sums.items()))
        f.flush()
        os.fsync(f.fileno())
    tmp.replace(path)
    return sums


def verify_model(model_dir):
    """Hash the model's files as this process reads them and compare with SHA256SUMS. Returns the
    files corrupted in RAM but intact on disk (drop and reload them); raises IntegrityError if a file
    differs on disk too."""
    model_dir = Path(model_dir)
    ref = model_manifest(model_dir)
    got = _hash_all([model_dir / name for name in ref])
    bad = [p.name for p, sha in got.items() if sha != ref[p.name]]
    for name in bad:
        disk = file_sha256(model_dir / name, direct=True)
        if disk != ref[name]:
            raise IntegrityError(f"{model_dir / name}: sha256 on disk {disk}, {MANIFEST} says {ref[name]}")
    return bad


def recorded_sha256(path, results):
    """The sha256 that the JSON records under `results` give for a file of this name (a key X holding the path with
    its X_sha256 beside it, e.g. projector / projector_sha256 in fit records, or path / sha256); None when no
    record names it, or when records disagree (one of them hashed a bad read, so none is trusted)."""
    import json
    name = Path(path).name
    found = set()

    def walk(o):
        if isinstance(o, dict):
            for k, v in o.items():
                if isinstance(v, str) and Path(v).name == name:
                    sha = o.get("sha256" if k == "path" else k + "_sha256")
                    if isinstance(sha, str):
                        found.add(sha)
                walk(v)
        elif isinstance(o, list):
            for v in o:
                walk(v)
    for f in sorted(Path(results).glob("*.json")) if Path(results).is_dir() else []:
        try:
            walk(json.loads(f.read_text()))
        except (ValueError, OSError):
            continue
    return found.pop() if len(found) == 1 else None


def read_verified(path, ref=None):
    """(bytes, sha256) of the file read normally and checked against ref (None: the disk copy read
    around the cache). On a mismatch the bytes are re-read from the disk; IntegrityError if the disk
    copy differs from ref too."""
    path = Path(path)
    data = path.read_bytes()
    got = hashlib.sha256(data).hexdigest()
    if ref is None:
        ref = file_sha256(path, direct=True)
    if got == ref:
        return data, got
    data = read_direct(path)
    got = hashlib.sha256(data).hexdigest()
    if got != ref:
        raise IntegrityError(f"{path}: sha256 {got} on disk, reference {ref}")
    drop_cache(path)
    return data, got
