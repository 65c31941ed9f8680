"""Tree manifests (tools/make_manifest.py:1-166): `MANIFEST.sha256` in sha256sum format and `MANIFEST.tsv` with one
row per file (path, bytes, sha256, kind, licence), both sorted by path, plus a verifier that recomputes every hash.

Files are the git-tracked files when the root is a git work tree, else every file below the root outside `.git`;
the two manifests never list themselves. `kind` and `licence` come from first-match path-prefix rules.

    python -m ridgefill_data_b200.release.manifest write ROOT
    python -m ridgefill_data_b200.release.manifest verify ROOT      # exit 1 on a changed, missing or unlisted file
"""
from __future__ import annotations

import csv
import hashlib
import subprocess
import sys
from pathlib import Path

SELF = ("MANIFEST.sha256", "MANIFEST.tsv")
KINDS = (("results/", "result"), ("derived/", "derived"), ("provenance/", "provenance"), ("profiles/", "profile"),
         ("tests/", "test"), ("ridgefill_data_b200/", "code"), ("", "documentation"))
LICENCES = (("", "Apache-2.0"),)


def first_match(path, rules):
    for prefix, value in rules:
        if path.startswith(prefix):
            return value
    return ""


def sha256_file(path, chunk=1 << 20):
    h = hashlib.sha256()
    with open(path, "rb") as f:
        while True:
            b = f.read(chunk)
            if not b:
                return h.hexdigest()
            h.update(b)


def tracked(root):
    root = Path(root)
    try:
        out = subprocess.run(["git", "-C", str(root), "ls-files", "-z"], capture_output=True, check=True).stdout
        paths = [p for p in out.decode("utf-8").split("\0") if p]
    except (OSError, subprocess.CalledProcessError):
        paths = [p.relative_to(root).as_posix() for p in root.rglob("*")
                 if p.is_file() and ".git" not in p.relative_to(root).parts]
    return sorted(p for p in paths if p not in SELF and (root / p).is_file())


def build(root, kinds=KINDS, licences=LICENCES):
    root = Path(root)
    return [dict(path=p, bytes=(root / p).stat().st_size, sha256=sha256_file(root / p),
                 kind=first_match(p, kinds), licence=first_match(p, licences)) for p in tracked(root)]


def write(root, rows=None):
    root = Path(root)
    rows = build(root) if rows is None else rows
    (root / "MANIFEST.sha256").write_text("".join(f"{r['sha256']}  {r['path']}\n" for r in rows))
    with open(root / "MANIFEST.tsv", "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=["path", "bytes", "sha256", "kind", "licence"], delimiter="\t")
        w.writeheader()
        w.writerows(rows)
    return rows


def read_sums(path):
    out = {}
    for s in Path(path).read_text().splitlines():
        if s.strip():
            digest, name = s.split("  ", 1)
            out[name] = digest
    return out


def verify(root):
    """(changed, missing, unlisted) path lists against MANIFEST.sha256."""
    root = Path(root)
    listed = read_sums(root / "MANIFEST.sha256")
    changed = [p for p, d in listed.items() if (root / p).is_file() and sha256_file(root / p) != d]
    missing = [p for p in listed if not (root / p).is_file()]
    unlisted = [p for p in tracked(root) if p not in listed]
    return changed, missing, unlisted


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="tree manifests")
    ap.add_argument("cmd", choices=["write", "verify"])
    ap.add_argument("root")
    a = ap.parse_args(argv)
    if a.cmd == "write":
        print(f"{len(write(a.root))} files")
        return 0
    changed, missing, unlisted = verify(a.root)
    for tag, ps in (("CHANGED", changed), ("MISSING", missing), ("UNLISTED", unlisted)):
        for p in ps:
            print(f"{tag:9s}{p}")
    print(f"{len(changed)} changed, {len(missing)} missing, {len(unlisted)} unlisted")
    return 1 if changed or missing or unlisted else 0


if __name__ == "__main__":
    sys.exit(main())
