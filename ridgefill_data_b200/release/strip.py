"""Copy a results tree with prompt text replaced by its hash (tools/strip_prompts.py:1-272): what a release may
publish when the prompts themselves are licensed or private.

Every file under SRC is copied to the same relative path under DST, except that
  * files matching an --exclude glob (against the relative path or any path component) are left out;
  * in .json / .jsonl files, a value under a key of --fields (at any depth) becomes
    {"stripped": true, "sha256": <sha256 of its canonical JSON>, "n": <len>} (canonical: sorted keys, separators
    "," and ":", UTF-8 unescaped), so a holder of the original can prove the match; a value under a key of
    --drop-fields becomes {"stripped": true, "n": <len>} with no hash (for short answer keys a hash would reveal),
    and that file's original hash is logged as "withheld";
  * every match of a --redact NAME=REGEX becomes "NAME-k", k numbering the distinct matched values in sorted order
    over the whole run (equal values keep equal labels);
  * files matching a --gzip glob are stored gzip-compressed with mtime 0 (reproducible bytes).
Untouched files are copied byte for byte. Each transformed file gets a row in the TSV log (path, origin sha256,
sha256, transforms, counts). DST must be empty or absent and outside SRC.
"""
from __future__ import annotations

import fnmatch
import gzip
import hashlib
import json
import os
import re
import sys
from dataclasses import dataclass, field
from pathlib import Path, PurePosixPath

LOG_FIELDS = ("path", "origin_sha256", "sha256", "transform", "detail")


def canonical(value):
    return json.dumps(value, sort_keys=True, separators=(",", ":"), ensure_ascii=False).encode("utf-8")


def _sha(b):
    return hashlib.sha256(b).hexdigest()


def _size(v):
    return len(v) if isinstance(v, (str, list, dict)) else None


def is_stripped(v):
    return isinstance(v, dict) and v.get("stripped") is True


@dataclass
class Stripper:
    fields: set = field(default_factory=set)        # hashed
    drop: set = field(default_factory=set)          # replaced without a hash
    redact: list = field(default_factory=list)      # [(name, compiled regex)]
    gzip_globs: list = field(default_factory=list)
    exclude: list = field(default_factory=list)

    def strip(self, obj, counts):
        if isinstance(obj, dict):
            out = {}
            for k, v in obj.items():
                if (k in self.fields or k in self.drop) and not is_stripped(v):
                    rec = {"stripped": True, "n": _size(v)}
                    if k not in self.drop:
                        rec["sha256"] = _sha(canonical(v))
                    out[k] = rec
                    tag = ("drop:" if k in self.drop else "strip:") + k
                    counts[tag] = counts.get(tag, 0) + 1
                else:
                    out[k] = self.strip(v, counts)
            return out
        if isinstance(obj, list):
            return [self.strip(v, counts) for v in obj]
        return obj

    # ---- file formats
    @staticmethod
    def _indent(text):
        second = text.split("\n", 2)[1] if "\n" in text else ""
        lead = len(second) - len(second.lstrip(" "))
        return lead or None

    def json_text(self, text, counts):
        c = {}
        new = self.strip(json.loads(text), c)
        if not c:
            return text
        counts.update(c)
        ind = self._indent(text)
        sep = None if ind is not None or '": ' in text[:4096] else (",", ":")
        return json.dumps(new, indent=ind, ensure_ascii=text.isascii(), separators=sep) + \
            ("\n" if text.endswith("\n") else "")

    def jsonl_text(self, text, counts):
        out = []
        for ln in text.splitlines(keepends=True):
            body = ln.rstrip("\r\n")
            if not body.strip():
                out.append(ln)
                continue
            c = {}
            new = self.strip(json.loads(body), c)
            if not c:
                out.append(ln)
                continue
            for k, v in c.items():
                counts[k] = counts.get(k, 0) + v
            sep = None if '": ' in body else (",", ":")
            out.append(json.dumps(new, ensure_ascii=body.isascii(), separators=sep) + ln[len(body):])
        return "".join(out)

    # ---- tree
    def excluded(self, rel):
        parts = PurePosixPath(rel).parts
        return any(fnmatch.fnmatch(rel, g) or any(fnmatch.fnmatch(p, g) for p in parts) for g in self.exclude)

    def labels(self, files):
        seen = {name: set() for name, _ in self.redact}
        for _, path in files:
            data = path.read_bytes()
            if b"\0" in data[:8192]:
                continue
            text = data.decode("utf-8", errors="replace")
            for name, rx in self.redact:
                seen[name].update(m.group(0) for m in rx.finditer(text))
        return {name: {v: f"{name}-{k}" for k, v in enumerate(sorted(vals), 1)} for name, vals in seen.items()}

    def copy_tree(self, src, dst, log=None):
        src, dst = Path(src).resolve(), Path(dst).resolve()
        if not src.is_dir():
            raise ValueError(f"{src} is not a directory")
        if dst == src or src in dst.parents:
            raise ValueError(f"destination {dst} lies inside the source {src}")
        if dst.exists() and any(dst.iterdir()):
            raise ValueError(f"destination {dst} is not empty")
        files = []
        for root, dirs, names in os.walk(src):
            dirs.sort()
            for n in sorted(names):
                p = Path(root) / n
                rel = p.relative_to(src).as_posix()
                if not self.excluded(rel):
                    files.append((rel, p))
        labels = self.labels(files) if self.redact else {}
        rows, withheld = [], set()
        for rel, p in files:
            data = p.read_bytes()
            counts, out = {}, data
            if b"\0" not in data[:8192]:
                try:
                    text = data.decode("utf-8")
                except UnicodeDecodeError:
                    text = None
                if text is not None:
                    new = text
                    if self.fields or self.drop:
                        if rel.endswith(".json"):
                            new = self.json_text(text, counts)
                        elif rel.endswith(".jsonl"):
                            new = self.jsonl_text(text, counts)
                    for name, rx in self.redact:
                        def sub(m, name=name):
                            counts[f"redact:{name}"] = counts.get(f"redact:{name}", 0) + 1
                            return labels[name][m.group(0)]
                        new = rx.sub(sub, new)
                    if new != text:
                        out = new.encode("utf-8")
            dst_rel = rel
            if any(fnmatch.fnmatch(PurePosixPath(rel).name, g) for g in self.gzip_globs):
                out = gzip.compress(out, compresslevel=9, mtime=0)
                dst_rel += ".gz"
                counts["gzip"] = 1
            target = dst / dst_rel
            target.parent.mkdir(parents=True, exist_ok=True)
            target.write_bytes(out)
            if counts:
                dropped = any(k.startswith("drop:") for k in counts)
                if dropped:
                    withheld.add(rel)
                rows.append(dict(path=dst_rel, origin_sha256="withheld" if dropped else _sha(data), sha256=_sha(out),
                                 transform=",".join(sorted(counts)),
                                 detail=";".join(f"{k}={v}" for k, v in sorted(counts.items()))))
        # a runner sidecar <file>.sha256 of a file with dropped fields would reveal its original hash
        for rel in withheld:
            side = dst / (rel + ".sha256")
            if side.exists():
                side.unlink()
                rows.append(dict(path=rel + ".sha256", origin_sha256="withheld", sha256="", transform="omitted",
                                 detail="sidecar of a file with dropped fields"))
        if log is not None:
            log = Path(log)
            new = not log.exists()
            with open(log, "a", encoding="utf-8") as f:
                if new:
                    f.write("\t".join(LOG_FIELDS) + "\n")
                for r in rows:
                    f.write("\t".join(str(r[k]) for k in LOG_FIELDS) + "\n")
        return len(files), rows, labels


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="copy a results tree with named JSON fields replaced by their hash")
    ap.add_argument("--src", required=True)
    ap.add_argument("--dst", required=True)
    ap.add_argument("--log", required=True)
    ap.add_argument("--fields", default="")
    ap.add_argument("--drop-fields", default="")
    ap.add_argument("--redact", action="append", default=[], help="NAME=REGEX")
    ap.add_argument("--gzip", action="append", default=[])
    ap.add_argument("--exclude", action="append", default=[])
    a = ap.parse_args(argv)
    red = []
    for item in a.redact:
        name, sep, rx = item.partition("=")
        if not sep or not name:
            ap.error(f"--redact wants NAME=REGEX, got {item!r}")
        red.append((name, re.compile(rx)))
    s = Stripper(fields={f for f in a.fields.split(",") if f}, drop={f for f in a.drop_fields.split(",") if f},
                 redact=red, gzip_globs=a.gzip, exclude=a.exclude)
    try:
        n, rows, labels = s.copy_tree(a.src, a.dst, a.log)
    except ValueError as e:
        ap.error(str(e))
    print(f"copied {n} files, transformed {len(rows)}; distinct redacted values "
          f"{sum(len(v) for v in labels.values())}", file=sys.stderr)
    return 0


if __name__ == "__main__":
    sys.exit(main())
