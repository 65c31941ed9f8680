"""Secret and privacy scan of a release tree (tools/scrub_check.py:1-170). Reports path:line and the rule name only,
never the matched text.

Every file outside `.git` is read line by line (`.gz` decompressed; files with a NUL byte in their first 8 KB are
binary and only get the file-level checks). Line rules: credential forms, private-key headers, home-directory
paths, GPU UUIDs, PCI bus ids, e-mail addresses, plus RULE<TAB>REGEX lines of unpublished local pattern files
(--private). File rules: forbidden names (keys, env files, pickles, raw tensors), files above the size limit, and
JSON under results/ or derived/ that still holds a prompt field. A hit passes only when a row of the allowlist
(a Markdown table | path glob | RULE | reason |, the reason at least 10 characters) names its path and rule; an
allowlist row that matches nothing is stale and fails the scan, so no exemption outlives its reason.

Exit status: 0 clean, 1 unallowed hits, 2 bad arguments or a malformed / stale allowlist.
"""
from __future__ import annotations

import fnmatch
import gzip
import re
import sys
from dataclasses import dataclass, field
from pathlib import Path

LINE_RULES = {
    "PRIVATE_KEY": r"-----BEGIN (?:RSA |EC |DSA |OPENSSH |ENCRYPTED )?PRIVATE KEY-----",
    "HF_TOKEN": r"\bhf_[A-Za-z0-9]{30,}\b",
    "GITHUB_TOKEN": r"\bgh[pousr]_[A-Za-z0-9]{30,}\b|\bgithub_pat_\w{40,}\b",
    "API_KEY": r"\bsk-[A-Za-z0-9_-]{20,}|\bAIza[0-9A-Za-z_-]{35}\b|\bxox[abprs]-[A-Za-z0-9-]{10,}",
    "AWS_KEY": r"\b(?:AKIA|ASIA)[0-9A-Z]{16}\b",
    "SECRET_ASSIGN": r"\b[A-Z][A-Z0-9_]*(?:TOKEN|API_KEY|SECRET|PASSWORD)\s*[=:]\s*['\"]?[^\s'\"$<{]{6,}",
    "HOME_PATH": r"/home/[A-Za-z0-9._-]+/|/Users/[A-Za-z0-9._-]+/",
    "GPU_UUID": r"\bGPU-[0-9a-fA-F]{8}(?:-[0-9a-fA-F]{4}){3}-[0-9a-fA-F]{12}\b",
    "PCI_ID": r"\b[0-9a-fA-F]{4,8}:[0-9a-fA-F]{2}:[0-9a-fA-F]{2}\.[0-7]\b",
    "EMAIL": r"\b[A-Za-z0-9][A-Za-z0-9._%+-]*@[A-Za-z0-9-]+(?:\.[A-Za-z0-9-]+)*\.[A-Za-z]{2,}\b",
}
FILE_RULES = ("FORBIDDEN_FILE", "BIG_FILE", "UNSTRIPPED_PROMPT")
FORBIDDEN = (".env", "*.env", "id_rsa*", "id_ed25519*", "*.pem", "*.key", ".netrc", "*.pkl", "*.pickle", "*.pt",
             "*.npy")
PROMPT_KEY = re.compile(r'"(?:prompt|messages|context|input)"\s*:\s*["\[]')


class ScrubError(ValueError):
    pass


@dataclass
class Allow:
    glob: str
    rule: str
    reason: str
    line: int
    used: int = 0


@dataclass
class Scan:
    rules: dict = field(default_factory=lambda: dict(LINE_RULES))
    allow: list = field(default_factory=list)
    max_bytes: int = 50 << 20
    private_loaded: int = 0

    def add_private(self, path):
        for n, s in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), 1):
            if not s.strip() or s.startswith("#"):
                continue
            rule, sep, rx = s.partition("\t")
            if not sep or not re.fullmatch(r"[A-Z][A-Z0-9_]*", rule) or rule in self.rules or rule in FILE_RULES:
                raise ScrubError(f"{path}:{n}: expected a new RULE<TAB>REGEX line")
            re.compile(rx)
            self.rules[rule] = rx
            self.private_loaded += 1

    def load_allowlist(self, path):
        for n, s in enumerate(Path(path).read_text(encoding="utf-8").splitlines(), 1):
            if not s.lstrip().startswith("|"):
                continue
            cells = [c.strip() for c in s.strip().strip("|").split("|")]
            if len(cells) != 3 or set(cells[0]) <= set("-: ") or cells[0].lower() == "path glob":
                continue
            glob, rule, reason = cells[0].strip("`"), cells[1], cells[2]
            if rule not in self.rules and rule not in FILE_RULES:
                if self.private_loaded:
                    raise ScrubError(f"allowlist line {n}: unknown rule {rule!r}")
                continue      # an exemption for a private rule that is not loaded in this (public) scan
            if len(reason) < 10:
                raise ScrubError(f"allowlist line {n}: the reason for {glob} {rule} is too short")
            self.allow.append(Allow(glob, rule, reason, n))

    def combined(self):
        return re.compile("|".join(f"(?P<{k}>{v})" for k, v in self.rules.items()))

    def file_hits(self, rel, path, rx):
        hits = []
        if any(fnmatch.fnmatch(path.name, g) for g in FORBIDDEN):
            hits.append((0, "FORBIDDEN_FILE"))
        if path.stat().st_size > self.max_bytes:
            hits.append((0, "BIG_FILE"))
        data = path.read_bytes()
        if path.suffix == ".gz":
            try:
                data = gzip.decompress(data)
            except OSError:
                return hits
        if b"\0" in data[:8192]:
            return hits
        prompts = rel.startswith(("results/", "derived/")) and ".json" in path.name
        for n, s in enumerate(data.decode("utf-8", errors="replace").splitlines(), 1):
            for rule in sorted({m.lastgroup for m in rx.finditer(s)}):
                hits.append((n, rule))
            if prompts and PROMPT_KEY.search(s):
                hits.append((n, "UNSTRIPPED_PROMPT"))
        return hits

    def run(self, root, skip=()):
        root = Path(root)
        if not root.is_dir():
            raise ScrubError(f"{root} is not a directory")
        rx = self.combined()
        skip = {Path(p).resolve() for p in skip}
        files = sorted(p for p in root.rglob("*") if p.is_file() and ".git" not in p.relative_to(root).parts
                       and p.resolve() not in skip)
        hits, allowed = [], []
        for p in files:
            rel = p.relative_to(root).as_posix()
            for n, rule in self.file_hits(rel, p, rx):
                where = f"{rel}:{n}" if n else rel
                row = next((a for a in self.allow if a.rule == rule and fnmatch.fnmatch(rel, a.glob)), None)
                if row is None:
                    hits.append((where, rule))
                else:
                    row.used += 1
                    allowed.append((where, rule, row.line))
        stale = [a for a in self.allow if a.used == 0]
        return Report(len(files), hits, allowed, stale, self.private_loaded)


@dataclass
class Report:
    files: int
    hits: list
    allowed: list
    stale: list
    private_loaded: int

    @property
    def status(self):
        return 2 if self.stale else (1 if self.hits else 0)

    def lines(self):
        out = [f"HIT      {w}  {r}" for w, r in self.hits]
        out += [f"ALLOWED  {w}  {r}  (allowlist line {n})" for w, r, n in self.allowed]
        out += [f"STALE    allowlist line {a.line}: {a.glob} {a.rule} matched nothing" for a in self.stale]
        out.append(f"files {self.files}; unallowed hits {len(self.hits)}; allowed {len(self.allowed)}; "
                   f"stale allowlist rows {len(self.stale)}; private rules loaded {self.private_loaded}")
        return out


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="secret and privacy scan of a release tree")
    ap.add_argument("root")
    ap.add_argument("--allowlist", required=True)
    ap.add_argument("--private", action="append", default=[], help="RULE<TAB>REGEX pattern file (unpublished)")
    ap.add_argument("--max-size-mib", type=float, default=50)
    ap.add_argument("--report")
    a = ap.parse_args(argv)
    try:
        scan = Scan(max_bytes=int(a.max_size_mib * (1 << 20)))
        for p in a.private:
            scan.add_private(p)
        scan.load_allowlist(a.allowlist)
        rep = scan.run(a.root, skip=[a.allowlist, __file__])
    except (ScrubError, OSError, re.error) as e:
        print(e, file=sys.stderr)
        return 2
    text = "\n".join(rep.lines()) + "\n"
    if a.report:
        Path(a.report).write_text(text, encoding="utf-8")
    print(rep.lines()[-1])
    return rep.status


if __name__ == "__main__":
    sys.exit(main())
