"""Hash-chained pre-registration ledger (the ledger that tools/verify_ledger.py:1-44 checks and that the protocol
gate reads for registered hypothesis ids).

A ledger folder holds `ledger.jsonl` (one JSON object per line, canonical form: sorted keys, no spaces) and
`index.tsv` (columns seq, sha256, prev, time). Entry k carries `"seq": k` and `"prev"`: the sha256 of entry k-1's
line ("" for the first); its own sha256 is that of its line's UTF-8 bytes without the newline. Changing, dropping
or reordering any entry therefore breaks every later link. A release may publish only the entries it cites
(`cite()` writes `cited.jsonl`); they still verify against the full index.

    led = Ledger("provenance/ledger")
    led.append({"type": "hypothesis", "id": "H1", "text": "..."})
    verify("provenance/ledger")             # raises LedgerError naming the first bad row
    python -m ridgefill_data_b200.release.ledger verify provenance/ledger
"""
from __future__ import annotations

import csv
import fcntl
import hashlib
import json
import os
import sys
import time
from pathlib import Path

INDEX_FIELDS = ("seq", "sha256", "prev", "time")


class LedgerError(RuntimeError):
    pass


def canonical_line(obj):
    return json.dumps(obj, sort_keys=True, separators=(",", ":"), ensure_ascii=False)


def sha256_text(s):
    return hashlib.sha256(s.encode("utf-8")).hexdigest()


def read_index(folder):
    path = Path(folder) / "index.tsv"
    if not path.exists():
        return []
    with path.open(newline="", encoding="utf-8") as f:
        return list(csv.DictReader(f, delimiter="\t"))


class Ledger:
    def __init__(self, folder):
        self.folder = Path(folder)

    def append(self, entry, now=None):
        """Append one entry (a dict without seq / prev); returns (seq, sha256). Appends are serialised by a file
        lock, and both files are flushed to disk before the lock is released."""
        if "seq" in entry or "prev" in entry:
            raise LedgerError("an entry's seq and prev are set by the ledger")
        self.folder.mkdir(parents=True, exist_ok=True)
        with open(self.folder / ".lock", "w") as lock:
            fcntl.flock(lock, fcntl.LOCK_EX)
            index = read_index(self.folder)
            seq = len(index)
            prev = index[-1]["sha256"] if index else ""
            text = canonical_line({**entry, "seq": seq, "prev": prev})
            digest = sha256_text(text)
            stamp = time.strftime("%Y-%m-%dT%H:%M:%SZ", time.gmtime(now))
            new_index = not (self.folder / "index.tsv").exists()
            for name, row in (("ledger.jsonl", text + "\n"),
                              ("index.tsv", ("\t".join(INDEX_FIELDS) + "\n" if new_index else "")
                               + "\t".join([str(seq), digest, prev, stamp]) + "\n")):
                with open(self.folder / name, "a", encoding="utf-8") as f:
                    f.write(row)
                    f.flush()
                    os.fsync(f.fileno())
            return seq, digest

    def entries(self):
        path = self.folder / "ledger.jsonl"
        return [json.loads(s) for s in path.read_text(encoding="utf-8").splitlines() if s.strip()] \
            if path.exists() else []

    def cite(self, seqs, dst=None):
        """Write the lines of the cited entries (in seq order) to `cited.jsonl` (or dst); returns the path."""
        want = set(int(s) for s in seqs)
        lines = [s for s in (self.folder / "ledger.jsonl").read_text(encoding="utf-8").splitlines()
                 if s.strip() and json.loads(s)["seq"] in want]
        dst = Path(dst) if dst else self.folder / "cited.jsonl"
        dst.write_text("".join(s + "\n" for s in lines), encoding="utf-8")
        return dst


def verify(folder, lines_file=None):
    """Check the chain: index seq 0..N-1 with each prev equal to the previous sha256, and every line of the entries
    file (ledger.jsonl, or cited.jsonl when only that is present, or `lines_file`) hashing to its index row with a
    matching seq / prev. Returns (entries in the index, lines checked)."""
    folder = Path(folder)
    index = read_index(folder)
    if not index:
        raise LedgerError(f"{folder}: no index.tsv rows")
    for i, row in enumerate(index):
        if int(row["seq"]) != i:
            raise LedgerError(f"index row {i}: seq {row['seq']}")
        if row["prev"] != (index[i - 1]["sha256"] if i else ""):
            raise LedgerError(f"index seq {i}: prev does not equal the sha256 of seq {i - 1}")
    if lines_file is None:
        lines_file = folder / "ledger.jsonl"
        if not lines_file.exists():
            lines_file = folder / "cited.jsonl"
    checked, last = 0, -1
    for s in Path(lines_file).read_text(encoding="utf-8").splitlines():
        if not s.strip():
            continue
        e = json.loads(s)
        seq = e.get("seq")
        if not isinstance(seq, int) or not 0 <= seq < len(index):
            raise LedgerError(f"{lines_file}: entry with seq {seq!r} outside the index")
        if seq <= last:
            raise LedgerError(f"{lines_file}: seq {seq} out of order")
        last = seq
        if sha256_text(s) != index[seq]["sha256"]:
            raise LedgerError(f"{lines_file}: seq {seq}: the line's sha256 differs from the index")
        if (e.get("prev") or "") != index[seq]["prev"]:
            raise LedgerError(f"{lines_file}: seq {seq}: prev differs from the index")
        checked += 1
    return len(index), checked


def main(argv=None):
    import argparse
    ap = argparse.ArgumentParser(description="hash-chained ledger")
    sub = ap.add_subparsers(dest="cmd", required=True)
    v = sub.add_parser("verify")
    v.add_argument("folder")
    v.add_argument("--lines")
    ad = sub.add_parser("append")
    ad.add_argument("folder")
    ad.add_argument("json", help="the entry as a JSON object")
    a = ap.parse_args(argv)
    if a.cmd == "append":
        seq, digest = Ledger(a.folder).append(json.loads(a.json))
        print(f"{seq}\t{digest}")
        return 0
    try:
        n, k = verify(a.folder, a.lines)
    except LedgerError as e:
        print(f"FAIL {e}")
        return 1
    print(f"PASS chain of {n} entries; {k} lines match their index hashes")
    return 0


if __name__ == "__main__":
    sys.exit(main())
