"""Prompt sets derived from the locked RULER rows (the sets of code/kva/derived.py):

twokey  each row of ruler/niah_multikey_1_<L>.jsonl holds four keyed needles and asks one. Turn 1 is the row as
        RULER runs it; turn 2, asked on the carried cache, names one of the three other keys in RULER's one-key
        wording, chosen by random.Random(f"{SEED}:{sample id}").choice over them in document order. A row that
        does not hold four distinct keys with four distinct 7-digit values, one of them the answer, under RULER's
        question and answer prefix for it, is refused by name.
qfirst  each row of the four RULER NIAH tasks, reordered to instruction, question, document, with " for <query>"
        cut from the answer prefix so the keys appear only ahead of the document.

Only ids, row numbers, needle ordinals and sha256 pins are committed (the manifest); the prompts are rebuilt from
the locked rows at run time and each one is compared with its manifest entry before use. Sample ids are
ruler2k-<L>-<row:02d> and rulerqf-<task>-<L>-<row:02d>. The patterns below quote RULER's templates, which the
rows have to match, so they read as RULER writes them.
"""
from __future__ import annotations

import hashlib
import json
import os
import random
import re
from pathlib import Path

from . import locked as LK
from . import text as TX

SEED = 20261004
NIAH_STEPS = 128
SETS = ("twokey", "qfirst")
TWOKEY_TASK = "niah_multikey_1"
QFIRST_TASKS = ("niah_single_1", "niah_multikey_1", "niah_multivalue", "niah_multiquery")

# RULER's wording
NEEDLE = re.compile(r"One of the special magic numbers for ([^\n.:]+?) is: (\d+)\.")
QUESTION = "What is the special magic number for {key} mentioned in the provided text?"
PREFIX = " The special magic number for {key} mentioned in the provided text is"
QUERY = re.compile(r"What (?:is|are all) the special magic numbers? for (.+) mentioned in the provided text\?")
INSTRUCTION = re.compile(r"(Some|A) special magic numbers? (are|is) hidden within the following text\. Make sure to "
                         r"memorize it\. I will quiz you about the numbers? afterwards\.")
_SEVEN_DIGITS = re.compile(r"[0-9]{7}")
_PINNED = ("source", "source_sha256", "row_sha256", "text_sha256", "turn1_needle", "turn2_needle")


class DerivedRowError(ValueError):
    """A locked row does not have the structure its derived set is built from."""


class DerivedSetMismatch(SystemExit):
    """What the locked rows give differs from the committed manifest."""


def derived_dir():
    return Path(os.environ["RF_DERIVED_DIR"]) if os.environ.get("RF_DERIVED_DIR") else TX.data_root() / "derived"


def manifest_path(which):
    return derived_dir() / f"ruler-{which}.json"


def _digest(data: bytes):
    return hashlib.sha256(data).hexdigest()


def sources(which):
    names = [TWOKEY_TASK] if which == "twokey" else list(QFIRST_TASKS)
    return [f"ruler/{name}_{L}.jsonl" for name in names for L in LK.RULER_LENGTHS]


def _task_len(rel):
    stem = rel.removeprefix("ruler/").removesuffix(".jsonl")
    task, _, L = stem.rpartition("_")
    return task, int(L)


def sample_id(which, rel, row):
    task, L = _task_len(rel)
    if which == "twokey":
        return f"ruler2k-{L}-{row:02d}"
    return f"rulerqf-{task}-{L}-{row:02d}"


def needles(text):
    """(key, value, first char, end char) of each numeric needle of a RULER document, in order."""
    return [(m[1], m[2], *m.span()) for m in NEEDLE.finditer(text)]


def twokey(row, sid):
    found = needles(row["input"])
    keys = [f[0] for f in found]
    vals = [f[1] for f in found]
    shape_ok = (len(found) == 4 and len(set(keys)) == 4 and len(set(vals)) == 4
                and all(_SEVEN_DIGITS.fullmatch(v) for v in vals))
    if not shape_ok:
        raise DerivedRowError(f"{sid}: expected 4 needles with 4 distinct keys and 4 distinct 7-digit values, found "
                              f"{len(found)} needles, {len(set(keys))} keys, {len(set(vals))} values")
    answer = [j for j, v in enumerate(vals) if row["outputs"] == [v]]
    if len(answer) != 1:
        raise DerivedRowError(f"{sid}: the outputs field matches {len(answer)} needle values, not exactly one")
    first = answer[0]
    last_line = row["input"].split("\n")[-1]
    if last_line != QUESTION.format(key=keys[first]) or row["answer_prefix"] != PREFIX.format(key=keys[first]):
        raise DerivedRowError(f"{sid}: the question or answer prefix is not RULER's one-key template for the answer")
    others = [j for j in range(4) if j != first]
    second = random.Random(f"{SEED}:{sid}").choice(others)
    turns = [{"key": keys[j], "value": vals[j], "chars": (found[j][2], found[j][3])} for j in (first, second)]
    follow = {"question": QUESTION.format(key=keys[second]), "reply": PREFIX.format(key=keys[second])}
    return {"user": row["input"], "reply": row["answer_prefix"], "turns": turns, "turn1_needle": first,
            "turn2_needle": second, "ask": follow}


def question_first(row, sid):
    lines = row["input"].split("\n")
    head, question = lines[0], lines[-1]
    context = "\n".join(lines[1:-1])
    if len(lines) < 2 or INSTRUCTION.fullmatch(head) is None:
        raise DerivedRowError(f"{sid}: the row does not open with RULER's NIAH instruction")
    q = QUERY.fullmatch(question)
    if q is None or not context:
        raise DerivedRowError(f"{sid}: the row does not close with RULER's NIAH question after the document")
    cut = f" for {q[1]}"
    prefix = row["answer_prefix"]
    reply = prefix.replace(cut, "")
    if prefix.count(cut) != 1 or q[1] in reply:
        raise DerivedRowError(f"{sid}: the query's keys occur {prefix.count(cut)} times in the answer prefix")
    return {"user": "\n".join((head, question, context)), "reply": reply}


def build_one(which, row, sid):
    return (twokey if which == "twokey" else question_first)(row, sid)


def text_sha256(which, built):
    """Pin of the text a derived sample feeds the model: sha256 of the JSON list of its pieces."""
    pieces = [built["user"], built["reply"]]
    if which == "twokey":
        pieces.extend((built["ask"]["question"], built["ask"]["reply"]))
    return _digest(json.dumps(pieces, ensure_ascii=False).encode())


def _rows(root, rel):
    """(row number, raw line, parsed row) of a locked JSONL file, blank lines skipped."""
    lines = [ln for ln in (Path(root) / rel).read_text().splitlines() if ln.strip()]
    return [(i, ln, json.loads(ln)) for i, ln in enumerate(lines)]


def _frozen_sha(root):
    return json.loads((Path(root) / "FROZEN.json").read_text())["manifest_sha256"]


def _record(which, rel, sha, i, line, row, built, sid):
    entry = {"id": sid, "source": rel, "source_sha256": sha, "row": i, "index": row.get("index"),
             "length": _task_len(rel)[1], "row_sha256": _digest(line.encode()),
             "text_sha256": text_sha256(which, built)}
    if which == "twokey":
        entry["turn1_needle"] = built["turn1_needle"]
        entry["turn2_needle"] = built["turn2_needle"]
    return entry


def build_manifest(which, root=None):
    """The committed manifest of a derived set, from the locked rows (pins only, no text)."""
    if which not in SETS:
        raise ValueError(f"derived set {which!r} is not one of {SETS}")
    root = LK.locked_dir() if root is None else Path(root)
    locked = LK.manifest(root)
    samples = []
    for rel in (r for r in sources(which) if r in locked):
        sha = LK.source(rel, locked, root)
        for i, line, row in _rows(root, rel):
            sid = sample_id(which, rel, i)
            samples.append(_record(which, rel, sha, i, line, row, build_one(which, row, sid), sid))
    return {"set": f"ruler-{which}", "version": 1, "seed": SEED, "builder": "ridgefill_data_b200.eval.derived",
            "locked_manifest_sha256": _frozen_sha(root), "sources": sources(which), "count": len(samples),
            "samples": samples}


def dumps(manifest):
    return json.dumps(manifest, indent=1, ensure_ascii=False) + "\n"


def token_spans(tok, text, chars, ids, base):
    """Token range [first, last + 1) covering each character span of `text`, where text encoded on its own sits
    at ids[base:]; refused when ids do not hold that encoding there."""
    enc = tok(text, add_special_tokens=False, return_offsets_mapping=True)
    own = list(enc["input_ids"])
    if ids[base:base + len(own)] != own:
        raise DerivedSetMismatch("the prompt does not hold the text's own encoding where the needle offsets point")
    offsets = enc["offset_mapping"]
    spans = []
    for lo, hi in chars:
        touching = [t for t, (a, b) in enumerate(offsets) if a < hi and b > lo]
        if not touching:
            raise DerivedSetMismatch(f"no token covers characters [{lo}, {hi})")
        spans.append((base + touching[0], base + touching[-1] + 1))
    return spans


def token_span(tok, text, start, end, ids, base):
    (span,) = token_spans(tok, text, [(start, end)], ids, base)
    return span


def _load_manifest(which, root):
    path = manifest_path(which)
    if not path.is_file():
        raise DerivedSetMismatch(f"missing {path}: write it with build_manifest / dumps")
    m = json.loads(path.read_text())
    expected = (_frozen_sha(root), SEED, sources(which))
    if (m.get("locked_manifest_sha256"), m.get("seed"), m.get("sources")) != expected:
        raise DerivedSetMismatch(f"{path} pins a different locked set, seed or source list")
    return path, m


def _twokey_fields(tok, fmt, built, ids):
    if fmt == "chat":
        base, body = len(TX.chat_pieces(tok)[0]), built["user"]
    else:
        base, body = len(TX.bos_ids(tok)), built["user"] + built["reply"]
    plan = []
    for t in built["turns"]:
        lo, hi = token_span(tok, body, *t["chars"], ids, base)
        plan.append({"key": t["key"], "value": t["value"], "needle_start": lo, "needle_end": hi})
    head = plan[0]
    return dict(set="multiturn", turn_plan=plan, asks=[built["ask"]], key=head["key"], value=head["value"],
                needle_start=head["needle_start"], needle_end=head["needle_end"])


def prompts(which, tok, fmt, man, max_len=None, tasks=None, lengths=None, max_new=None, root=None):
    """(prompts, skipped source files) of a derived set; every prompt is checked against the manifest first."""
    root = LK.locked_dir() if root is None else Path(root)
    path, m = _load_manifest(which, root)
    pinned = {s["id"]: s for s in m["samples"]}
    tasks, lengths = LK.ruler_selection(tasks, lengths)
    caps = LK.check_max_new(max_new)
    chosen = [rel for rel in sources(which) if _task_len(rel)[0] in tasks and _task_len(rel)[1] in lengths]
    out, skipped, built_ids = [], [], set()
    for rel in chosen:
        task, L = _task_len(rel)
        if max_len and L > max_len:
            skipped.append(rel)
            continue
        sha = LK.source(rel, man, root)
        for i, line, row in _rows(root, rel):
            sid = sample_id(which, rel, i)
            try:
                built = build_one(which, row, sid)
            except DerivedRowError as e:
                raise DerivedSetMismatch(str(e)) from None
            want = pinned.get(sid)
            if want is None:
                raise DerivedSetMismatch(f"{sid} from {rel} has no entry in {path}")
            have = _record(which, rel, sha, i, line, row, built, sid)
            differ = [k for k in _PINNED if want.get(k) != have.get(k)]
            if differ:
                raise DerivedSetMismatch(f"{sid}: {', '.join(differ)} do not match {path}")
            built_ids.add(sid)
            ids = LK.wrap(tok, fmt, built["user"], built["reply"])
            q = dict(name=sid, task=task, ruler_task="niah", length=L, source=rel, source_sha256=sha, row=i,
                     index=row.get("index"), max_new=caps.get(task, NIAH_STEPS), format=fmt,
                     derived=f"ruler-{which}", derived_sha256=want["text_sha256"], ids=ids)
            if which == "qfirst":
                q.update(set="ruler", metric="string_match_all", refs=row["outputs"], variant="qfirst",
                         needles=LK.needle_spans(tok, fmt, built["user"], built["reply"], ids, row["outputs"], sid))
            else:
                q.update(_twokey_fields(tok, fmt, built, ids))
            out.append(q)
    live = set(chosen) - set(skipped)
    orphans = sorted(s["id"] for s in m["samples"] if s["source"] in live and s["id"] not in built_ids)
    if orphans:
        raise DerivedSetMismatch(f"{path} pins samples that the locked rows no longer give: {orphans[:5]}")
    return out, skipped


def pick_decode_docs(paths, n=20, max_len=32768, seed=SEED):
    """n long-prompt documents for the decode study: the manifest's long-prompts/*.txt files of at most max_len
    tokens, shuffled by random.Random(seed), then dealt round-robin from the length bins in ascending order.
    Returns lp-<file stem> names."""
    docs = [p for p in paths if p.startswith("long-prompts/") and p.endswith(".txt") and LK.doc_length(p) <= max_len]
    random.Random(seed).shuffle(docs)
    bins = {}
    for p in docs:
        bins.setdefault(LK.doc_length(p), []).append(p)
    queues = [bins[L] for L in sorted(bins)]
    picked = []
    while len(picked) < n and any(queues):
        for q in queues:
            if q and len(picked) < n:
                picked.append(q.pop(0))
    if len(picked) < n:
        raise ValueError(f"{n} long-prompt documents of at most {max_len} tokens wanted, {len(picked)} available")
    return ["lp-" + Path(p).stem for p in picked]
