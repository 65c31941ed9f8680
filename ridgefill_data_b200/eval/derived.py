"""Prompt sets derived from locked RULER rows (code/kva/derived.py): a second question on a cached prefix
(twokey) and the question placed before the document (qfirst). Manifests hold ids, row numbers, needle ordinals
and sha256 hashes only; prompts are rebuilt from the locked rows at run time and every sample is checked against
its manifest entry first.

twokey  every row of ruler/niah_multikey_1_<L>.jsonl (4 keyed needles, one asked). Turn 1 is the row as RULER runs
        it; turn 2 asks one of the other three keys, random.Random(f"{SEED}:{sample id}").choice over them in
        document order, in RULER's one-key wording. Rows without exactly 4 distinct keys and 4 distinct 7-digit
        values, one of them the answer, and RULER's question / prefix for it, are refused by name.
qfirst  every row of the 4 RULER NIAH tasks: instruction \\n question \\n context, and the answer prefix without
        " for <query>", so the keys appear only before the document.
Sample ids: ruler2k-<L>-<row:02d> and rulerqf-<task>-<L>-<row:02d>. The wording regexes follow RULER's templates
(they have to match RULER's text).
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
NEEDLE = re.compile(r"One of the special magic numbers for ([^\n.:]+?) is: (\d+)\.")
QUESTION = "What is the special magic number for {key} mentioned in the provided text?"
PREFIX = " The special magic number for {key} mentioned in the provided text is"
QUERY = re.compile(r"What (?:is|are all) the special magic numbers? for (.+) mentioned in the provided text\?")
INSTRUCTION = re.compile(r"(Some|A) special magic numbers? (are|is) hidden within the following text\. Make sure to "
                         r"memorize it\. I will quiz you about the numbers? afterwards\.")
TWOKEY_TASK = "niah_multikey_1"
QFIRST_TASKS = ("niah_single_1", "niah_multikey_1", "niah_multivalue", "niah_multiquery")
NIAH_STEPS = 128
SETS = ("twokey", "qfirst")


class DerivedRowError(ValueError):
    """A locked row lacks the structure a derived set needs."""


class DerivedSetMismatch(SystemExit):
    """The rebuilt prompts do not match the committed manifest."""


def derived_dir():
    env = os.environ.get("RF_DERIVED_DIR")
    return Path(env) if env else TX.data_root() / "derived"


def manifest_path(which):
    return derived_dir() / f"ruler-{which}.json"


def _sha(obj):
    return hashlib.sha256(json.dumps(obj, ensure_ascii=False).encode()).hexdigest()


def sources(which):
    tasks = (TWOKEY_TASK,) if which == "twokey" else QFIRST_TASKS
    return [f"ruler/{t}_{L}.jsonl" for t in tasks for L in LK.RULER_LENGTHS]


def _task_len(rel):
    task, L = rel[len("ruler/"):-len(".jsonl")].rsplit("_", 1)
    return task, int(L)


def sample_id(which, rel, row):
    task, L = _task_len(rel)
    return f"ruler2k-{L}-{row:02d}" if which == "twokey" else f"rulerqf-{task}-{L}-{row:02d}"


def needles(text):
    """[(key, value, char start, char end)] of RULER's numeric needles, in document order."""
    return [(m.group(1), m.group(2), m.start(), m.end()) for m in NEEDLE.finditer(text)]


def twokey(row, sid):
    ns = needles(row["input"])
    keys, values = [n[0] for n in ns], [n[1] for n in ns]
    if len(ns) != 4 or len(set(keys)) != 4 or len(set(values)) != 4 or not all(re.fullmatch(r"\d{7}", v) for v in values):
        raise DerivedRowError(f"{sid}: needs 4 needles with distinct keys and distinct 7-digit values "
                              f"({len(ns)} needles, {len(set(keys))} keys, {len(set(values))} values)")
    asked = [j for j, v in enumerate(values) if [v] == row["outputs"]]
    if len(asked) != 1:
        raise DerivedRowError(f"{sid}: outputs is not exactly one needle's value ({len(asked)} matches)")
    t = asked[0]
    if row["input"].rsplit("\n", 1)[-1] != QUESTION.format(key=keys[t]) or row["answer_prefix"] != PREFIX.format(key=keys[t]):
        raise DerivedRowError(f"{sid}: question line or answer prefix is not RULER's one-key wording for the asked key")
    u = random.Random(f"{SEED}:{sid}").choice([j for j in range(4) if j != t])
    turns = [dict(key=keys[j], value=values[j], chars=(ns[j][2], ns[j][3])) for j in (t, u)]
    return dict(user=row["input"], reply=row["answer_prefix"], turns=turns, turn1_needle=t, turn2_needle=u,
                ask=dict(question=QUESTION.format(key=keys[u]), reply=PREFIX.format(key=keys[u])))


def question_first(row, sid):
    head, _, rest = row["input"].partition("\n")
    context, _, question = rest.rpartition("\n")
    if not INSTRUCTION.fullmatch(head):
        raise DerivedRowError(f"{sid}: the first line is not RULER's NIAH instruction")
    q = QUERY.fullmatch(question)
    if q is None or not context:
        raise DerivedRowError(f"{sid}: the last line is not RULER's NIAH question after a document")
    tag = f" for {q.group(1)}"
    reply = row["answer_prefix"].replace(tag, "")
    if row["answer_prefix"].count(tag) != 1 or q.group(1) in reply:
        raise DerivedRowError(f"{sid}: the answer prefix does not carry the question's keys exactly once")
    return dict(user=f"{head}\n{question}\n{context}", reply=reply)


def build_one(which, row, sid):
    return twokey(row, sid) if which == "twokey" else question_first(row, sid)


def text_sha256(which, built):
    parts = [built["user"], built["reply"]]
    if which == "twokey":
        parts += [built["ask"]["question"], built["ask"]["reply"]]
    return _sha(parts)


def _lines(rel, root):
    return [line for line in (root / rel).read_text().splitlines() if line.strip()]


def _frozen_sha(root):
    return json.loads((root / "FROZEN.json").read_text())["manifest_sha256"]


def _record(which, rel, sha, i, line, row, built, sid):
    s = dict(id=sid, source=rel, source_sha256=sha, row=i, index=row.get("index"), length=_task_len(rel)[1],
             row_sha256=hashlib.sha256(line.encode()).hexdigest(), text_sha256=text_sha256(which, built))
    if which == "twokey":
        s.update(turn1_needle=built["turn1_needle"], turn2_needle=built["turn2_needle"])
    return s


def build_manifest(which, root=None):
    """The manifest of a derived set from the locked rows (no text inside)."""
    if which not in SETS:
        raise ValueError(f"unknown derived set {which!r}: one of {SETS}")
    root = Path(root) if root is not None else LK.locked_dir()
    man = LK.manifest(root)
    samples = []
    for rel in sources(which):
        if rel not in man:
            continue
        sha = LK.source(rel, man, root)
        for i, line in enumerate(_lines(rel, root)):
            row, sid = json.loads(line), sample_id(which, rel, i)
            samples.append(_record(which, rel, sha, i, line, row, build_one(which, row, sid), sid))
    return dict(set=f"ruler-{which}", version=1, seed=SEED, builder="ridgefill_data_b200.eval.derived",
                locked_manifest_sha256=_frozen_sha(root), sources=sources(which), count=len(samples), samples=samples)


def dumps(manifest):
    return json.dumps(manifest, indent=1, ensure_ascii=False) + "\n"


def token_spans(tok, text, chars, ids, base):
    """[first, last + 1) of the tokens of `text` (encoded alone, placed at ids[base:]) overlapping each character
    span of `chars`; refuses when that encoding is not the one in ids."""
    enc = tok(text, add_special_tokens=False, return_offsets_mapping=True)
    got = list(enc["input_ids"])
    if ids[base:base + len(got)] != got:
        raise DerivedSetMismatch("the prompt's token ids are not the text's encoding (tokenizer offsets)")
    out = []
    for start, end in chars:
        hit = [i for i, (s, e) in enumerate(enc["offset_mapping"]) if s < end and e > start]
        if not hit:
            raise DerivedSetMismatch("a needle maps to no token")
        out.append((base + hit[0], base + hit[-1] + 1))
    return out


def token_span(tok, text, start, end, ids, base):
    return token_spans(tok, text, [(start, end)], ids, base)[0]


def prompts(which, tok, fmt, man, max_len=None, tasks=None, lengths=None, max_new=None, root=None):
    """(prompts, skipped files) of a derived set, every sample checked against its manifest."""
    root = Path(root) if root is not None else LK.locked_dir()
    path = manifest_path(which)
    if not path.is_file():
        raise DerivedSetMismatch(f"{path} does not exist (build_manifest writes it)")
    m = json.loads(path.read_text())
    if m.get("locked_manifest_sha256") != _frozen_sha(root) or m.get("seed") != SEED or m.get("sources") != sources(which):
        raise DerivedSetMismatch(f"{path} was built from another locked set, seed or source list")
    by_id = {s["id"]: s for s in m["samples"]}
    tasks, lengths = LK.ruler_selection(tasks, lengths)
    caps = LK.check_max_new(max_new)
    chosen = [rel for rel in sources(which) if _task_len(rel)[0] in tasks and _task_len(rel)[1] in lengths]
    out, skipped, seen = [], [], set()
    for rel in chosen:
        task, L = _task_len(rel)
        if max_len and L > max_len:
            skipped.append(rel)
            continue
        sha = LK.source(rel, man, root)
        for i, line in enumerate(_lines(rel, root)):
            row, sid = json.loads(line), sample_id(which, rel, i)
            try:
                built = build_one(which, row, sid)
            except DerivedRowError as e:
                raise DerivedSetMismatch(str(e))
            want = by_id.get(sid)
            got = _record(which, rel, sha, i, line, row, built, sid)
            if want is None:
                raise DerivedSetMismatch(f"{sid} ({rel}) is not in {path}")
            bad = [k for k in ("source", "source_sha256", "row_sha256", "text_sha256", "turn1_needle", "turn2_needle")
                   if want.get(k) != got.get(k)]
            if bad:
                raise DerivedSetMismatch(f"{sid}: {', '.join(bad)} differ from {path}")
            seen.add(sid)
            ids = LK.wrap(tok, fmt, built["user"], built["reply"])
            q = dict(name=sid, task=task, ruler_task="niah", length=L, source=rel, source_sha256=sha, row=i,
                     index=row.get("index"), max_new=caps.get(task, NIAH_STEPS), format=fmt, derived=f"ruler-{which}",
                     derived_sha256=want["text_sha256"], ids=ids)
            if which == "qfirst":
                q.update(set="ruler", metric="string_match_all", refs=row["outputs"], variant="qfirst",
                         needles=LK.needle_spans(tok, fmt, built["user"], built["reply"], ids, row["outputs"], sid))
            else:
                if fmt == "chat":
                    base, body = len(TX.chat_pieces(tok)[0]), built["user"]
                else:
                    base, body = len(TX.bos_ids(tok)), built["user"] + built["reply"]
                plan = []
                for t in built["turns"]:
                    s, e = token_span(tok, body, *t["chars"], ids, base)
                    plan.append(dict(key=t["key"], value=t["value"], needle_start=s, needle_end=e))
                q.update(set="multiturn", turn_plan=plan, asks=[built["ask"]], key=plan[0]["key"],
                         value=plan[0]["value"], needle_start=plan[0]["needle_start"], needle_end=plan[0]["needle_end"])
            out.append(q)
    extra = sorted(s["id"] for s in m["samples"] if s["source"] in chosen and s["source"] not in skipped
                   and s["id"] not in seen)
    if extra:
        raise DerivedSetMismatch(f"{path} lists samples the locked rows do not have: {extra[:5]}")
    return out, skipped


def pick_decode_docs(paths, n=20, max_len=32768, seed=SEED):
    """Long-prompt documents for the decode study: the manifest's long-prompt files up to max_len, shuffled by
    random.Random(seed), taken round-robin over the length bins (ascending) until n. Returns lp-<stem> names."""
    docs = [p for p in paths if p.startswith("long-prompts/") and p.endswith(".txt")]
    docs = [p for p in docs if LK.doc_length(p) <= max_len]
    random.Random(seed).shuffle(docs)
    bins = {L: [p for p in docs if LK.doc_length(p) == L] for L in sorted({LK.doc_length(p) for p in docs})}
    picked = []
    while len(picked) < n and any(bins.values()):
        for L in bins:
            if bins[L] and len(picked) < n:
                picked.append(bins[L].pop(0))
    if len(picked) < n:
        raise ValueError(f"only {len(picked)} long-prompt documents <= {max_len} tokens, {n} wanted")
    return ["lp-" + p.rsplit("/", 1)[-1][:-len(".txt")] for p in picked]
