"""The locked test sets (code/kva/locked.py): RULER, LongBench v1 and long-prompt NLL prompts built from a frozen
directory, every file checked against its manifest before anything runs.

Layout of a set directory (RF_LOCKED_DIR, default <data root>/test-set-locked):
  FROZEN.json              {"manifest_sha256": sha256 of MANIFEST.tsv}
  MANIFEST.tsv             path, sha256, domain/task (tab separated)
  ruler/<task>_<L>.jsonl   RULER rows: input, answer_prefix, outputs, index
  longbench/<task>.jsonl   LongBench rows: context, input, answers, all_classes, length, dataset, _id
  longbench/dataset2prompt.json, dataset2maxlen.json   LongBench's own prompt templates / generation budgets
  long-prompts/SPLITS.tsv + long-prompts/*_<L>_<k>.txt  documents with the prompt / continuation split point

ruler      prompt = RULER input then its answer_prefix (raw: BOS + the joined text; chat: input as the user turn,
           answer_prefix opening the reply); greedy up to RULER's tokens_to_generate; scored by string_match_all
           (niah, vt, cwe, fwe) or string_match_part (qa). NIAH rows also carry the token spans of the needles they
           score (for the filled-region readout).
longbench  LongBench v1 pred.py: template, middle truncation to max_len tokens (half from each end, decoded and
           joined), chat template except trec / lcc / repobench-p; greedy up to the task's budget; official metric.
longppl    BOS + text[:split_char] + text[split_char:] (each part encoded alone); score = NLL of every continuation
           token; the novel-token mask as the graded set's.
The task table (RULER's tokens_to_generate and metrics) is kept as RULER defines it so scores compare.
"""
from __future__ import annotations

import csv
import hashlib
import json
import os
from pathlib import Path

from . import metrics as MT
from . import text as TX

SETS = ("ruler", "longbench", "longppl")
GEN_SETS = ("ruler", "longbench")
RULER_TASKS = {            # task: (RULER kind, tokens_to_generate, metric)
    "niah_single_1": ("niah", 128, "string_match_all"),
    "niah_multikey_1": ("niah", 128, "string_match_all"),
    "niah_multivalue": ("niah", 128, "string_match_all"),
    "niah_multiquery": ("niah", 128, "string_match_all"),
    "vt": ("variable_tracking", 30, "string_match_all"),
    "cwe": ("common_words_extraction", 120, "string_match_all"),
    "fwe": ("freq_words_extraction", 50, "string_match_all"),
    "qa_1": ("qa", 32, "string_match_part"),
}
RULER_LENGTHS = (8192, 16384, 32768, 65536)
LONGBENCH_NO_CHAT = ("trec", "triviaqa", "samsum", "lsht", "lcc", "repobench-p")


class LockedSetError(SystemExit):
    """The set on disk is not the frozen one (or a request names something it does not hold)."""


def locked_dir():
    env = os.environ.get("RF_LOCKED_DIR")
    return Path(env) if env else TX.data_root() / "test-set-locked"


def _sha256(path):
    with open(path, "rb") as f:
        return hashlib.file_digest(f, "sha256").hexdigest()


def manifest(root=None, pin=None, name="the locked set"):
    """{relative path: {sha256, domain}} from MANIFEST.tsv once it matches FROZEN.json (and `pin` when given)."""
    root = Path(root) if root is not None else locked_dir()
    path, frozen = root / "MANIFEST.tsv", root / "FROZEN.json"
    if not path.is_file() or not frozen.is_file():
        raise LockedSetError(f"{name}: {root} has no MANIFEST.tsv / FROZEN.json")
    got = _sha256(path)
    if got != json.loads(frozen.read_text())["manifest_sha256"]:
        raise LockedSetError(f"{path} does not match FROZEN.json: {name} changed")
    if pin is not None and got != pin:
        raise LockedSetError(f"{name}: MANIFEST.tsv hashes to {got}, the config pins {pin}")
    with path.open() as f:
        return {r["path"]: dict(sha256=r["sha256"], domain=r["domain/task"].split("/")[0])
                for r in csv.DictReader(f, delimiter="\t")}


def source(rel, man, root=None):
    """A file's manifest sha256 after checking the file still has it."""
    root = Path(root) if root is not None else locked_dir()
    if rel not in man:
        raise LockedSetError(f"{rel} is not in the MANIFEST.tsv of {root}")
    if _sha256(root / rel) != man[rel]["sha256"]:
        raise LockedSetError(f"{root / rel} does not match its MANIFEST.tsv sha256")
    return man[rel]["sha256"]


def rows(rel, root=None):
    root = Path(root) if root is not None else locked_dir()
    return [json.loads(line) for line in (root / rel).read_text().splitlines() if line.strip()]


def wrap(tok, fmt, user, reply=""):
    """raw: BOS + user + reply as one text; chat: user as the user turn (thinking off), reply opening the reply."""
    if fmt == "raw":
        return TX.bos_ids(tok) + TX.encode(tok, user + reply)
    if fmt == "chat":
        head, reply_open = TX.chat_pieces(tok)
        return head + TX.encode(tok, user) + reply_open + (TX.encode(tok, reply) if reply else [])
    raise ValueError(f"unknown format {fmt!r}")


def fmt_of(cfg, model, protocol):
    """The prompt format: the protocol's niah_format for the model, else the config's; never both disagreeing."""
    want = protocol.get("models", {}).get(model, {}).get("niah_format")
    got = cfg.get("niah_format")
    if want and got and want != got:
        raise LockedSetError(f"config niah_format {got!r} differs from the protocol's {want!r} for {model}")
    if not (want or got):
        raise LockedSetError(f"no niah_format for {model} in the protocol or the config")
    return want or got


def check_max_new(max_new):
    """{task: tokens} that only LOWERS RULER's tokens_to_generate for named RULER tasks."""
    if max_new is None:
        return {}
    caps = dict(max_new)

    def allowed(task, v):
        return task in RULER_TASKS and type(v) is int and 0 < v <= RULER_TASKS[task][1]
    bad = {t: v for t, v in caps.items() if not allowed(t, v)}
    if bad:
        raise LockedSetError(f"ruler_max_new {bad}: each cap names a RULER task and lowers its tokens_to_generate")
    return caps


def ruler_selection(tasks=None, lengths=None):
    tasks = list(RULER_TASKS if tasks is None else tasks)
    lengths = list(RULER_LENGTHS if lengths is None else lengths)
    bad = [t for t in tasks if t not in RULER_TASKS]
    bad += [L for L in lengths if L not in RULER_LENGTHS]
    if bad or not (tasks and lengths):
        raise LockedSetError(f"ruler_tasks / ruler_lengths: {bad or 'empty'} not RULER's")
    return tasks, lengths


class NeedleSpanError(ValueError):
    """A NIAH row whose scored values are not each found exactly once among its needles."""


def needle_spans(tok, fmt, user, reply, ids, refs, name):
    """Token spans [start, end) of the numeric needles whose value a NIAH row scores, in document order."""
    from . import derived
    hits = [(value, lo, hi) for _, value, lo, hi in derived.needles(user) if value in refs]
    if sorted(h[0] for h in hits) != sorted(refs):
        raise NeedleSpanError(f"{name}: its {len(refs)} scored values are not each found exactly once among its "
                              f"needles ({len(hits)} carry one)")
    if fmt == "chat":
        text, base = user, len(TX.chat_pieces(tok)[0])
    else:
        text, base = user + reply, len(TX.bos_ids(tok))
    spans = derived.token_spans(tok, text, [(lo, hi) for _, lo, hi in hits], ids, base)
    return [[a, b] for a, b in spans]


def ruler_prompts(tok, fmt, man, max_len=None, tasks=None, lengths=None, max_new=None, root=None):
    out, skipped = [], []
    tasks, lengths = ruler_selection(tasks, lengths)
    caps = check_max_new(max_new)
    for task in (t for t in RULER_TASKS if t in tasks):
        kind, steps, metric = RULER_TASKS[task]
        for L in (x for x in RULER_LENGTHS if x in lengths):
            rel = f"ruler/{task}_{L}.jsonl"
            if max_len and L > max_len:
                skipped.append(rel)
                continue
            sha = source(rel, man, root)
            for i, r in enumerate(rows(rel, root)):
                name = f"ruler-{task}-{L}-{i:02d}"
                user, reply = r["input"], r["answer_prefix"]
                ids = wrap(tok, fmt, user, reply)
                q = {"name": name, "set": "ruler", "task": task, "ruler_task": kind, "length": L, "source": rel,
                     "source_sha256": sha, "row": i, "index": r.get("index"), "max_new": caps.get(task, steps),
                     "metric": metric, "refs": r["outputs"], "format": fmt, "ids": ids}
                if kind == "niah":
                    q["needles"] = needle_spans(tok, fmt, user, reply, ids, r["outputs"], name)
                out.append(q)
    return out, skipped


def middle_truncate(tok, prompt, max_len):
    """LongBench pred.py: over max_len tokens (default special tokens), keep the first and last int(max_len / 2)
    tokens, each half decoded without special tokens, joined as text."""
    ids = tok(prompt).input_ids
    if len(ids) <= max_len:
        return prompt, False
    keep = int(max_len / 2)
    head = tok.decode(ids[:keep], skip_special_tokens=True)
    tail = tok.decode(ids[len(ids) - keep:], skip_special_tokens=True)
    return head + tail, True


def longbench_prompts(tok, fmt, man, max_len, root=None):
    if not max_len:
        raise LockedSetError("longbench needs longbench_max_len (LongBench's middle-truncation length)")
    root = Path(root) if root is not None else locked_dir()
    try:
        templates = json.loads((root / "longbench" / "dataset2prompt.json").read_text())
        budgets = json.loads((root / "longbench" / "dataset2maxlen.json").read_text())
    except FileNotFoundError as e:
        raise LockedSetError(f"longbench: {e.filename} missing (LongBench's config files belong beside its rows)")
    out = []
    for task in sorted(t for t in templates if f"longbench/{t}.jsonl" in man):
        rel = f"longbench/{task}.jsonl"
        sha = source(rel, man, root)
        for i, r in enumerate(rows(rel, root)):
            if r["dataset"] != task:
                raise LockedSetError(f"{rel} row {i} is from {r['dataset']!r}")
            prompt, cut = middle_truncate(tok, templates[task].format(**r), max_len)
            row_fmt = fmt if task not in LONGBENCH_NO_CHAT else "raw"
            q = {"name": f"lb-{task}-{i:02d}", "set": "longbench", "task": task, "length": r.get("length"),
                 "source": rel, "source_sha256": sha, "row": i, "id": r.get("_id"), "max_new": budgets[task],
                 "metric": MT.LONGBENCH_METRIC[task].__name__, "refs": r["answers"],
                 "all_classes": r.get("all_classes"), "truncated": cut, "format": row_fmt}
            q["ids"] = wrap(tok, row_fmt, prompt)
            out.append(q)
    return out, []


def splits_column(model, columns):
    """The SPLITS.tsv token-count column whose tokenizer name prefixes the model's, or None."""
    prefix = "prompt_tokens_"
    names = [c.removeprefix(prefix) for c in columns if c.startswith(prefix)]
    matching = sorted((k for k in names if model.startswith(k)), key=len)
    return matching[-1] if matching else None


def doc_length(rel):
    """Nominal length of a long-prompt file <name>_<L>_<k>.txt."""
    stem = Path(rel).name.removesuffix(".txt")
    return int(stem.split("_")[-2])


def longppl_docs(tok, man, model, max_len=None, root=None):
    root = Path(root) if root is not None else locked_dir()
    with (root / "long-prompts" / "SPLITS.tsv").open() as f:
        splits = list(csv.DictReader(f, delimiter="\t"))
    col = splits_column(model, splits[0].keys()) if splits else None
    bos = TX.bos_ids(tok)
    out, skipped = [], []
    for r in sorted(splits, key=lambda r: r["path"]):
        rel = r["path"]
        L = doc_length(rel)
        if max_len and L > max_len:
            skipped.append(rel)
            continue
        sha = source(rel, man, root)
        body = (root / rel).read_text()
        s = int(r["split_char"])
        head, cont = TX.encode(tok, body[:s]), TX.encode(tok, body[s:])
        if col:
            counted = (int(r[f"prompt_tokens_{col}"]), int(r[f"continuation_tokens_{col}"]))
            if counted != (len(head), len(cont)):
                raise LockedSetError(f"{rel}: {len(head)} + {len(cont)} tokens, SPLITS.tsv counts differ for {col}")
        ids = bos + head + cont
        out.append({"name": "lp-" + Path(rel).name.removesuffix(".txt"), "set": "longppl",
                    "task": man[rel]["domain"], "length": L, "source": rel, "source_sha256": sha, "split_char": s,
                    "cont_len": len(cont), "novel": TX.novel_mask(ids, len(cont)), "format": "raw", "ids": ids})
    return out, skipped


DATASETS = {"fresh-long-20261008": ("longppl",)}        # config 'dataset' -> the sets that frozen set holds


def dataset_dir(name):
    """A frozen set other than the locked one (config 'dataset'): beside the locked set; unknown names refused."""
    if name not in DATASETS:
        raise LockedSetError(f"dataset {name!r} is not a known set {sorted(DATASETS)} (absent: the locked set)")
    return locked_dir().parent / name


def prompts(which, tok, cfg, model, protocol, root=None):
    """(prompts, skipped files) of one locked set for this model; config 'dataset' names another frozen set (its
    MANIFEST.tsv sha256 pinned by 'dataset_manifest_sha256'), which replaces the locked set for the sets it holds."""
    name = cfg.get("dataset")
    if name is not None:
        droot = Path(root) if root is not None else dataset_dir(name)
        if name not in DATASETS:
            raise LockedSetError(f"dataset {name!r} is not a known set {sorted(DATASETS)}")
        if which not in DATASETS[name]:
            raise LockedSetError(f"dataset {name!r} holds the {'/'.join(DATASETS[name])} set only, not {which!r}")
        if not cfg.get("dataset_manifest_sha256"):
            raise LockedSetError(f"dataset {name!r}: the config pins no dataset_manifest_sha256")
        man = manifest(droot, cfg["dataset_manifest_sha256"], name)
        return longppl_docs(tok, man, model, cfg.get("longppl_max_len"), droot)
    man = manifest(root)
    if which == "ruler":
        sel = dict(tasks=cfg.get("ruler_tasks"), lengths=cfg.get("ruler_lengths"), max_new=cfg.get("ruler_max_new"))
        variant = cfg.get("ruler_variant")
        if variant == "qfirst":
            from . import derived
            return derived.prompts("qfirst", tok, fmt_of(cfg, model, protocol), man, cfg.get("ruler_max_len"),
                                   root=root, **sel)
        if variant is not None:
            raise LockedSetError(f"ruler_variant {variant!r}: the only RULER variant is 'qfirst'")
        return ruler_prompts(tok, fmt_of(cfg, model, protocol), man, cfg.get("ruler_max_len"), root=root, **sel)
    if which == "longbench":
        return longbench_prompts(tok, fmt_of(cfg, model, protocol), man, cfg.get("longbench_max_len"), root)
    if which == "longppl":
        return longppl_docs(tok, man, model, cfg.get("longppl_max_len"), root)
    raise ValueError(which)


def check_tails(prompts_, tails):
    """longppl: every scored row (the last prompt token on) must lie in every arm's exact tail: tail >= cont + 1.
    tails: {arm name: fn(prompt) -> tail}."""
    bad = [(a, q["name"], fn(q), q["cont_len"]) for q in prompts_ for a, fn in tails.items() if fn(q) < q["cont_len"] + 1]
    if bad:
        raise LockedSetError(f"longppl: the continuation must lie inside every arm's exact tail: {bad[:5]}")


def score(q, text):
    """Per generation-set row: the prediction as scored, its 0-1 score and the metric's name."""
    if q["set"] != "ruler":
        value = MT.longbench_row(q["task"], text, q["refs"], q["all_classes"])
        return {"pred": text, "metric": q["metric"], "score": value}
    pred = MT.postprocess_pred(text)
    return {"pred": pred, "metric": q["metric"], "score": MT.ruler_row(q["metric"], pred, q["refs"])}


def nll(logprobs, mask=None):
    picked = list(logprobs) if mask is None else [x for x, keep in zip(logprobs, mask) if keep]
    return -sum(picked) / len(picked)
