"""Text prompt sets re-tokenised per model (code/kva/data.py): tokenizer helpers, the copy / novel-token masks,
chat-template pieces, the graded prompts, the K20 needle-in-a-haystack generator, end-of-sequence ids and the
calibration document lists.

Data files live under a data root (RF_DATA, default <repo>/data):
  inputs/plan-grade.json, plan-train.json, plan-held.json, plan-sterm.json, swap_summary.json   prompt plans
  corpus/<source>.txt                                                                      NIAH haystack texts
  calibration-exclude.json                                                                 {list: [doc names]}
None of them ship with the framework; every function that needs one names the missing file.

Kept alike on purpose, so results compare with the reference's: the masks' token-id rule, the chat-template
split, the capping rule (drop from the left after the BOS), and the K20 generator's seeded draws (one
random.Random(20260930) stream over lengths x sources x depths, haystack start, key and 7-digit value).
"""
from __future__ import annotations

import hashlib
import json
import random
import re
from pathlib import Path

from ..utils import paths

MAX_LEN = 32768
SCORED = 512
COPY_SPAN = 8


def data_root():
    return paths.DATA


def inputs_dir():
    return data_root() / "inputs"


def _need(path):
    path = Path(path)
    if not path.exists():
        raise FileNotFoundError(f"{path}: data file missing (set RF_DATA to the data root)")
    return path


# ------------------------------------------------------------------------------------- tokenizer helpers

class _Encoding(dict):
    __getattr__ = dict.__getitem__


class CharTokenizer:
    """Dry-run tokenizer without files: one id per character (code point + 10, ids below 10 reserved: 1 BOS,
    2 EOS), offsets, decode and a minimal chat template. For tiny random models only."""
    bos_token_id, eos_token_id = 1, 2
    OFFSET = 10

    def __call__(self, text, add_special_tokens=True, return_offsets_mapping=False):
        ids = [self.bos_token_id] if add_special_tokens else []
        ids.extend(ord(ch) + self.OFFSET for ch in text)
        enc = _Encoding(input_ids=ids)
        if return_offsets_mapping:
            enc["offset_mapping"] = list(zip(range(len(text)), range(1, len(text) + 1)))
        return enc

    def decode(self, ids, skip_special_tokens=False):
        return "".join(chr(t - self.OFFSET) for t in map(int, ids) if t >= self.OFFSET)

    def apply_chat_template(self, msgs, tokenize=False, add_generation_prompt=True, **_):
        return f"<u>{msgs[0]['content']}</u><a>"


def tokenizer(model_path):
    """The model's tokenizer (transformers, local files); "char" gives the dry-run CharTokenizer."""
    if str(model_path) == "char":
        return CharTokenizer()
    import transformers
    return transformers.AutoTokenizer.from_pretrained(str(model_path))


def bos_ids(tok):
    """[BOS] when the tokenizer's default encoding starts with one (Llama), else [] (Qwen)."""
    bos = tok.bos_token_id
    first = tok("a").input_ids[:1]
    return first if bos is not None and first == [bos] else []


def encode(tok, text):
    return list(tok(text, add_special_tokens=False).input_ids)


def cap(ids, head, max_len=MAX_LEN):
    """At most max_len ids: drop from the left, after the `head` ids, so the scored end survives."""
    if len(ids) <= max_len:
        return ids
    return head + ids[len(ids) - (max_len - len(head)):]


def copy_mask(ids, span=COPY_SPAN):
    """True at every token inside a window of `span` ids that already occurred verbatim starting at an earlier
    position (a window's first occurrence is not marked; overlapping repeats mark the union)."""
    seen = {}
    mask = [False] * len(ids)
    for s in range(len(ids) - span + 1):
        w = tuple(ids[s:s + span])
        if w in seen:
            mask[s:s + span] = [True] * span
        else:
            seen[w] = s
    return mask


def novel_mask(ids, scored, span=COPY_SPAN):
    """Novel-token mask of the last `scored` ids: a token is novel unless copy_mask marks it (a token-id rule)."""
    copied = copy_mask(ids, span)[-scored:]
    return [not c for c in copied]


def chat_pieces(tok):
    """(user-turn open ids, assistant-turn open ids) of the model's chat template around one user message, with
    thinking off where the template has the switch."""
    return _around(tok, "\x00DOC\x00", enable_thinking=False)


def _around(tok, mark, **options):
    """Token ids of the chat template before and after one user message (with the assistant header)."""
    convo = [dict(role="user", content=mark)]
    before, after = tok.apply_chat_template(convo, tokenize=False, add_generation_prompt=True, **options).split(mark)
    return encode(tok, before), encode(tok, after)


def eos_ids(model_path, tok):
    """The tokenizer's EOS plus every eos_token_id of generation_config.json / config.json (text_config too)."""
    found = set()
    if tok.eos_token_id is not None:
        found.add(tok.eos_token_id)
    for f in (Path(model_path) / "generation_config.json", Path(model_path) / "config.json"):
        if not f.exists():
            continue
        conf = json.loads(f.read_text())
        value = conf["eos_token_id"] if "eos_token_id" in conf else conf.get("text_config", {}).get("eos_token_id")
        if isinstance(value, list):
            found.update(value)
        elif value is not None:
            found.add(value)
    return found


# ----------------------------------------------------------------------------------------- graded set
CHAT_ASK = "\n\nContinue the text above from exactly where it stops."


def _grade_builder(tok, fmt):
    """(head ids kept when capping, text -> prompt ids) of one graded-prompt format."""
    bos = bos_ids(tok)
    if fmt == "raw":
        return bos, lambda text: bos + encode(tok, text)
    if fmt != "chat":
        raise ValueError(f"unknown grade format {fmt!r}")
    user_open, reply_open = chat_pieces(tok)
    ask = encode(tok, CHAT_ASK)

    def chat(text):
        doc = encode(tok, text)
        cut = len(doc) - SCORED
        return user_open + doc[:cut] + ask + reply_open + doc[cut:]
    return user_open, chat


def _helps_table():
    f = inputs_dir() / "swap_summary.json"
    if not f.exists():
        return {}
    return {row["name"]: row["helps"] for row in json.loads(f.read_text())["rows"]}


def grade_prompts(tok, fmt="raw", drop_bos=False, plan=None, helps=None):
    """The graded prompts: scored on the last SCORED tokens, novel tokens primary.
    raw: BOS + the text. chat: the text minus its last SCORED tokens plus CHAT_ASK as the user turn, then the
    assistant header, then those SCORED tokens as the reply (joined as ids, so the scored ids equal raw's).
    Capping drops from the left after the head. drop_bos: the same prompts without their (required) BOS.
    plan / helps default to inputs/plan-grade.json and inputs/swap_summary.json."""
    plan = json.loads(_need(inputs_dir() / "plan-grade.json").read_text()) if plan is None else plan
    helps = _helps_table() if helps is None else helps
    head, build = _grade_builder(tok, fmt)
    bos = bos_ids(tok)
    out = []
    for p in plan:
        full = build(p["text"])
        ids = cap(full, head)
        short = build(p["text"][p["short_start"]:])
        rec = {"name": p["name"], "kind": p["kind"], "ids": ids, "full_len": len(full),
               "truncated": len(ids) < len(full), "short_ids": short,
               "short_tail_match": ids[-SCORED:] == short[-SCORED:], "novel": novel_mask(ids[1:], SCORED),
               "helps16": helps.get(p["name"]), "format": fmt}
        if drop_bos:
            starts_with_bos = bool(bos) and ids[0] == bos[0] and short[0] == bos[0]
            if not starts_with_bos:
                raise ValueError(f"drop_bos: prompt {p['name']} does not start with a BOS")
            rec.update(ids=ids[1:], short_ids=short[1:], bos_dropped=True)
        out.append(rec)
    return out


# ------------------------------------------------------------------------------------------ K20 NIAH
NIAH_LENGTHS = (8704, 16384, 32768)
NIAH_DEPTHS = (0.1, 0.3, 0.5, 0.7, 0.9)
NIAH_SOURCES = ("prose", "docs", "code", "rust")
NIAH_SEED = 20260930
NIAH_KEYS = ("amber-falcon", "quiet-harbor", "silver-lantern", "crimson-meadow", "paper-comet", "iron-willow",
             "velvet-canyon", "frozen-orchid", "hollow-summit", "golden-reef", "misty-anchor", "rapid-thistle")
CHARS_PER_TOKEN = 7


def corpus(root=None):
    """{source: text} from <data root>/corpus/*.txt."""
    root = Path(root) if root is not None else data_root() / "corpus"
    return {p.stem: p.read_text() for p in sorted(root.glob("*.txt"))}


def _draw_value(rng):
    return str(rng.randrange(1_000_000, 10_000_000))


def k20_cells(text_of, lengths=NIAH_LENGTHS, sources=NIAH_SOURCES):
    """Per (length, source) cell: the haystack's character range and, per depth, (depth, key, value). One seeded
    stream serves every cell in (length, source) order; per cell it draws the haystack offset, then a key and a
    value for each depth."""
    rng = random.Random(NIAH_SEED)
    cells = []
    for L in lengths:
        span = L * CHARS_PER_TOKEN
        for si, src in enumerate(sources):
            back = si * 1000 + rng.randrange(20000)
            start = max(0, len(text_of[src]) - span - back)
            needles = []
            for depth in NIAH_DEPTHS:
                key = rng.choice(NIAH_KEYS)
                needles.append((depth, key, _draw_value(rng)))
            cells.append({"length": L, "source": src, "char_start": start, "char_end": start + span,
                          "needles": needles})
    return cells


def niah_question(fmt, key):
    if fmt == "chat":
        return (f"\n\nWhat is the special magic number for {key} mentioned in the text above? "
                f"Answer with the 7-digit number only.")
    return (f"\n\nWhat is the special magic number for {key} mentioned in the text above? "
            f"The special magic number for {key} is")


def niah_needle(key, value):
    return f"\nThe special magic number for {key} is {value}.\n"


def _frame(tok, fmt):
    """(head ids, tail ids) around a NIAH body: raw BOS / nothing; chat the template's user and assistant opens."""
    if fmt != "chat":
        return bos_ids(tok), []
    return _around(tok, "\x00NIAH\x00")


def _splice(head, body, sentences):
    """head + body with each needle sentence inserted at int(depth * len(body)) (sentences in depth order);
    returns (ids, [start, end) of the target sentence)."""
    ids = list(head)
    span = (None, None)
    cut = 0
    for depth, sentence, target in sentences:
        at = int(depth * len(body))
        ids.extend(body[cut:at])
        if target:
            span = (len(ids), len(ids) + len(sentence))
        ids.extend(sentence)
        cut = at
    ids.extend(body[cut:])
    return ids, span


def _distractors(name, key, depth):
    """mk4: three other keys at three other depths with fresh values, from the prompt's own seeded stream."""
    r = random.Random(f"{name}-mk4")
    keys = r.sample([k for k in NIAH_KEYS if k != key], 3)
    depths = r.sample([x for x in NIAH_DEPTHS if x != depth], 3)
    return [(dd, kk, _draw_value(r)) for dd, kk in zip(depths, keys)]


def niah_prompts(tok, fmt="raw", variant=None, text_of=None, lengths=NIAH_LENGTHS, sources=NIAH_SOURCES):
    """K20 prompts: haystack tokens, the needle sentence (encoded alone) spliced at int(depth * len(body)), the
    question at the end (raw: ending in 'The special magic number for KEY is'; chat: the user turn with an
    answer-format instruction, then the assistant header). variant 'mk4': plus 3 distractor needles (other keys
    and values) at 3 of the other depths, drawn from a per-prompt RNG so the target is unchanged."""
    if variant not in (None, "mk4"):
        raise ValueError(f"unknown NIAH variant {variant!r}")
    text_of = corpus() if text_of is None else text_of
    head, tail = _frame(tok, fmt)
    out = []
    for c in k20_cells(text_of, lengths, sources):
        L, src = c["length"], c["source"]
        hay = encode(tok, text_of[src][c["char_start"]:c["char_end"]])
        if len(hay) < L:
            raise RuntimeError(f"NIAH haystack {src}: {len(hay)} tokens < {L}")
        for d, key, value in c["needles"]:
            name = f"niah-{L}-{src}-{int(d * 100)}"
            extra = _distractors(name, key, d) if variant == "mk4" else []
            placed = [(d, key, value, True)] + [(dd, kk, vv, False) for dd, kk, vv in extra]
            sentences = sorted(((dd, encode(tok, niah_needle(kk, vv)), target) for dd, kk, vv, target in placed),
                               key=lambda x: x[0])
            q = encode(tok, niah_question(fmt, key))
            body = hay[:L - sum(len(n) for _, n, _ in sentences) - len(q)]
            ids, (start, end) = _splice(head, body, sentences)
            rec = {"name": name, "length": L, "source": src, "depth": d, "key": key, "value": value, "format": fmt,
                   "char_start": c["char_start"], "char_end": c["char_end"], "needle_start": start,
                   "needle_end": end, "ids": ids + q + tail}
            if variant:
                rec["variant"] = variant
                rec["distractors"] = [{"depth": dd, "key": kk, "value": vv} for dd, kk, vv in extra]
            out.append(rec)
    return out


_THINK = re.compile(r"<think>.*?(</think>|$)", re.S)
_SEVEN = re.compile(r"(?<!\d)\d{7}(?!\d)")


def niah_correct(text, value):
    """The first standalone 7-digit number, after dropping any think block, equals the value."""
    visible = _THINK.sub("", text)
    found = _SEVEN.search(visible)
    return found is not None and found.group(0) == value


# ---------------------------------------------------------------------------------- calibration sets
# held documents left out of lambda selection, by the sha256 of their (non-public) name
HELD_EXCLUDE_SHA256 = {"84f57b5fa277a7ed4af11992762af87605d6b02b1d71b0589743ac4a29d9c73d"}


def name_sha256(name):
    return hashlib.sha256(name.encode("utf-8")).hexdigest()


def calib_exclude(which, path=None):
    """Names excluded from the 'train' / 'held' / 'sterm' list (calibration-exclude.json; required)."""
    path = _need(path or data_root() / "calibration-exclude.json")
    return set(json.loads(path.read_text()).get(which, []))


def calib_docs(which):
    """[{name, text}]: train = plan-train's 'calib' documents; held = plan-held's documents of >= 1024 tokens;
    sterm = plan-sterm's; minus the exclusion list (and the held hash list)."""
    ex = calib_exclude(which)
    if which == "train":
        rows = json.loads(_need(inputs_dir() / "plan-train.json").read_text())
        keep = [x for x in rows if x["kind"] == "calib"]
    elif which == "held":
        rows = json.loads(_need(inputs_dir() / "plan-held.json").read_text())
        keep = [x for x in rows if x["tokens"] >= 1024 and name_sha256(x["name"]) not in HELD_EXCLUDE_SHA256]
    elif which == "sterm":
        keep = json.loads(_need(inputs_dir() / "plan-sterm.json").read_text())
    else:
        raise ValueError(which)
    return [dict(name=x["name"], text=x["text"]) for x in keep if x["name"] not in ex]


def calib_ids(tok, which, limit=None):
    bos = bos_ids(tok)
    docs = calib_docs(which)
    if limit:
        docs = docs[:limit]
    return [{"name": d["name"], "ids": cap(bos + encode(tok, d["text"]), bos)} for d in docs]


GRAM = 50


def grams(ids, n=GRAM):
    return {tuple(ids[i:i + n]) for i in range(len(ids) - n + 1)}


def adapt_docs(tok, slices, eval_prompts):
    """Adaptation documents: corpus slices {source: [(start, end)]} kept only when they share no token 50-gram
    with any evaluation prompt's ids. Returns (docs, dropped names)."""
    text_of = corpus()
    bos = bos_ids(tok)
    taken = set()
    for p in eval_prompts:
        taken |= grams(p["ids"])
    docs, dropped = [], []
    for src, spans in slices.items():
        for s, e in spans:
            name = f"adapt-{src}-{s}"
            doc_ids = bos + encode(tok, text_of[src][s:e])
            if taken.isdisjoint(grams(doc_ids)):
                docs.append({"name": name, "source": f"corpus/{src}.txt[{s}:{e}]", "ids": doc_ids})
            else:
                dropped.append(name)
    return docs, dropped
