"""Non-numeric needle-in-a-haystack prompts (code/kva/niahg.py): names, phrases, hex ids, identifiers and
sentences as the hidden value, re-rendered for each model's tokenizer from a plan file, plus their scoring.

plan.json rows: name, type, subtype, length, source, depth, key, value, needle_text, question. The haystack is the
K20 cell's (eval.text.k20_cells over the same corpus), body = hay[: L - len(needle) - len(question)] tokens, the
needle at int(depth * len(body)).
  chat  the plan's question (ending in an answer-format instruction) in the chat template
  raw   the question's first sentence then the needle's lead-in up to the value
Scoring: the reply is cut at the first end-of-turn token, think blocks and special tokens removed, its first
non-empty line taken, a restated lead-in dropped, then the answer and the value normalised per type. chat: exact
match; raw (a completion runs on): the normalised answer must start with the normalised value at a word boundary
(hex ids: the answer up to its first space). Misses are classed none / truncated / near (edit distance <= 2) / wrong.
"""
from __future__ import annotations

import json
import re
import unicodedata
from pathlib import Path

from . import text as TX

TYPES = ("name", "phrase", "hexid", "ident", "sentence")


def plan_path():
    return TX.data_root() / "niah-general-dev" / "plan.json"


def prompts(tok, fmt="raw", types=TYPES, plan=None, text_of=None, lengths=TX.NIAH_LENGTHS):
    """lengths: the K20 generator's length grid (its draws depend on the whole grid)."""
    plan = json.loads(Path(plan_path()).read_text()) if plan is None else plan
    plan = [p for p in plan if p["type"] in types]
    text_of = TX.corpus() if text_of is None else text_of
    cells = {(c["length"], c["source"]): c for c in TX.k20_cells(text_of, lengths=lengths)}
    head, tail = TX._frame(tok, fmt)
    hay = {}
    out = []
    for p in plan:
        L, src, value, needle_text = p["length"], p["source"], p["value"], p["needle_text"]
        c = cells[(L, src)]
        if (L, src) not in hay:
            hay[(L, src)] = TX.encode(tok, text_of[src][c["char_start"]:c["char_end"]])
            if len(hay[(L, src)]) < L:
                raise RuntimeError(f"niahg haystack {L}-{src}: {len(hay[(L, src)])} tokens < {L}")
        v0 = needle_text.index(value)
        lead = needle_text[:v0].strip()
        q_text = p["question"] if fmt == "chat" else p["question"].split("?")[0] + "? " + lead
        enc = tok(needle_text, add_special_tokens=False, return_offsets_mapping=True)
        needle = list(enc["input_ids"])
        vt = [i for i, (s, e) in enumerate(enc["offset_mapping"]) if s < v0 + len(value) and e > v0]
        q = TX.encode(tok, q_text)
        body = hay[(L, src)][:L - len(needle) - len(q)]
        at = int(p["depth"] * len(body))
        ids = head + body[:at] + needle + body[at:] + q + tail
        ns = len(head) + at
        out.append(dict(name=p["name"], type=p["type"], subtype=p.get("subtype"), length=L, source=src,
                        depth=p["depth"], key=p["key"], value=value, format=fmt, char_start=c["char_start"],
                        char_end=c["char_end"], needle_start=ns, needle_end=ns + len(needle),
                        value_start=ns + vt[0], value_end=ns + vt[-1] + 1, ids=ids))
    return out


# --------------------------------------------------------------------------------------------- scoring
_THINK = re.compile(r"<think>.*?(?:</think>|$)", re.S)
_SPECIAL = re.compile(r"<\|[a-z_]+\|>")
_END = ("<|im_end|>", "<|endoftext|>", "<|eot_id|>")
_LEAD = re.compile(r"^(?:answer\s*:\s*)?(?:the\s+)?(?:special\s+)?(?:contact person|meeting place|password|identifier|"
                   r"function name|quote|magic number)(?:\s+for\s+[\w-]+)?(?:\s+mentioned in the text above)?\s+"
                   r"(?:is|was)\s*:?\s*", re.I)
_QUOTES = "\"'`“”‘’«»*"
_DASHES = str.maketrans({"–": "-", "—": "-", "‐": "-", "‑": "-", "−": "-"})
_WORD = re.compile(r"[\w'-]")


def reply_text(text):
    for end in _END:
        text = text.split(end)[0]
    return _SPECIAL.sub(" ", _THINK.sub(" ", text))


def extract(text):
    lines = [ln.strip() for ln in reply_text(text).splitlines() if ln.strip()]
    if not lines:
        return ""
    a = lines[0].lstrip("-•> ").strip().strip(_QUOTES).strip()
    return _LEAD.sub("", a).strip().strip(_QUOTES).strip()


def normalize(s, typ):
    s = unicodedata.normalize("NFKC", s).translate(_DASHES)
    if typ == "ident":
        s = re.sub(r"\(\)$", "", s.strip().strip(_QUOTES).strip())
        return s.rstrip(".,;:!?").strip(_QUOTES)
    if typ == "hexid":
        s = re.sub(r"\s+", "", s.casefold().strip().strip(_QUOTES))
        return s.rstrip(".,;:!?").strip(_QUOTES)
    s = "".join(c if c.isalnum() or c in " -'" or c.isspace() else " " for c in s.casefold())
    s = re.sub(r"(?<![a-z0-9])['-]|['-](?![a-z0-9])", " ", s)     # only inner hyphens / apostrophes survive
    return re.sub(r"\s+", " ", s).strip()


def edit_distance(a, b, cap=3):
    """Levenshtein distance, or cap + 1 once the lengths alone differ by more than cap."""
    if abs(len(a) - len(b)) > cap:
        return cap + 1
    row = list(range(len(b) + 1))
    for i, ca in enumerate(a, 1):
        nxt = [i]
        for j, cb in enumerate(b, 1):
            nxt.append(min(row[j] + 1, nxt[j - 1] + 1, row[j - 1] + (ca != cb)))
        row = nxt
    return row[-1]


def score(text, value, typ, fmt):
    """dict(correct, form, answer); form: ok / none / truncated / near / wrong."""
    ans = extract(text)
    cut = re.split(r"\s", ans, maxsplit=1)[0] if (fmt != "chat" and typ == "hexid") else ans
    na, nv = normalize(cut, typ), normalize(value, typ)
    if fmt == "chat":
        ok = na == nv
    else:
        ok = na.startswith(nv) and not _WORD.match(na[len(nv):len(nv) + 1])
        na = na[:len(nv)]
    if ok:
        form = "ok"
    elif not na:
        form = "none"
    elif nv.startswith(na):
        form = "truncated"
    elif edit_distance(na, nv) <= 2:
        form = "near"
    else:
        form = "wrong"
    return dict(correct=ok, form=form, answer=ans)
