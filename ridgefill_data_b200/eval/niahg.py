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


class _Haystacks:
    """Token ids of each K20 cell's haystack for one tokenizer, encoded on first use."""

    def __init__(self, tok, text_of, lengths):
        self.tok, self.text_of = tok, text_of
        self.cells = {(c["length"], c["source"]): c for c in TX.k20_cells(text_of, lengths=lengths)}
        self.ids = {}

    def __call__(self, L, src):
        key = (L, src)
        if key not in self.ids:
            c = self.cells[key]
            hay = TX.encode(self.tok, self.text_of[src][c["char_start"]:c["char_end"]])
            if len(hay) < L:
                raise RuntimeError(f"niahg haystack {L}-{src}: {len(hay)} tokens < {L}")
            self.ids[key] = hay
        return self.ids[key]


def _needle(tok, needle_text, value):
    """(needle ids, [first, last] token of the value inside them, the lead-in text before the value)."""
    at = needle_text.index(value)
    enc = tok(needle_text, add_special_tokens=False, return_offsets_mapping=True)
    stop = at + len(value)
    inside = [t for t, (a, b) in enumerate(enc["offset_mapping"]) if a < stop and b > at]
    return list(enc["input_ids"]), (inside[0], inside[-1]), needle_text[:at].strip()


def _question(p, fmt, lead):
    if fmt == "chat":
        return p["question"]
    first = p["question"].split("?")[0]
    return f"{first}? {lead}"


def prompts(tok, fmt="raw", types=TYPES, plan=None, text_of=None, lengths=TX.NIAH_LENGTHS):
    """The plan's prompts for this tokenizer. lengths: the K20 generator's length grid (its draws depend on the
    whole grid)."""
    if plan is None:
        plan = json.loads(Path(plan_path()).read_text())
    text_of = TX.corpus() if text_of is None else text_of
    hay = _Haystacks(tok, text_of, lengths)
    head, tail = TX._frame(tok, fmt)
    out = []
    for p in (row for row in plan if row["type"] in types):
        L, src = p["length"], p["source"]
        needle, (v_first, v_last), lead = _needle(tok, p["needle_text"], p["value"])
        q = TX.encode(tok, _question(p, fmt, lead))
        body = hay(L, src)[:L - len(needle) - len(q)]
        cut = int(p["depth"] * len(body))
        start = len(head) + cut
        c = hay.cells[L, src]
        rec = {"name": p["name"], "type": p["type"], "subtype": p.get("subtype"), "length": L, "source": src,
               "depth": p["depth"], "key": p["key"], "value": p["value"], "format": fmt,
               "char_start": c["char_start"], "char_end": c["char_end"], "needle_start": start,
               "needle_end": start + len(needle), "value_start": start + v_first, "value_end": start + v_last + 1}
        rec["ids"] = head + body[:cut] + needle + body[cut:] + q + tail
        out.append(rec)
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
    """The reply up to its first end-of-turn token, with think blocks and special tokens blanked."""
    cut = min((text.find(e) for e in _END if e in text), default=len(text))
    return _SPECIAL.sub(" ", _THINK.sub(" ", text[:cut]))


def _unquote(t):
    return t.strip().strip(_QUOTES).strip()


def extract(text):
    """The answer: the reply's first non-empty line, unquoted, with a restated lead-in dropped."""
    first = next((ln.strip() for ln in reply_text(text).splitlines() if ln.strip()), "")
    if not first:
        return ""
    return _unquote(_LEAD.sub("", _unquote(first.lstrip("-•> "))))


def _tail_clean(t):
    return t.rstrip(".,;:!?").strip(_QUOTES)


def normalize(s, typ):
    """Comparable form of an answer or a value of one needle type."""
    s = unicodedata.normalize("NFKC", s).translate(_DASHES)
    if typ == "ident":
        return _tail_clean(re.sub(r"\(\)$", "", _unquote(s)))
    if typ == "hexid":
        return _tail_clean(re.sub(r"\s+", "", s.casefold().strip().strip(_QUOTES)))
    kept = "".join(ch if (ch.isalnum() or ch.isspace() or ch in "-'") else " " for ch in s.casefold())
    kept = re.sub(r"(?<![a-z0-9])['-]|['-](?![a-z0-9])", " ", kept)     # only inner hyphens / apostrophes stay
    return " ".join(kept.split())


def edit_distance(a, b, cap=3):
    """Levenshtein distance; cap + 1 as soon as the lengths alone differ by more than cap."""
    if abs(len(a) - len(b)) > cap:
        return cap + 1
    prev = list(range(len(b) + 1))
    for i in range(1, len(a) + 1):
        cur = [i] + [0] * len(b)
        for j in range(1, len(b) + 1):
            cur[j] = min(prev[j] + 1, cur[j - 1] + 1, prev[j - 1] + (a[i - 1] != b[j - 1]))
        prev = cur
    return prev[len(b)]


def _miss_form(got, want):
    if not got:
        return "none"
    if want.startswith(got):
        return "truncated"
    return "near" if edit_distance(got, want) <= 2 else "wrong"


def score(text, value, typ, fmt):
    """{"correct", "form", "answer"}; form is ok, none, truncated, near or wrong."""
    answer = extract(text)
    compared = answer.split(None, 1)[0] if (answer and fmt != "chat" and typ == "hexid") else answer
    got, want = normalize(compared, typ), normalize(value, typ)
    if fmt == "chat":
        ok = got == want
    else:                                    # a completion runs on: the value must end at a word boundary
        ok = got.startswith(want) and _WORD.match(got[len(want):len(want) + 1]) is None
        got = got[:len(want)]
    return {"correct": ok, "form": "ok" if ok else _miss_form(got, want), "answer": answer}
