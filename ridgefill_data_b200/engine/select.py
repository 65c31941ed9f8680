"""Exact-row selection: which prefix rows of a RidgeFill arm are recomputed exactly through the late layers
(finish(exact_rows=...)) instead of being filled. Selector semantics follow code/kva/select.py:1-72.

Content rules (every matching row; with a `budget`, a seeded uniform subset of round(budget N) of them):
  digits     a row whose token text contains an ASCII digit
  regex      digits, plus every row of a whitespace-delimited word of 4+ characters containing a digit, plus
             capitalised name words (not in the stop list) that sit next to another name word without sentence
             punctuation between them, or that are not sentence-initial and span 2+ tokens
  verbatim   regex, plus URLs, e-mail addresses, one-line quotations of 2+ tokens and code identifiers
             (snake_case / camelCase words of 6+ characters)
Ranked signals (the round(budget N) highest-scoring prefix rows, earlier rows first on ties):
  qattn      attention mass the last WINDOW rows put on each prefix row in the exact lower attention layers
  pred       predicted surprisal (engine/pred.py)          freq       token rarity (-log unigram frequency)
  frag       tokens of the row's word, then rarity           keydiff    1 - cosine of each key to the mean key
  deviation  how far the ridge map moves the late K/V reads from the identity fill
  qfp        attention a row receives from the later prefix rows, per later row
Composite and control arms: blend (the first signal's top rows plus a share taken from a second signal, no
duplicates), band (a fixed distance band before the prompt end), start_recent (the first rows, and the rest of the
budget as a longer exact tail), random (as many rows as a matched arm, seeded by the prompt), tail_match (the
matched arm's count added to the exact tail).
The name-word pattern, its stop list and the verbatim patterns are kept as the reference states them, so the same
prompt yields the same rows.
"""
from __future__ import annotations

import hashlib
import re
import unicodedata

import torch

WINDOW = 64
LAYERS = (3, 7, 11, 15)
RULES = ("digits", "regex", "verbatim")
FIRSTS = ("qattn", "qfp")
SECONDS = ("pred", "freq", "frag", "keydiff", "deviation", "qfp", "regex", "verbatim")
KINDS = RULES[:1] + RULES[1:] + ("qattn", "pred", "freq", "frag", "blend", "start_recent", "keydiff", "deviation",
                                 "band", "qfp", "random", "tail_match")
NEG = float("-inf")


def signals(sel):
    """The signal kinds a selection reads (a blend reads two)."""
    if sel["kind"] != "blend":
        return {sel["kind"]}
    return {sel.get("first", "qattn"), sel.get("second", "pred")}


def _seed(text):
    digest = hashlib.sha256(text.encode()).digest()
    return int.from_bytes(digest[:8], "little") // 2


def _gen(text):
    return torch.Generator().manual_seed(_seed(text))


# ------------------------------------------------------------------------------------------ vocabulary views
def digit_ids(tok):
    """Vocabulary ids whose token piece contains an ASCII digit (added special tokens excluded)."""
    skip = set(getattr(tok, "added_tokens_decoder", {}) or {})
    found = set()
    for i, piece in enumerate(tok.convert_ids_to_tokens(list(range(len(tok))))):
        if piece is not None and i not in skip and any("0" <= c <= "9" for c in piece):
            found.add(i)
    return found


def _byte_alphabet():
    """{printable stand-in character: byte} of the byte-level BPE alphabet (GPT-2's reversible byte map: the
    printable bytes stand for themselves, the others are shifted past 255 in byte order)."""
    direct = set(range(ord("!"), ord("~") + 1)) | set(range(0xA1, 0xAD)) | set(range(0xAE, 0x100))
    table, shift = {}, 0
    for byte in range(256):
        if byte in direct:
            table[chr(byte)] = byte
        else:
            table[chr(0x100 + shift)] = byte
            shift += 1
    return table


def token_bytes(tok):
    """Raw bytes of every vocabulary id (None for added / special tokens)."""
    alphabet = _byte_alphabet()
    skip = set(getattr(tok, "added_tokens_decoder", {}) or {})
    out = []
    for i, piece in enumerate(tok.convert_ids_to_tokens(list(range(len(tok))))):
        if piece is None or i in skip:
            out.append(None)
        elif set(piece) <= alphabet.keys():
            out.append(bytes(alphabet[c] for c in piece))
        else:
            out.append(piece.encode())
    return out


def prefix_text(ids, P, tbytes):
    """(bytes of prefix rows [0, P), owning row of every byte); a special token reads as one space."""
    chunks, owner = [], []
    for r in range(P):
        piece = tbytes[int(ids[r])] or b" "
        chunks.append(piece)
        owner.extend([r] * len(piece))
    return b"".join(chunks), owner


# ------------------------------------------------------------------------------------------ content rules
NAME_WORD = re.compile(r"^[A-Z][a-z]+(?:[-'][A-Z]?[a-z]+)*$")
STOP_CAPS = frozenset("The A An In On At Of For And But Or If When While This That These Those It Its We You He She "
                      "They I My Our Your His Her Their To From By With As Is Are Was Were Be Not No Yes So Then "
                      "There Here What Which Who How Why Where All Any Each Every Some Use See Note Returns "
                      "Return".split())
URL = re.compile(rb"(?:https?|ftp)://\S+|www\.\S+")
EMAIL = re.compile(rb"\S+@\S+\.\S+")
QUOTED = re.compile(rb"\"([^\"\n]+)\"|(?<![\w'])'([^'\n]+)'(?!\w)")
IDENT = re.compile(rb"(?<!\w)[A-Za-z_]\w{5,}(?!\w)")
CODE = re.compile(rb"_|[a-z][A-Z]")
_PUNCT_EDGES = "\"'`([{<,.;:!?)]}>*"
_SENTENCE_END = ".!?:;"


def digits(ids, P, digit_set):
    return [r for r, t in enumerate(ids[:P]) if int(t) in digit_set]


def _words(text, owner):
    """[(word text, rows it covers, byte before it)] for every whitespace-delimited word."""
    out = []
    for m in re.finditer(rb"\S+", text):
        a, b = m.span()
        out.append((m.group().decode("utf-8", errors="replace"), sorted(set(owner[a:b])), text[a - 1:a] if a else b""))
    return out


def regex_rows(ids, P, digit_set, tbytes):
    text, owner = prefix_text(ids, P, tbytes)
    wl = _words(text, owner)
    chosen = set(digits(ids, P, digit_set))
    ends_sentence = [w[-1:] in tuple(_SENTENCE_END) if w else False for w, _, _ in wl]
    name = []
    for w, rows, _ in wl:
        if len(w) >= 4 and any("0" <= c <= "9" for c in w):
            chosen.update(rows)
        core = w.strip(_PUNCT_EDGES)
        name.append(NAME_WORD.match(core) is not None and core not in STOP_CAPS)
    for k, (w, rows, before) in enumerate(wl):
        if not name[k]:
            continue
        joined_left = k > 0 and name[k - 1] and not ends_sentence[k - 1]
        joined_right = k + 1 < len(wl) and name[k + 1] and not ends_sentence[k]
        sentence_start = k == 0 or before in (b"\n", b"") or ends_sentence[k - 1]
        if joined_left or joined_right or (len(rows) >= 2 and not sentence_start):
            chosen.update(rows)
    return sorted(chosen)


def verbatim_rows(ids, P, digit_set, tbytes):
    text, owner = prefix_text(ids, P, tbytes)
    chosen = set(regex_rows(ids, P, digit_set, tbytes))
    spans = [m.span() for pat in (URL, EMAIL) for m in pat.finditer(text)]
    for m in QUOTED.finditer(text):
        g = 1 if m.group(1) is not None else 2
        inner = set(owner[m.start(g):m.end(g)])
        if len(inner) >= 2:
            chosen |= inner
    spans += [m.span() for m in IDENT.finditer(text) if CODE.search(m.group()) and re.search(rb"[A-Za-z]", m.group())]
    for a, b in spans:
        chosen.update(owner[a:b])
    return sorted(chosen)


def rule_rows(kind, ids, P, digit_set, tbytes=None):
    if kind == "digits":
        return digits(ids, P, digit_set)
    if tbytes is None:
        raise ValueError(f"the {kind!r} rule reads token bytes: pass token_bytes(tokenizer)")
    return {"regex": regex_rows, "verbatim": verbatim_rows}[kind](ids, P, digit_set, tbytes)


def rule_score(rows, P, name, kind):
    """A content rule's rows as a ranking [P] (others -inf): a seeded uniform order of the rows, so a smaller budget
    takes a subset of a larger one."""
    score = torch.full((P,), NEG, dtype=torch.float64)
    order = torch.randperm(len(rows), generator=_gen(f"{kind}|{name}|{P}"))
    picked = torch.as_tensor(rows, dtype=torch.long)[order]
    score[picked] = torch.linspace(len(rows), 1, len(rows), dtype=torch.float64) if len(rows) else score[picked]
    return score


# ------------------------------------------------------------------------------------------ ranked signals
def qattn_layers(model, split, layers=None):
    """The exact lower attention layers a window-mass signal reads."""
    return [L for L in (LAYERS if layers is None else layers) if L < split and model.layer_types[L] == "attn"]


@torch.no_grad()
def window_mass(model, win, cache, layers, end=None):
    """Attention mass [n] (fp64, host) the window rows [end - w, end) put on every row, summed over query heads,
    window rows and the given layers. win {L: layer L's inputs of the window rows}; cache: the lower layers' K."""
    total = None
    for L in layers:
        keys = cache[L]["k"]
        n_kv, n, _ = keys.shape
        rows = win[L]
        stop = n if end is None else end
        qpos = torch.arange(stop - rows.shape[0], stop, device=keys.device)
        q = model.queries(L, model.in_norm(rows, model.W[L]["ln1"]), qpos)
        if keys.is_cuda and keys.dtype == torch.bfloat16 and q.shape[-1] % 16 == 0:
            from ..ops.kernels import window_mass as wm_kernel      # two-pass tensor-core kernel (csrc/reduce.cu)
            part = wm_kernel(q.to(torch.bfloat16), keys, qpos, model.scale)
        else:
            group = q.shape[0] // n_kv
            future = torch.arange(n, device=keys.device)[None, :] > qpos[:, None]
            part = torch.zeros(n, dtype=torch.float64, device=keys.device)
            for g in range(n_kv):
                logits = (q[g * group:(g + 1) * group].float() @ keys[g].float().T) * model.scale
                part += torch.softmax(logits.masked_fill(future, NEG), -1).sum((0, 1)).double()
        total = part if total is None else total + part
    return total.cpu()


def _is_break(ch):
    return ch not in ("", "�") and (ch.isspace() or unicodedata.category(ch)[0] in "PS")


def word_breaks(tok):
    """(token starts a new word [V], token ends its word [V]) from each token's decoded first / last character."""
    texts = [tok.decode([i]) for i in range(len(tok))]
    return torch.tensor([_is_break(t[:1]) for t in texts]), torch.tensor([_is_break(t[-1:]) for t in texts])


def words(ids, P, starts, ends):
    """Word index [P] of every prefix row (a new word where a token starts one or its predecessor ended one)."""
    t = torch.as_tensor(list(ids[:P]), dtype=torch.long)
    boundary = starts[t].clone()
    if P:
        boundary[1:] |= ends[t[:-1]]
        boundary[0] = True
    return torch.cumsum(boundary.long(), 0) - 1


def rarity(ids, P, logfreq):
    return -(logfreq[torch.as_tensor(list(ids[:P]), dtype=torch.long)].double())


def frag_scores(ids, P, starts, ends, logfreq):
    """Rows of many-token words first (the word's token count), rarer tokens first within a count."""
    if not P:
        return torch.zeros(0, dtype=torch.float64)
    w = words(ids, P, starts, ends)
    rare = rarity(ids, P, logfreq)
    return torch.bincount(w)[w].double() + rare / (rare.max().item() + 1)


@torch.no_grad()
def key_diff(cache, layers, P):
    """Per prefix row, the sum over layers and KV heads of 1 - cos(row's key, the heads' mean key)."""
    out = torch.zeros(P, dtype=torch.float64)
    for L in layers:
        keys = cache[L]["k"][:, :P].float()
        centre = keys.mean(1, keepdim=True)
        cos = (keys * centre).sum(-1) / (keys.norm(dim=-1) * centre.norm(dim=-1)).clamp_min(1e-12)
        out += (1 - cos).sum(0).double().cpu()
    return out


@torch.no_grad()
def fill_deviation(model, projector, h, split, P, block=4096):
    """Per prefix row, the summed relative squared change the map makes to the late attention layers' K/V reads
    compared with the identity fill."""
    from .prefill import kv_target
    attn = [i for i in range(split, model.n_layers) if model.layer_types[i] == "attn"]
    out = torch.zeros(P, dtype=torch.float64)
    for lo in range(0, P, block):
        rows = h[lo:min(lo + block, P)].to(model.device)
        dev = torch.zeros(rows.shape[0], dtype=torch.float64, device=rows.device)
        for i in attn:
            base = kv_target(model, i, rows).float()
            moved = kv_target(model, i, projector(i, rows)).float()
            dev += ((moved - base).square().sum(-1) / base.square().sum(-1).clamp_min(1e-12)).double()
        out[lo:lo + rows.shape[0]] = dev.cpu()
    return out


def per_later_token(received_low, P):
    """qfp: attention a row receives from the later prefix rows, divided by how many later prefix rows there are
    (at least 1); rows at or past P score 0."""
    n = received_low.shape[0]
    later = (P - 1 - torch.arange(n, dtype=torch.float64)).clamp_min(1.0)
    out = received_low.double() / later
    out[P:] = 0.0
    return out


# ------------------------------------------------------------------------------------------ picking
def _rank(score, P):
    """Prefix row indices by descending score, earlier rows first on ties."""
    return torch.sort(-score[:P].double(), stable=True).indices


def top_rows(score, P, b):
    take = min(max(int(b), 0), P)
    return sorted(_rank(score, P)[:take].tolist())


def blend_rows(first, second, P, b, b_second):
    """b rows: the first signal's top b - b_second, then the second signal's ranked (finite) rows not yet taken, then
    the first signal's next rows if the second runs out. Returns (rows, how many of the second's top b_second rows
    the first had already taken)."""
    b = min(max(int(b), 0), P)
    b2 = min(int(b_second), b)
    primary = _rank(first, P).tolist() if first is not None else []
    taken = set(primary[:b - b2])
    secondary = []
    if b2 > 0:
        s = second[:P].double()
        order = _rank(s, P)
        secondary = order[s[order] != NEG].tolist()
    overlap = len(taken.intersection(secondary[:b2]))
    for r in secondary + primary[b - b2:]:
        if len(taken) == b:
            break
        taken.add(r)
    return sorted(taken), overlap


def random_rows(name, P, b, salt="bypass"):
    """round-free count-matched control: b of the P prefix rows, uniform, seeded by (salt, prompt, P, b)."""
    take = min(max(int(b), 0), P)
    perm = torch.randperm(P, generator=_gen(f"{salt}|{name}|{P}|{take}"))
    return sorted(perm[:take].tolist())


def ranges(rows):
    """Sorted rows as [start, end) runs."""
    runs = []
    for r in rows:
        if runs and runs[-1][1] == r:
            runs[-1][1] += 1
        else:
            runs.append([r, r + 1])
    return runs


class _Chooser:
    """Selections of one prompt; matched arms read their reference arm's count (picked once, on demand)."""

    def __init__(self, arms, n, ids, name, digit_set, sources, breaks, tbytes, known):
        self.by_name = {a.name: a for a in arms}
        self.n, self.ids, self.name = n, ids, name
        self.digit_set, self.src, self.breaks, self.tbytes, self.known = digit_set, sources, breaks, tbytes, known
        self.done = {}

    def signal(self, arm, kind, sel, P, end):
        s = self.src
        if kind == "qattn":
            return s["mass"](arm.split, sel.get("layers"), end)
        if kind == "pred":
            return s["pred"](arm.split, sel["predictor"], P)
        if kind == "freq":
            return rarity(self.ids, P, s["freq"](sel["table"]))
        if kind == "frag":
            return frag_scores(self.ids, P, *self.breaks, s["freq"](sel["table"]))
        if kind == "keydiff":
            return s["keys"](arm.split, sel.get("layers"), P)
        if kind == "deviation":
            return s["dev"](arm, P)
        if kind == "qfp":
            return s["recv"](arm.split, P)
        raise ValueError(f"{arm.name}: {kind!r} does not rank rows")

    def pick(self, arm):
        if arm.name in self.done:
            return self.done[arm.name]
        sel = arm.meta["select"]
        kind, n, P = sel["kind"], self.n, arm.prefix_len(self.n)
        budget = round(sel.get("budget", 0.05) * n)
        end = P if sel.get("window") == "prefix" else (self.known if self.known is not None else n)
        extra, more = 0, ({"window_end": end} if "qattn" in signals(sel) else {})
        if kind in RULES:
            rows = rule_rows(kind, self.ids, P, self.digit_set, self.tbytes)
            if "budget" in sel:
                rows = top_rows(rule_score(rows, P, self.name, kind), P, min(budget, len(rows)))
        elif kind == "qattn" or kind in SECONDS:
            rows = top_rows(self.signal(arm, kind, sel, P, end), P, budget)
        elif kind == "blend":
            rows, more["overlap"] = self._blend(arm, sel, P, end, budget)
        elif kind == "band":
            lo, hi = int(sel["lo"]), int(sel["hi"])
            rows = list(range(max(0, n - hi), min(P, max(0, n - lo))))
        elif kind == "start_recent":
            cap = min(budget, P)
            head = min(sel.get("start", 64), budget, P)
            extra = cap - head
            rows = list(range(min(head, P - extra)))
        elif kind in ("random", "tail_match"):
            target = self.by_name[sel["match"]]
            if "match" in target.meta["select"]:
                raise ValueError(f"{arm.name}: its matched arm {target.name} is itself a matched control")
            count = self.pick(target)["count"]
            rows, extra = (random_rows(self.name, P, count), 0) if kind == "random" else ([], count)
        else:
            raise ValueError(f"{arm.name}: unknown selector {kind!r} (one of {KINDS})")
        self.done[arm.name] = dict(kind=kind, rows=rows, extra_tail=extra, count=len(rows) + extra, **more)
        return self.done[arm.name]

    def _blend(self, arm, sel, P, end, budget):
        share = sel.get("share", 0.5)
        first, second = sel.get("first", "qattn"), sel.get("second", "pred")
        if first not in FIRSTS or second not in SECONDS or not 0 <= share <= 1:
            raise ValueError(f"{arm.name}: blend of {first!r} and {second!r} at share {share} is not defined")
        cap = min(budget, P)
        b2 = round(share * cap)
        s1 = self.signal(arm, first, sel, P, end) if (b2 < cap or second in RULES) else None
        if b2 and second in RULES:
            s2 = torch.full((P,), NEG, dtype=torch.float64)
            hit = torch.as_tensor(rule_rows(second, self.ids, P, self.digit_set, self.tbytes), dtype=torch.long)
            s2[hit] = s1[:P].double()[hit]
        else:
            s2 = self.signal(arm, second, sel, P, end) if b2 else None
        return blend_rows(s1, s2, P, budget, b2)


def choose(arms, n, ids, name, digit_set=None, mass_of=None, pred_of=None, keys_of=None, dev_of=None, freq_of=None,
           breaks=None, recv_of=None, tbytes=None, known=None):
    """{arm name: dict(kind, rows, extra_tail, count[, overlap][, window_end])} for every arm with a selection on
    one prompt of n rows. The callbacks supply the ranking signals: mass_of(split, layers, end), pred_of(split,
    predictor, P), keys_of(split, layers, P), dev_of(arm, P), freq_of(table), recv_of(split, P). known: the rows
    available before anything is scored (window signals end there)."""
    if known is not None and not 0 < known <= n:
        raise ValueError(f"known = {known} rows must lie in (0, {n}]")
    sources = dict(mass=mass_of, pred=pred_of, keys=keys_of, dev=dev_of, freq=freq_of, recv=recv_of)
    c = _Chooser(arms, n, ids, name, digit_set, sources, breaks, tbytes, known)
    for a in arms:
        if a.meta.get("select"):
            c.pick(a)
    return c.done
