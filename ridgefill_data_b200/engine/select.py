"""Exact-row selectors: which prefix rows [0, P) of an arm run exactly through the late layers
(finish(exact_rows=...)). Semantics of the reference's selector module (code/kva/select.py:1-72).

Content rules (natural budget, or a seeded uniform sample of round(budget * N) rows):
  digits     rows whose token text holds an ASCII digit
  regex      digits, rows of whitespace words of >= 4 chars with a digit, and capitalised names (a NAME_WORD not in
             STOP_CAPS, kept next to another name word without sentence punctuation between, or when not
             sentence-initial and >= 2 tokens long)
  verbatim   regex plus URLs, emails, the inside of one-line quotes (>= 2 tokens), snake_case / camelCase
             identifiers of >= 6 chars
Ranked signals (top round(budget * N) rows, ties by position):
  qattn      attention mass the last WINDOW rows give each prefix row at the exact lower attention layers
  pred       predicted surprisal (engine/pred.py), freq (token rarity), frag (pieces of the row's word, ties by
             rarity), keydiff (1 - cos of each key to the mean key), deviation (how far the projector moves the
             late attention reads from the identity fill), qfp (attention received per later prefix row)
Composites / controls: blend (a first signal plus a share of a second one, rank fusion without duplicates),
band (a fixed distance band before the prompt end), start_recent (the first rows plus a longer tail),
random (as many rows as a matched arm, seeded), tail_match (the tail grows by the matched arm's count).
The word rules' stop list and patterns are kept as the reference defines them, so a selection is the same
set of rows on the same prompt.
"""
from __future__ import annotations

import hashlib
import re
import unicodedata

import torch

WINDOW = 64
LAYERS = (3, 7, 11, 15)
KINDS = ("digits", "regex", "verbatim", "qattn", "pred", "freq", "frag", "blend", "start_recent", "keydiff",
         "deviation", "band", "qfp", "random", "tail_match")
RULES = ("digits", "regex", "verbatim")
SECONDS = ("pred", "freq", "frag", "keydiff", "deviation", "qfp", "regex", "verbatim")
FIRSTS = ("qattn", "qfp")


def signals(sel):
    if sel["kind"] == "blend":
        return {sel.get("first", "qattn"), sel.get("second", "pred")}
    return {sel["kind"]}


def _seed(text):
    return int.from_bytes(hashlib.sha256(text.encode()).digest()[:8], "little") >> 1


# ------------------------------------------------------------------------------ token text helpers

def digit_ids(tok):
    added = set(getattr(tok, "added_tokens_decoder", {}) or {})
    pieces = tok.convert_ids_to_tokens(list(range(len(tok))))
    return {i for i, s in enumerate(pieces) if s is not None and i not in added and re.search("[0-9]", s)}


def _bpe_byte_inverse():
    """Printable character -> byte of the byte-level BPE alphabet (GPT-2's reversible byte map)."""
    keep = list(range(33, 127)) + list(range(161, 173)) + list(range(174, 256))
    chars, extra = {}, 0
    for b in range(256):
        if b in keep:
            chars[chr(b)] = b
        else:
            chars[chr(256 + extra)] = b
            extra += 1
    return chars


def token_bytes(tok):
    """Bytes of every vocabulary id (None for added/special tokens); BPE pieces mapped back to raw bytes."""
    inv = _bpe_byte_inverse()
    added = set(getattr(tok, "added_tokens_decoder", {}) or {})
    out = []
    for i, s in enumerate(tok.convert_ids_to_tokens(list(range(len(tok))))):
        if s is None or i in added:
            out.append(None)
        elif all(c in inv for c in s):
            out.append(bytes(inv[c] for c in s))
        else:
            out.append(s.encode())
    return out


def prefix_text(ids, P, tbytes):
    """(bytes of rows [0, P), row of each byte); special tokens read as a space."""
    text, row = bytearray(), []
    for r in range(P):
        b = tbytes[int(ids[r])]
        b = b" " if b is None else b
        text += b
        row += [r] * len(b)
    return bytes(text), row


WORD = re.compile(rb"\S+")
NAME_WORD = re.compile(r"^[A-Z][a-z]+(?:[-'][A-Z]?[a-z]+)*$")
STOP_CAPS = frozenset("The A An In On At Of For And But Or If When While This That These Those It Its We You He She "
                      "They I My Our Your His Her Their To From By With As Is Are Was Were Be Not No Yes So Then "
                      "There Here What Which Who How Why Where All Any Each Every Some Use See Note Returns "
                      "Return".split())
SENT_END = re.compile(r"[.!?:;]$")
URL = re.compile(rb"(?:https?|ftp)://\S+|www\.\S+")
EMAIL = re.compile(rb"\S+@\S+\.\S+")
QUOTED = re.compile(rb"\"([^\"\n]+)\"|(?<![\w'])'([^'\n]+)'(?!\w)")
IDENT = re.compile(rb"(?<!\w)[A-Za-z_]\w{5,}(?!\w)")
CODE = re.compile(rb"_|[a-z][A-Z]")


def digits(ids, P, digit_set):
    return [r for r in range(P) if int(ids[r]) in digit_set]


def regex_rows(ids, P, digit_set, tbytes):
    text, row = prefix_text(ids, P, tbytes)
    words = [(m.group().decode("utf-8", errors="replace"), sorted(set(row[m.start():m.end()])),
              text[max(0, m.start() - 1):m.start()]) for m in WORD.finditer(text)]
    out = set(digits(ids, P, digit_set))
    is_name = []
    for w, rows, _ in words:
        if len(w) >= 4 and re.search(r"[0-9]", w):
            out.update(rows)
        core = w.strip("\"'`([{<,.;:!?)]}>*")
        is_name.append(bool(NAME_WORD.match(core)) and core not in STOP_CAPS)
    for k, (w, rows, before) in enumerate(words):
        if not is_name[k]:
            continue
        prev_ok = k > 0 and is_name[k - 1] and not SENT_END.search(words[k - 1][0])
        next_ok = k + 1 < len(words) and is_name[k + 1] and not SENT_END.search(w)
        initial = k == 0 or before in (b"\n", b"") or bool(SENT_END.search(words[k - 1][0]))
        if prev_ok or next_ok or (not initial and len(rows) >= 2):
            out.update(rows)
    return sorted(out)


def verbatim_rows(ids, P, digit_set, tbytes):
    text, row = prefix_text(ids, P, tbytes)
    out = set(regex_rows(ids, P, digit_set, tbytes))
    for pat in (URL, EMAIL):
        for m in pat.finditer(text):
            out.update(row[m.start():m.end()])
    for m in QUOTED.finditer(text):
        grp = 1 if m.group(1) is not None else 2
        inside = set(row[m.start(grp):m.end(grp)])
        if len(inside) >= 2:
            out.update(inside)
    for m in IDENT.finditer(text):
        if CODE.search(m.group()) and re.search(rb"[A-Za-z]", m.group()):
            out.update(row[m.start():m.end()])
    return sorted(out)


def rule_rows(kind, ids, P, digit_set, tbytes=None):
    if kind == "digits":
        return digits(ids, P, digit_set)
    if tbytes is None:
        raise ValueError(f"select kind {kind!r} needs token_bytes(tok)")
    return (regex_rows if kind == "regex" else verbatim_rows)(ids, P, digit_set, tbytes)


def rule_score(rows, P, name, kind):
    """A content rule's rows as a ranking [P]: its rows in a seeded uniform order (budgets nest), others -inf."""
    s = torch.full((P,), float("-inf"), dtype=torch.float64)
    perm = torch.randperm(len(rows), generator=torch.Generator().manual_seed(_seed(f"{kind}|{name}|{P}")))
    s[torch.as_tensor(rows, dtype=torch.long)[perm]] = torch.arange(len(rows), 0, -1, dtype=torch.float64)
    return s


# ------------------------------------------------------------------------------ ranked signals

def qattn_layers(model, split, layers=None):
    layers = LAYERS if layers is None else layers
    return [L for L in layers if L < split and model.layer_types[L] == "attn"]


@torch.no_grad()
def window_mass(model, win, cache, layers, end=None):
    """Attention mass [n] (fp64, CPU) the window rows [end - w, end) give every row, summed over query heads,
    window rows and the given exact lower attention layers. win {L: inputs of layer L for the window rows}."""
    mass = None
    for L in layers:
        k = cache[L]["k"]
        hkv, n, _ = k.shape
        h = win[L]
        w = h.shape[0]
        e = n if end is None else end
        qpos = torch.arange(e - w, e, device=k.device)
        q = model.queries(L, model.in_norm(h, model.W[L]["ln1"]), qpos)
        rep = q.shape[0] // hkv
        if k.is_cuda and k.dtype == torch.bfloat16 and q.shape[-1] % 16 == 0:
            from ..ops.kernels import window_mass as wm_kernel      # two-pass tensor-core kernel (csrc/reduce.cu)
            acc = wm_kernel(q.to(torch.bfloat16), k, qpos, model.scale)
            mass = acc if mass is None else mass + acc
            continue
        mask = torch.arange(n, device=k.device)[None, :] > qpos[:, None]
        acc = torch.zeros(n, dtype=torch.float64, device=k.device)
        for gi in range(hkv):
            s = torch.matmul(q[gi * rep:(gi + 1) * rep].float(), k[gi].float().T) * model.scale
            s.masked_fill_(mask, float("-inf"))
            acc += torch.softmax(s, -1).sum((0, 1)).double()
        mass = acc if mass is None else mass + acc
    return mass.cpu()


def _breaks(text):
    return text not in ("", "�") and (text.isspace() or unicodedata.category(text)[0] in "PS")


def word_breaks(tok):
    texts = [tok.decode([i]) for i in range(len(tok))]
    return torch.tensor([_breaks(t[:1]) for t in texts]), torch.tensor([_breaks(t[-1:]) for t in texts])


def words(ids, P, starts, ends):
    t = torch.as_tensor(list(ids[:P]), dtype=torch.long)
    new = starts[t].clone()
    new[1:] |= ends[t[:-1]]
    if P:
        new[0] = True
    return new.long().cumsum(0) - 1


def rarity(ids, P, logfreq):
    return -logfreq[torch.as_tensor(list(ids[:P]), dtype=torch.long)].double()


def frag_scores(ids, P, starts, ends, logfreq):
    if P == 0:
        return torch.zeros(0, dtype=torch.float64)
    w = words(ids, P, starts, ends)
    r = rarity(ids, P, logfreq)
    return torch.bincount(w)[w].double() + r / (float(r.max()) + 1)


@torch.no_grad()
def key_diff(cache, layers, P):
    score = torch.zeros(P, dtype=torch.float64)
    for L in layers:
        k = cache[L]["k"][:, :P].float()
        mean = k.mean(1, keepdim=True)
        cos = (k * mean).sum(-1) / (k.norm(dim=-1) * mean.norm(dim=-1)).clamp_min(1e-12)
        score += (1 - cos).sum(0).double().cpu()
    return score


@torch.no_grad()
def fill_deviation(model, projector, h, split, P, block=4096):
    from .prefill import kv_target
    late = [i for i in range(split, model.n_layers) if model.layer_types[i] == "attn"]
    out = torch.zeros(P, dtype=torch.float64)
    for r in range(0, P, block):
        b = h[r:min(r + block, P)].to(model.device)
        acc = torch.zeros(b.shape[0], dtype=torch.float64, device=b.device)
        for i in late:
            ident = kv_target(model, i, b).float()
            d = kv_target(model, i, projector(i, b)).float() - ident
            acc += (d.square().sum(-1) / ident.square().sum(-1).clamp_min(1e-12)).double()
        out[r:r + b.shape[0]] = acc.cpu()
    return out


def per_later_token(received_low, P):
    """qfp score: attention a row receives from later prefix rows, per later prefix row."""
    later = torch.clamp(P - 1 - torch.arange(received_low.shape[0], dtype=torch.float64), min=1.0)
    out = received_low.double() / later
    out[P:] = 0.0
    return out


# ------------------------------------------------------------------------------ picking

def top_rows(score, P, b):
    b = max(0, min(int(b), P))
    order = torch.sort(-score[:P].double(), stable=True).indices
    return sorted(order[:b].tolist())


def blend_rows(first, second, P, b, b_second):
    """b rows: first's top b - b_second, then second's ranked rows not yet taken (first refills if second runs
    out). Returns (rows, overlap)."""
    b = max(0, min(int(b), P))
    b_second = min(int(b_second), b)
    head = torch.sort(-first[:P].double(), stable=True).indices.tolist() if first is not None else []
    rows = set(head[:b - b_second])
    order = []
    if b_second > 0:
        s = second[:P].double()
        idx = torch.sort(-s, stable=True).indices
        order = idx[s[idx] > float("-inf")].tolist()
    overlap = len(rows & set(order[:b_second]))
    for r in order + head[b - b_second:]:
        if len(rows) >= b:
            break
        rows.add(r)
    return sorted(rows), overlap


def random_rows(name, P, b, salt="bypass"):
    b = max(0, min(int(b), P))
    g = torch.Generator().manual_seed(_seed(f"{salt}|{name}|{P}|{b}"))
    return sorted(torch.randperm(P, generator=g)[:b].tolist())


def ranges(rows):
    out = []
    for r in rows:
        if out and out[-1][1] == r:
            out[-1][1] = r + 1
        else:
            out.append([r, r + 1])
    return out


def choose(arms, n, ids, name, digit_set=None, mass_of=None, pred_of=None, keys_of=None, dev_of=None, freq_of=None,
           breaks=None, recv_of=None, tbytes=None, known=None):
    """Per prompt, for each arm with meta['select']: {arm: dict(kind, rows, extra_tail, count[, overlap,
    window_end])}. Matched arms (random, tail_match) read the matched arm's count. The signal callbacks
    supply the scores (mass_of(split, layers, end), pred_of(split, predictor, P), keys_of(split, layers, P),
    dev_of(arm, P), freq_of(table), recv_of(split, P)). known: rows available before anything is scored."""
    by_name = {a.name: a for a in arms}
    if known is not None and not 0 < known <= n:
        raise ValueError(f"known rows {known} not in (0, n = {n}]")
    out = {}

    def score(a, kind, sel, P, end):
        if kind == "qattn":
            return mass_of(a.split, sel.get("layers"), end)
        if kind == "pred":
            return pred_of(a.split, sel["predictor"], P)
        if kind == "freq":
            return rarity(ids, P, freq_of(sel["table"]))
        if kind == "frag":
            return frag_scores(ids, P, *breaks, freq_of(sel["table"]))
        if kind == "keydiff":
            return keys_of(a.split, sel.get("layers"), P)
        if kind == "deviation":
            return dev_of(a, P)
        if kind == "qfp":
            return recv_of(a.split, P)
        raise ValueError(f"{a.name}: {kind!r} is not a ranking signal")

    def pick(a):
        if a.name in out:
            return out[a.name]
        sel = a.meta["select"]
        kind = sel["kind"]
        P = a.prefix_len(n)
        rows, extra, more = [], 0, {}
        b = round(sel.get("budget", 0.05) * n)
        end = P if sel.get("window") == "prefix" else (n if known is None else known)
        if "qattn" in signals(sel):
            more["window_end"] = end
        if kind in RULES:
            rows = rule_rows(kind, ids, P, digit_set, tbytes)
            if "budget" in sel:
                rows = top_rows(rule_score(rows, P, name, kind), P, min(b, len(rows)))
        elif kind in ("qattn",) + SECONDS:
            rows = top_rows(score(a, kind, sel, P, end), P, b)
        elif kind == "blend":
            share, first, second = sel.get("share", 0.5), sel.get("first", "qattn"), sel.get("second", "pred")
            if not 0 <= share <= 1 or first not in FIRSTS or second not in SECONDS:
                raise ValueError(f"{a.name}: blend share {share}, first {first!r}, second {second!r}")
            b2 = round(share * min(b, P))
            s1 = score(a, first, sel, P, end) if b2 < min(b, P) or second in RULES else None
            if b2 > 0 and second in RULES:
                s2 = torch.full((P,), float("-inf"), dtype=torch.float64)
                r2 = torch.as_tensor(rule_rows(second, ids, P, digit_set, tbytes), dtype=torch.long)
                s2[r2] = s1[:P].double()[r2]
            else:
                s2 = score(a, second, sel, P, end) if b2 > 0 else None
            rows, more["overlap"] = blend_rows(s1, s2, P, b, b2)
        elif kind == "band":
            lo, hi = int(sel["lo"]), int(sel["hi"])
            rows = list(range(max(0, n - hi), min(P, max(0, n - lo))))
        elif kind == "start_recent":
            k = min(sel.get("start", 64), b, P)
            extra = min(b, P) - k
            rows = list(range(min(k, P - extra)))
        elif kind in ("random", "tail_match"):
            ref = by_name[sel["match"]]
            if "match" in ref.meta["select"]:
                raise ValueError(f"{a.name}: matched arm {ref.name} is itself matched")
            count = pick(ref)["count"]
            if kind == "random":
                rows = random_rows(name, P, count)
            else:
                extra = count
        else:
            raise ValueError(f"{a.name}: select kind {kind!r} not in {KINDS}")
        out[a.name] = dict(kind=kind, rows=rows, extra_tail=extra, count=len(rows) + extra, **more)
        return out[a.name]

    for a in arms:
        if a.meta.get("select"):
            pick(a)
    return out
