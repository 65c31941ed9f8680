"""Task metrics whose definitions must match the official benchmark scorers so scores stay comparable
(code/kva/metrics.py:26-205): RULER string_match_all / string_match_part, LongBench qa F1, classification,
code similarity (fuzz ratio of the first code line) and ROUGE-L (summary level, sentence split on '.')."""
from __future__ import annotations

import difflib
import re
import string
from collections import Counter


# ---------------------------------------------------------------------------------- RULER
def postprocess_pred(text):
    return re.sub(r"[\x00-\x1f]", "\n", text.strip()).strip()


def ruler_row(metric, pred, ref):
    """One row's term (0-1) of string_match_all (share of references found) or string_match_part (any found)."""
    text = pred.lower()
    found = [float(r.lower() in text) for r in ref]
    combine = {"string_match_all": lambda: sum(found) / len(ref), "string_match_part": lambda: max(found)}
    if metric not in combine:
        raise ValueError(f"unknown RULER metric {metric!r}")
    return combine[metric]()


def ruler_score(rows):
    return round(sum(rows) / len(rows) * 100, 2)


def string_match_all(preds, refs):
    return ruler_score([ruler_row("string_match_all", p, r) for p, r in zip(preds, refs)])


def string_match_part(preds, refs):
    return ruler_score([ruler_row("string_match_part", p, r) for p, r in zip(preds, refs)])


# ---------------------------------------------------------------------------------- LongBench
def normalize_answer(s):
    s = s.lower()
    s = "".join(ch for ch in s if ch not in set(string.punctuation))
    s = re.sub(r"\b(a|an|the)\b", " ", s)
    return " ".join(s.split())


def f1_score(prediction, ground_truth, **_):
    same = sum((Counter(prediction) & Counter(ground_truth)).values())
    if same == 0:
        return 0
    p, r = same / len(prediction), same / len(ground_truth)
    return 2 * p * r / (p + r)


def qa_f1_score(prediction, ground_truth, **_):
    return f1_score(normalize_answer(prediction).split(), normalize_answer(ground_truth).split())


def classification_score(prediction, ground_truth, **kw):
    matches = [c for c in kw["all_classes"] if c in prediction]
    # the official scorer removes items from the list while iterating it (so it skips the next term)
    for term in matches:
        if term in ground_truth and term != ground_truth:
            matches.remove(term)
    return 1.0 / len(matches) if ground_truth in matches else 0.0


def fuzz_ratio(a, b):
    if a is None or b is None:
        return 0
    if a == b:
        return 100
    if not a or not b:
        return 0
    return int(round(100 * difflib.SequenceMatcher(None, a, b).ratio()))


def code_sim_score(prediction, ground_truth, **_):
    first = ""
    for line in prediction.lstrip("\n").split("\n"):
        if "`" not in line and "#" not in line and "//" not in line:
            first = line
            break
    return fuzz_ratio(first, ground_truth) / 100


def _sentences(text):
    return [" ".join(p.split()) for p in text.split(".") if len(p) > 0]


def _lcs_table(x, y):
    """lengths[i][j] = LCS length of x[:i] and y[:j]."""
    lengths = [[0] * (len(y) + 1)]
    for xi in x:
        prev, row = lengths[-1], [0]
        for j, yj in enumerate(y, 1):
            row.append(prev[j - 1] + 1 if xi == yj else max(prev[j], row[j - 1]))
        lengths.append(row)
    return lengths


def _lcs_words(x, y):
    """One longest common subsequence of word lists x and y, read back from the end (on a tie the step drops a
    word of y, as the official ROUGE-L scorer does)."""
    lengths = _lcs_table(x, y)
    words = []
    i, j = len(x), len(y)
    while i and j:
        if x[i - 1] == y[j - 1]:
            words.append(x[i - 1])
            i -= 1
            j -= 1
        elif lengths[i - 1][j] > lengths[i][j - 1]:
            i -= 1
        else:
            j -= 1
    return words


def rouge_l(hyp, ref):
    hyp, ref = _sentences(hyp), _sentences(ref)
    if not hyp or not ref:
        raise ValueError("Collections must contain at least 1 sentence.")
    m = len({w for s in ref for w in s.split(" ")})
    n = len({w for s in hyp for w in s.split(" ")})
    union = set()
    for rs in ref:
        for hs in hyp:
            union |= set(_lcs_words(rs.split(" "), hs.split(" ")))
    r, p = len(union) / m, len(union) / n
    return 2.0 * ((p * r) / (p + r + 1e-8))


def rouge_score(prediction, ground_truth, **_):
    try:
        return rouge_l(prediction, ground_truth)
    except (ValueError, ZeroDivisionError):
        return 0.0


LONGBENCH_METRIC = {"narrativeqa": qa_f1_score, "qasper": qa_f1_score, "hotpotqa": qa_f1_score,
                    "2wikimqa": qa_f1_score, "gov_report": rouge_score, "trec": classification_score,
                    "lcc": code_sim_score, "repobench-p": code_sim_score}
FIRST_LINE = ("trec", "triviaqa", "samsum", "lsht")


def longbench_row(dataset, prediction, answers, all_classes):
    if dataset in FIRST_LINE:
        prediction = prediction.lstrip("\n").split("\n")[0]
    return max([0.0] + [LONGBENCH_METRIC[dataset](prediction, gt, all_classes=all_classes) for gt in answers])


def longbench_score(rows):
    return round(100 * sum(rows) / len(rows), 2)
