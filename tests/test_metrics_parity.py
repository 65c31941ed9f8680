"""Scoring parity with the reference's kva/metrics.py (installed in baseline/_ref) on generated answers: RULER string
match, LongBench F1 / QA F1 / ROUGE-L / code similarity / classification and the row and task aggregates must give
the same numbers, so scores from either harness compare."""
import random
import sys
from pathlib import Path

import pytest
from hypothesis import given, settings
from hypothesis import strategies as st

from ridgefill_data_b200.eval import metrics as M

REF = Path(__file__).resolve().parent.parent / "baseline" / "_ref"
if (REF / "kva" / "metrics.py").exists():
    sys.path.insert(0, str(REF))
    from kva import metrics as RM
else:
    RM = None
pytestmark = pytest.mark.skipif(RM is None, reason="baseline/_ref not installed")

WORDS = ["the", "a", "Paris", "paris,", "42", "forty-two", "def", "return", "x", "(", ")", "An", "answer:", "\n",
         "magic", "number", "7654321", "is", "<think>", "</think>", "blue", "Blue!", "ok."]
text = st.lists(st.sampled_from(WORDS), min_size=0, max_size=25).map(" ".join)
FAST = settings(max_examples=150, deadline=None, derandomize=True)


@FAST
@given(text, st.lists(text, min_size=1, max_size=3))
def test_longbench_metrics(pred, answers):
    for fn in ("f1_score", "qa_f1_score", "rouge_score", "code_sim_score"):
        ours = getattr(M, fn)(pred, answers[0])
        ref = getattr(RM, fn)(pred, answers[0])
        assert ours == pytest.approx(ref, abs=1e-12), fn
    classes = sorted(set(answers + ["blue", "red"]))
    assert M.classification_score(pred, answers[0], all_classes=classes) == pytest.approx(
        RM.classification_score(pred, answers[0], all_classes=classes), abs=1e-12)
    for ds in ("hotpotqa", "gov_report", "lcc", "trec", "narrativeqa"):
        assert M.longbench_row(ds, pred, answers, classes) == pytest.approx(RM.longbench_row(ds, pred, answers, classes),
                                                                             abs=1e-12), ds


@FAST
@given(text, st.lists(text, min_size=1, max_size=4))
def test_ruler_metrics(pred, refs):
    assert M.postprocess_pred(pred) == RM.postprocess_pred(pred)
    for metric in ("string_match_all", "string_match_part"):
        assert M.ruler_row(metric, pred, refs) == pytest.approx(RM.ruler_row(metric, pred, refs), abs=1e-12)


def test_aggregates():
    r = random.Random(0)
    rows = [r.random() for _ in range(37)]
    assert M.ruler_score(rows) == RM.ruler_score(rows)
    assert M.longbench_score(rows) == RM.longbench_score(rows)
