"""Impact corpus on the CPU: token classes, per-window impact from the engine (tiny hybrid), corpus files with a
checksummed index, aggregation (row 0 excluded, enrichment, provenance digests) and its refusals."""
import json

import numpy as np
import pytest
import torch

from ridgefill_data_b200.eval import impact_corpus as IC
from ridgefill_data_b200.eval.text import CharTokenizer
from ridgefill_data_b200.models.base import from_config
from ridgefill_data_b200.models.tiny import tiny_configs


def test_token_classes():
    c = lambda s, sp=False: IC.CLASSES[IC.token_class(s, sp)]  # noqa: E731
    assert c("<s>", True) == "special" and c("\n") == "newline" and c("  ") == "space"
    assert c(" 42") == "number" and c("...") == "punct" and c(" river") == "word-start"
    assert c(" River") == "word-start-cap" and c("ing") == "word-piece" and c("Ing") == "word-piece-cap"
    assert c("x9") == "mixed"


def test_corpus_roundtrip(tmp_path):
    model = from_config(tiny_configs(8, 64)["qwen3.5-9b"], seed=0, device="cpu", dtype=torch.float32)
    tok = CharTokenizer()
    text = "The river Stone, 42 amber clouds.\nnorth alpha Beta; " * 3
    ids = [1] + [ord(ch) + 10 for ch in text]
    P, scored = 100, 16
    for m in ("model-a", "model-b"):
        w = IC.CorpusWriter(tmp_path, m)
        for j in range(2):
            imp = IC.window_impact(model, ids, 4, P, lambda i, b: b, scored)
            assert imp.shape == (P,) and np.isfinite(imp).all()
            w.add(f"doc{j}", 0, imp, IC.classes_of(tok, ids[:P]))
        w.close()
    res = IC.aggregate(tmp_path, ["model-a", "model-b"])
    a = res["models"]["model-a"]
    assert a["n_windows"] == 2 and a["totals"]["N"] == 2 * (P - 1)                   # row 0 excluded
    assert sum(c["N_c"] for c in a["classes"].values()) == a["totals"]["N"]
    assert abs(sum(c["sum_abs_impact"] for c in a["classes"].values()) - a["totals"]["sum_abs_impact"]) < 1e-9
    assert a["classes"]["special"]["N_c"] == 0                                          # BOS is row 0
    assert a["provenance"]["npz_count"] == 2 and len(a["provenance"]["sorted_npz_sha256_list_sha256"]) == 64
    json.dumps(res, allow_nan=False)
    # a changed file or different document sets are refused
    f = next((tmp_path / "model-a").glob("*.npz"))
    data = bytearray(f.read_bytes())
    data[len(data) // 2] ^= 0xFF
    f.write_bytes(bytes(data))
    with pytest.raises(IC.CorpusError, match="checksum"):
        IC.aggregate_model(tmp_path, "model-a")
    w = IC.CorpusWriter(tmp_path, "model-c")
    w.add("other", 0, np.ones(4), np.zeros(4, dtype=np.int8))
    w.close()
    with pytest.raises(IC.CorpusError, match="document sets"):
        IC.aggregate(tmp_path, ["model-b", "model-c"])
