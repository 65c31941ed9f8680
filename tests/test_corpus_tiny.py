"""Corpus fingerprints and cut points; tiny dry-run checkpoints load and run through the loader."""
import numpy as np
import torch

from ridgefill_data_b200.eval import corpus as CP
from ridgefill_data_b200.models.base import load
from ridgefill_data_b200.models.tiny import make_tiny


def test_grams_shared_and_seen(tmp_path):
    words = [f"w{i}" for i in range(120)]
    a = " ".join(words)
    g = CP.grams(a, n=50)
    assert len(g) == 71 and len(np.unique(g)) == 71
    assert np.array_equal(CP.grams(" ".join(words[10:70]), n=50), g[10:21])
    ref = CP.reference([], texts=[" ".join(words[:60])])
    assert CP.shared(g, ref) == 11
    assert abs(CP.self_repeat(CP.grams(" ".join(words[:60] * 2), n=50)) - 11 / 71) < 1e-12
    seen = CP.Seen()
    seen.add("doc0", g)
    share, owner = seen.containment(CP.grams(" ".join(words[:80]), n=50))
    assert owner == "doc0" and share == 1.0
    (tmp_path / "x.jsonl").write_text('{"t": "%s", "k": 1}\n' % a)
    assert np.array_equal(CP.file_grams(tmp_path / "x.jsonl"), np.unique(g))


def test_cut_points():
    assert CP.cut_points(40000) == [20000, 30000, 40000]
    assert CP.cut_points(9000) == [9000]
    assert CP.cut_points(8000) == []


def test_tiny_checkpoints_load(tmp_path):
    paths = make_tiny(tmp_path, layers=8)
    for name, p in paths.items():
        m = load(p, dtype=torch.float32)
        logits, _ = m.forward_exact(torch.arange(12), keep=torch.tensor([11]))
        assert logits.shape[-1] == m.cfg.vocab and torch.isfinite(logits).all(), name
    assert load(paths["llama-3.1-swiftkv-8b-instruct"]).cfg.swift_layers == 4


def test_overlap_report(tmp_path):
    words = [f"w{i}" for i in range(200)]
    (tmp_path / "calib").mkdir()
    (tmp_path / "eval").mkdir()
    (tmp_path / "calib" / "a.txt").write_text(" ".join(words[:120]))
    (tmp_path / "calib" / "b.txt").write_text(" ".join(f"x{i}" for i in range(120)))
    (tmp_path / "eval" / "e.jsonl").write_text('{"text": "%s"}\n' % " ".join(words[60:200]))
    rows = CP.overlap_report(CP._texts([tmp_path / "calib"]), CP._texts([tmp_path / "eval"]), n=50)
    assert rows[0]["name"].endswith("a.txt") and rows[0]["shared"] == 11 and rows[1]["shared"] == 0
    assert CP.main(["--calib", str(tmp_path / "calib"), "--eval", str(tmp_path / "eval"), "--tsv",
                    str(tmp_path / "o.tsv")]) == 0
    assert len(CP.read_tsv(tmp_path / "o.tsv")) == 2
