"""Fit CLI on the tiny preset (CPU, fp32): sweep with saved statistics, listing their documents, refitting
from them without a capture, and the weighted fit."""
from ridgefill_data_b200 import fit


def test_fit_cli_paths(tmp_path, capsys):
    common = ["tiny-llama", "4", "--docs", "3", "--doc-len", "48", "--backend", "torch", "--device", "cpu",
              "--dtype", "fp32", "--lambdas", "0.01,0.1"]
    assert fit.main(common + ["--held", "1", "--out", str(tmp_path), "--save-stats"]) == 0
    stats = tmp_path / "tiny-llama-s4.pt"
    assert stats.exists() and (tmp_path / "tiny-llama-sweep-s4.safetensors").exists()
    capsys.readouterr()
    assert fit.main(["tiny-llama", "4", "--list-docs", str(stats)]) == 0
    assert len(capsys.readouterr().out.split()) == 3
    assert fit.main(common + ["--from-stats", str(stats)]) == 0
    assert "split 4, 2 lambdas" in capsys.readouterr().out
    assert fit.main(common + ["--weight", "rank", "--held", "0", "--out", str(tmp_path / "w")]) == 0
    assert (tmp_path / "w" / "tiny-llama-wrank-s4.pt").exists()
