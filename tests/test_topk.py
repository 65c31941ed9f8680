"""Deterministic block top-k against a (score desc, index asc) reference: heavy exact ties, NaN garbage past the
visible prefix and inside it, rows wider than 512 columns."""
import torch

from ridgefill_data_b200.engine.topk import block_topk, reference_topk


def test_block_topk_matches_reference():
    g = torch.Generator().manual_seed(0)
    for case in range(300):
        rows = int(torch.randint(1, 5, (1,), generator=g))
        cols = int(torch.randint(1, 700, (1,), generator=g))
        k = int(torch.randint(1, 64, (1,), generator=g))
        s = torch.randint(0, 6, (rows, cols), generator=g).float()           # few distinct values: many ties
        vis = torch.randint(0, cols + 1, (rows,), generator=g)
        for r in range(rows):
            s[r, int(vis[r]):] = float("nan")                                # garbage past the visible prefix
        nan_in = torch.rand(rows, cols, generator=g) < 0.01
        s[nan_in] = float("nan")
        got, counts = block_topk(s, k, vis)
        want = reference_topk(s, k, vis)
        assert torch.equal(got, want), case
        assert torch.equal(counts, (want >= 0).sum(1))


def test_reproducibility_gates(tmp_path):
    from ridgefill_data_b200.eval import checks
    x = torch.randn(3, 50)
    d1 = checks.dump_logits(tmp_path / "a.bin", x)
    d2 = checks.dump_logits(tmp_path / "b.bin", x.clone())
    assert d1 == d2 and checks.same_dump(tmp_path / "a.bin", tmp_path / "b.bin")[0]
    y = x.clone()
    y[1, 7] += 1e-3
    checks.dump_logits(tmp_path / "c.bin", y)
    same, first, mx = checks.same_dump(tmp_path / "a.bin", tmp_path / "c.bin")
    assert not same and first == 57 and mx > 0
    assert checks.rerun_bitwise(lambda: torch.ones(4) * 3)[0]
