"""Own torch forward vs transformers on tiny random checkpoints (fp32, CPU), plus cache/decode
equivalence: prefill followed by token-by-token decode equals the full forward."""
import pytest
import torch

from ridgefill_data_b200.models.base import load


def _hf_logits(m, ids):
    with torch.no_grad():
        return m(ids[None]).logits[0].float()


@pytest.mark.parametrize("fixture", ["tiny_llama", "tiny_qwen3", "tiny_qwen35", "tiny_qwen35_moe"])
def test_forward_matches_transformers(fixture, request):
    path, hf = request.getfixturevalue(fixture)
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (150,), generator=torch.Generator().manual_seed(5))
    got, _ = m.forward_exact(ids, keep=torch.arange(150))
    ref = _hf_logits(hf, ids)
    assert torch.allclose(got, ref, atol=2e-4, rtol=1e-4), (got - ref).abs().max()


def test_positive_control_llama_layer_on_qwen3(tiny_qwen3):
    """The Llama layer on Qwen3 weights (no q/k norm) must NOT match: the comparison has teeth."""
    from ridgefill_data_b200.models.checkpoint import Checkpoint
    from ridgefill_data_b200.models.config import ModelConfig
    from ridgefill_data_b200.models.llama import Llama
    path, hf = tiny_qwen3
    cfg = ModelConfig.from_dir(path).replace(arch="llama")
    m = Llama(cfg, Checkpoint(path), dtype=torch.float32)
    ids = torch.randint(0, 300, (40,), generator=torch.Generator().manual_seed(6))
    got, _ = m.forward_exact(ids, keep=torch.arange(40))
    assert not torch.allclose(got, _hf_logits(hf, ids), atol=1e-2)


@pytest.mark.parametrize("fixture", ["tiny_llama", "tiny_qwen3", "tiny_qwen35", "tiny_qwen35_moe"])
def test_prefill_then_decode_equals_full(fixture, request):
    path, _ = request.getfixturevalue(fixture)
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (70,), generator=torch.Generator().manual_seed(7))
    full, _ = m.forward_exact(ids, keep=torch.arange(70))
    n0 = 64
    _, cache = m.forward_exact(ids[:n0])
    for t in range(n0, 70):
        h = m.embed(ids[t:t + 1])
        pos = torch.tensor([t])
        for i in range(m.n_layers):
            h = m.layer(i, h, pos, cache)
        lg = m.logits(h)[0]
        assert torch.allclose(lg, full[t], atol=2e-4, rtol=1e-4), (t, (lg - full[t]).abs().max())


def test_gdn_row_segments_invariant(tiny_qwen35, monkeypatch):
    from ridgefill_data_b200.models import hybrid
    path, _ = tiny_qwen35
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (200,), generator=torch.Generator().manual_seed(8))
    ref, _ = m.forward_exact(ids, keep=torch.arange(200))
    monkeypatch.setattr(hybrid, "GDN_ROWS", 64)
    got, _ = m.forward_exact(ids, keep=torch.arange(200))
    assert torch.allclose(got, ref, atol=1e-5)


def test_fill_writes_what_layer_writes(tiny_qwen35):
    path, _ = tiny_qwen35
    m = load(path, dtype=torch.float32)
    ids = torch.randint(0, 300, (90,), generator=torch.Generator().manual_seed(9))
    got = {}
    _, cache = m.forward_exact(ids, hook=lambda i, h: got.__setitem__(i, h))
    pos = torch.arange(90)
    for i in range(m.n_layers):
        c = m.new_cache()
        m.fill(i, got[i], pos, c)
        if m.layer_types[i] == "attn":
            assert torch.allclose(c[i]["k"], cache[i]["k"]) and torch.allclose(c[i]["v"], cache[i]["v"])
        else:
            assert torch.allclose(c[i]["rec"], cache[i]["rec"], atol=1e-6)
            assert torch.allclose(c[i]["conv"], cache[i]["conv"])
