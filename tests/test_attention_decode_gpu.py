"""The batched decode attention (csrc/attention_decode.cu) against the per-sequence path it replaces (head_norm_rope
K/V writes and query norm + RoPE, then the tcgen05 attention at the query's position): the K/V rows it appends are
the same bits, and the logits of several decode steps of sequences of different lengths agree within bf16 rounding,
with contiguous caches and with the paged pool, for head dims 256 (gated, zero-centred norms, partial RoPE), 128 and
64 (no head norm, Llama-3 RoPE)."""
import pytest
import torch

from ridgefill_data_b200.engine.prefill import run_lower
from ridgefill_data_b200.models.base import from_config

from test_b200_model_gpu import HYB, LLAMA, QWEN3

pytestmark = pytest.mark.gpu


def _decode(cfg, paged, batched_kernel, lens, toks, steps):
    from ridgefill_data_b200.models.kvpool import KVPool
    from ridgefill_data_b200.ops._ext import check_errors
    m = from_config(cfg, seed=0, device="cuda", std=0.05, backend="b200")
    if paged:
        m.kv_pool = KVPool(m, 64, 128)
    if not batched_kernel:
        m._attn_decode_ok = lambda: False
    g = torch.Generator().manual_seed(3)
    caches = []
    with torch.no_grad():
        for n in lens:
            ids = torch.randint(0, cfg.vocab, (n,), generator=g).cuda()
            caches.append(run_lower(m, ids, [m.n_layers], reserve=64)[1])
    att = [i for i, t in enumerate(m.layer_types) if t == "attn"][0]
    out, rows = [], []
    pos = list(lens)
    with torch.no_grad():
        for s in range(steps):
            out.append(m.decode_batch(toks[s], pos, caches).float())
            if s == 0:      # the first attention layer's new K/V rows (same inputs on both paths at the first step)
                for c, p in zip(caches, pos):
                    e = c[att]
                    if paged:
                        pool, ps = m.kv_pool, m.kv_pool.page_size
                        pg = e["pages"][p // ps]
                        rows.append((pool.k[att][pg, :, p % ps].clone(), pool.v[att][pg, :, p % ps].clone()))
                    else:
                        rows.append((e["kbuf"][:, p].clone(), e["vbuf"][:, p].clone()))
            pos = [p + 1 for p in pos]
    torch.cuda.synchronize()
    check_errors()
    return out, rows


@pytest.mark.parametrize("cfg", [HYB, QWEN3, LLAMA], ids=lambda c: c.name)
@pytest.mark.parametrize("paged", [False, True])
def test_batched_decode_attention_matches_per_sequence_path(cfg, paged):
    if paged and cfg.head_dim not in (128, 256):
        pytest.skip("the paged pool serves head_dim 128 / 256 (the tcgen05 prefill attention's tiles)")
    lens, steps = [130, 257, 64], 4
    g = torch.Generator().manual_seed(5)
    toks = [[int(t) for t in torch.randint(0, cfg.vocab, (len(lens),), generator=g)] for _ in range(steps)]
    new, new_rows = _decode(cfg, paged, True, lens, toks, steps)
    old, old_rows = _decode(cfg, paged, False, lens, toks, steps)
    for (ka, va), (kb, vb) in zip(new_rows, old_rows):
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    for a, b in zip(new, old):
        assert torch.isfinite(a).all()
        assert (a - b).abs().max().item() / b.abs().max().item() < 3e-2
