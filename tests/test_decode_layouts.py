"""Index arithmetic of the decode kernels, restated in numpy and checked on the CPU.

- csrc/gemv.cu gemv_mma_kernel: lane (g, t) loads k 8t .. 8t + 7 of weight rows g, g + 8 and activation row g of
  every 32-wide k block; the two m16n8k16 steps take words {0, 1} and {2, 3} of those pieces as the A and B
  fragments (the PTX fragment layout: A a0 (g, 2t..) a1 (g+8, 2t..) a2 (g, 2t+8..) a3 (g+8, 2t+8..); B b0 (k 2t.., n g)
  b1 (k 2t+8.., n g); C c0,c1 (g, 2t..) c2,c3 (g+8, 2t..)). The permutation of k is the same in A and B, so the
  products are the plain x @ w.T.
- csrc/attention_decode.cu: keys per split L = 64 ceil((p + 1) / 4096) leave at most DEC_SPLITS splits for any
  position p, and the splits [s L, (s + 1) L) that start at or before p cover keys 0 .. p once.
"""
import numpy as np
import pytest

from ridgefill_data_b200.ops.kernels import DEC_SPLITS, decode_attention_supported, gdn_decode_supported


def _gemv_mma(X, W, warps=8, unroll=4):
    """Output [M, N] of the kernel's fragment arithmetic (fp64), one 16-column CTA at a time."""
    M, K = X.shape
    N = W.shape[0]
    nf = 1 if M <= 8 else 2
    nb = (K + 31) // 32
    out = np.zeros((M, N))
    for c0 in range(0, N, 16):
        red = np.zeros((warps, nf, 4, 32))
        for w in range(warps):
            for b in range(w, nb, warps):
                wv = np.zeros((2, 32, 8))
                xv = np.zeros((nf, 32, 8))
                for lane in range(32):
                    g, t = lane >> 2, lane & 3
                    k = b * 32 + 8 * t
                    if k >= K:
                        continue
                    for h in range(2):
                        if c0 + g + 8 * h < N:
                            wv[h, lane] = W[c0 + g + 8 * h, k:k + 8]
                    for f in range(nf):
                        if g + 8 * f < M:
                            xv[f, lane] = X[g + 8 * f, k:k + 8]
                for s in range(2):
                    A = np.zeros((16, 16))
                    for lane in range(32):
                        g, t = lane >> 2, lane & 3
                        A[g, 2 * t:2 * t + 2] = wv[0, lane, 4 * s:4 * s + 2]
                        A[g + 8, 2 * t:2 * t + 2] = wv[1, lane, 4 * s:4 * s + 2]
                        A[g, 2 * t + 8:2 * t + 10] = wv[0, lane, 4 * s + 2:4 * s + 4]
                        A[g + 8, 2 * t + 8:2 * t + 10] = wv[1, lane, 4 * s + 2:4 * s + 4]
                    for f in range(nf):
                        B = np.zeros((16, 8))
                        for lane in range(32):
                            g, t = lane >> 2, lane & 3
                            B[2 * t:2 * t + 2, g] = xv[f, lane, 4 * s:4 * s + 2]
                            B[2 * t + 8:2 * t + 10, g] = xv[f, lane, 4 * s + 2:4 * s + 4]
                        D = A @ B
                        for lane in range(32):
                            g, t = lane >> 2, lane & 3
                            red[w, f, :, lane] += (D[g, 2 * t], D[g, 2 * t + 1], D[g + 8, 2 * t], D[g + 8, 2 * t + 1])
        for i in range(nf * 4 * 32):
            lane, f, r = i & 31, i >> 7, (i >> 5) & 3
            c = c0 + (lane >> 2) + 8 * (r >> 1)
            m = 8 * f + 2 * (lane & 3) + (r & 1)
            if m < M and c < N:
                out[m, c] = red[:, f, r, lane].sum()
    return out


@pytest.mark.parametrize("m", [1, 5, 9, 16])
def test_gemv_mma_fragment_arithmetic_is_the_plain_product(m):
    rng = np.random.default_rng(m)
    X = rng.standard_normal((m, 200))            # K not a multiple of the 32-wide block
    W = rng.standard_normal((37, 200))           # N not a multiple of the 16-column CTA
    np.testing.assert_allclose(_gemv_mma(X, W), X @ W.T, rtol=0, atol=1e-10)


def _split_keys(p):
    return 64 * max(1, -(-(p + 1) // 4096))


@pytest.mark.parametrize("p", [0, 1, 63, 64, 4095, 4096, 4097, 16383, 65535, 131071, 262143, (1 << 20) - 1])
def test_decode_attention_splits_cover_every_key_once(p):
    L = _split_keys(p)
    starts = [s * L for s in range(DEC_SPLITS) if s * L <= p]
    assert len(starts) == p // L + 1 <= DEC_SPLITS
    keys = np.concatenate([np.arange(s, min(s + L, p + 1)) for s in starts])
    assert np.array_equal(keys, np.arange(p + 1))
    assert starts[-1] <= p < starts[-1] + L          # one split holds the new row


def test_decode_kernel_shape_predicates():
    assert decode_attention_supported(256, 24, 4, 64)        # the 27B hybrid
    assert decode_attention_supported(256, 16, 2, 64)        # the Flash-Next MoE
    assert decode_attention_supported(128, 32, 8, 128)       # Qwen3-8B
    assert decode_attention_supported(64, 8, 2, 64)
    assert not decode_attention_supported(96, 8, 2, 96)      # head_dim outside 64 / 128 / 256
    assert not decode_attention_supported(128, 12, 4, 128)   # 3 query heads per KV head
    assert not decode_attention_supported(256, 24, 4, 36)    # rotary dims not whole lane pairs
    assert gdn_decode_supported(128, 128, 4)
    assert not gdn_decode_supported(64, 64, 4)
    assert not gdn_decode_supported(128, 128, 1)


def test_decode_kernel_routing_rules():
    """Which decode rows take the batched kernels (models/b200.py): the GDN step needs one GPU, head dims 128 and
    fp32 contiguous states a prefill made; the attention needs one GPU and a supported head shape."""
    from types import SimpleNamespace

    import torch

    from ridgefill_data_b200.models.b200 import _B200
    cfg = SimpleNamespace(gdn_dk=128, gdn_dv=128, conv_k=4, rot_dim=64)
    m = SimpleNamespace(cfg=cfg, tp=None, nk=2, nv=6, conv_dim=2 * 2 * 128 + 6 * 128, head_dim=256, n_heads=24,
                        n_kv=4)
    ok = dict(conv=torch.zeros(3, m.conv_dim, dtype=torch.bfloat16), rec=torch.zeros(6, 128, 128))
    assert _B200._gdn_decode_ok(m, [ok, ok])
    assert not _B200._gdn_decode_ok(m, [ok, dict(ok, rec=ok["rec"].half())])          # fp32 states only
    assert not _B200._gdn_decode_ok(m, [dict(ok, conv=None)])                          # no prefill yet
    assert not _B200._gdn_decode_ok(m, [dict(ok, rec=ok["rec"].transpose(1, 2))])      # contiguous states
    assert not _B200._gdn_decode_ok(SimpleNamespace(**dict(vars(m), tp=object())), [ok])   # TP ranks
    assert not _B200._gdn_decode_ok(SimpleNamespace(**dict(vars(m), cfg=SimpleNamespace(**dict(vars(cfg),
                                                                                         gdn_dk=64)))), [ok])
    assert _B200._attn_decode_ok(m)
    assert not _B200._attn_decode_ok(SimpleNamespace(**dict(vars(m), tp=object())))
    assert not _B200._attn_decode_ok(SimpleNamespace(**dict(vars(m), n_heads=12)))    # 3 query heads per KV head
