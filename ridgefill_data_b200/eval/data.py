"""Seeded synthetic token data (the GPU boxes have no datasets): Zipf(s) calibration documents and
uniform-random prompts, reproducible across machines (CPU generator, fixed seeds)."""
from __future__ import annotations

import torch


def zipf_ids(n, vocab, s=1.1, seed=1, generator=None):
    """n token ids with P(rank r) ~ r^-s over the vocabulary, ranks mapped to ids by a seeded permutation."""
    g = generator or torch.Generator().manual_seed(seed)
    ranks = torch.arange(1, vocab + 1, dtype=torch.float64)
    p = ranks.pow(-s)
    p /= p.sum()
    r = torch.multinomial(p, n, replacement=True, generator=g)
    perm = torch.randperm(vocab, generator=torch.Generator().manual_seed(seed + 7919))
    return perm[r]


def zipf_docs(n_docs, length, vocab, s=1.1, seed=1):
    """[{'name', 'ids'}] calibration documents."""
    g = torch.Generator().manual_seed(seed)
    return [dict(name=f"zipf{s}-seed{seed}-{j}", ids=zipf_ids(length, vocab, s, generator=g)) for j in range(n_docs)]


def uniform_prompt(n, vocab, seed=2):
    return torch.randint(0, vocab, (n,), generator=torch.Generator().manual_seed(seed))


def synthetic_maps(d, split, n_layers, device, seed=123, dtype=torch.bfloat16):
    """Ridge maps of the right shape for benchmarks without a fit: per late layer i in [split, n_layers),
    W_i = 0.9 I + N(0, 0.01) [d, d] and c_i ~ N(0, 0.01) [d], drawn in layer order from one seeded generator on
    `device` (the same maps on every run of every implementation on that device type)."""
    g = torch.Generator(device=device).manual_seed(seed)
    W, B = {}, {}
    for i in range(split, n_layers):
        w = 0.01 * torch.randn(d, d, device=device, generator=g)
        w.diagonal().add_(0.9)
        W[i] = w.to(dtype)
        B[i] = (0.01 * torch.randn(d, device=device, generator=g)).to(dtype)
    return W, B
