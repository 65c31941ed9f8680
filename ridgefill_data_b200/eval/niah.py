"""Synthetic needle-in-a-haystack prompts in token-id space (no tokenizer or dataset needed on the GPU boxes).

A haystack of Zipf(1.1) filler ids holds `n_keys` needles "KEY_i -> VALUE_i" (each a short run of reserved ids)
at relative depths; the prompt ends with a query run naming the target key. Scoring is exact: the greedy
continuation must reproduce the target's value ids. The shape follows the reference's K20 NIAH generator
(lengths 8704 / 16384 / 32768, depths 0.1 .. 0.9; code/kva/data.py:140-237) so the same depth x length grid can
be run on synthetic weights; with a real tokenizer, text variants can be built from data files instead.
"""
from __future__ import annotations

import torch

from .data import zipf_ids

LENGTHS = (8704, 16384, 32768)
DEPTHS = (0.1, 0.3, 0.5, 0.7, 0.9)


def niah_prompt(length, vocab, depth, n_keys=4, key_len=4, value_len=6, seed=0, reserved=256):
    """dict(ids [length], key, value, needle_start, needle_end, target) with the target needle at `depth`."""
    g = torch.Generator().manual_seed(seed)
    fill_vocab = vocab - reserved
    ids = zipf_ids(length, fill_vocab, seed=seed + 1) + reserved
    keys = [torch.randint(0, reserved // 2, (key_len,), generator=g) for _ in range(n_keys)]
    vals = [torch.randint(reserved // 2, reserved, (value_len,), generator=g) for _ in range(n_keys)]
    target = int(torch.randint(0, n_keys, (1,), generator=g))
    query = torch.cat((keys[target], torch.tensor([0])))
    body = length - query.numel()
    spans = {}
    for j in range(n_keys):
        d = depth if j == target else float(torch.rand(1, generator=g)) * 0.9 + 0.05
        start = min(body - key_len - value_len - 1, int(d * body))
        needle = torch.cat((keys[j], vals[j]))
        ids[start:start + needle.numel()] = needle
        spans[j] = (start, start + needle.numel())
    ids[body:] = query
    s, e = spans[target]
    return dict(ids=ids, key=keys[target], value=vals[target], needle_start=s, needle_end=e, target=target)


def niah_correct(generated, value):
    v = value.tolist()
    gen = list(generated)
    return any(gen[i:i + len(v)] == v for i in range(max(1, len(gen) - len(v) + 1)))
