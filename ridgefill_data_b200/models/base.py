"""Model base: the per-layer API over explicit caches that the RidgeFill engine drives.

  layer(i, h, pos, cache)        exact layer on rows h (positions pos), appending to cache[i]
  fill(i, x, pos, cache)         cache-only fill from (predicted) layer inputs x: attention K/V, or the
                                 Gated DeltaNet conv + recurrent state; no attention output, no MLP
  fill_kv(i, k, v, pos, cache)   attention cache fill from given pre-RoPE K/V
  layer_rows(i, x, pos, rows, cache)  fill, plus the exact layer output of rows x[rows]
  queries(i, x, pos)             post-RoPE queries of normed inputs (the qattn selector)
  reads(i, x)                    what layer i reads from its input (pre-RoPE K/V, or GDN in-projections)
  forward_exact(ids, hook, keep) exact forward over all rows

The same API as the reference's model module (code/kva/model.py:1-18); subclasses define the math.
This module is the torch implementation (CPU oracle, fp32-capable); models/b200.py overrides the
layer math with the sm_100a kernels.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import oracle as ops
from .checkpoint import Checkpoint, DictSource, RandomSource, random_weights
from .config import ModelConfig

MLP_ROWS = 4096      # MLP row block (bounds the [rows, FFN] intermediate)
KV_RESERVE = 64      # spare K/V rows per layer buffer (decode appends in place)
GDN_ROWS = 8192      # Gated DeltaNet row segment (a multiple of the 64-token chunk)
ROW_BYTES = 1 << 25  # layer_rows: exact rows beyond one [rows, hidden] activation of this size go in runs


def _rows(fn, x, block=MLP_ROWS):
    if x.shape[0] <= block:
        return fn(x)
    return torch.cat([fn(x[a:a + block]) for a in range(0, x.shape[0], block)], 0)


class Model:
    """Shared machinery: config, weights, embedding, logits, KV append, exact forward."""

    def __init__(self, cfg: ModelConfig, source, device="cpu", dtype=torch.bfloat16, load_lm_head=True,
                 extras=True):
        self.cfg = cfg
        self.source = source
        self.device = torch.device(device)
        self.dtype = dtype
        self.n_layers = cfg.n_layers
        self.hidden = cfg.hidden
        self.eps = cfg.eps
        self.max_positions = cfg.max_positions
        self.layer_types = list(cfg.layer_types)
        self.n_heads, self.n_kv, self.head_dim = cfg.n_heads, cfg.n_kv, cfg.head_dim
        self.scale = self.head_dim ** -0.5
        self.prefix = self._prefix()
        self._setup()
        self.W = [self._load_layer(i) for i in range(self.n_layers)]
        p = self.prefix
        self.embed_w = self._get(f"{p}embed_tokens.weight")
        self.norm_w = self._get(f"{p}norm.weight")
        if load_lm_head:
            self.lm_head = self.embed_w if cfg.tie_embeddings else self._get("lm_head.weight")
        else:
            self.lm_head = None
        self.swift = None
        if extras:
            self._load_extras()

    # ---- construction helpers
    def _prefix(self):
        src = self.source
        if "model.language_model.embed_tokens.weight" in src:
            return "model.language_model."
        return "model."

    def _get(self, key):
        return self.source.get(key, self.device, self.dtype)

    def _get_raw(self, key):
        return self.source.get(key, self.device)

    def _setup(self):
        pass

    def _load_extras(self):
        pass

    # ---- common ops
    def new_cache(self):
        """One empty per-layer cache entry per layer."""
        return [{} for _ in range(self.n_layers)]

    def embed(self, ids):
        return F.embedding(ids.to(self.embed_w.device), self.embed_w).to(self.device)

    def final_norm(self, h):
        return self.in_norm(h, self.norm_w)

    def logits(self, h):
        return F.linear(self.final_norm(h), self.lm_head).float()

    def mlp(self, i, h):
        w = self.W[i]

        def run(x):
            x = self.post_norm(x, w["ln2"])
            act = F.silu(F.linear(x, w["gate"])) * F.linear(x, w["up"])
            return F.linear(act, w["down"])

        return h + _rows(run, h)

    def row_block(self):
        return max(1, ROW_BYTES // (self.hidden * self.dtype.itemsize))

    def mlp_rows(self, i, h):
        limit = self.row_block()
        if h.shape[0] <= limit:
            return self.mlp(i, h)
        step = max(MLP_ROWS, (limit // MLP_ROWS) * MLP_ROWS)     # whole MLP blocks per run, in place
        for lo in range(0, h.shape[0], step):
            h[lo:lo + step] = self.mlp(i, h[lo:lo + step])
        return h

    def _append_kv(self, cache, k, v):
        """Append rows k, v [Hkv, m, d] to the layer's K/V. Storage is a capacity-grown buffer written
        in place; cache['k'] / cache['v'] are views of the first cache['n'] rows. Shallow copies of a
        cache (per-arm forks) share the buffer; rows below every copy's length are never rewritten
        (code/kva/model.py:139-159)."""
        have = cache.get("n", 0)
        total = have + k.shape[1]
        if "kbuf" not in cache or total > cache["kbuf"].shape[1]:
            grown = {}
            for name, rows in (("kbuf", k), ("vbuf", v)):
                buf = rows.new_empty(rows.shape[0], total + KV_RESERVE, rows.shape[2])
                if have:
                    buf[:, :have] = cache[name][:, :have]
                grown[name] = buf
            cache.update(grown)
        cache["kbuf"][:, have:total] = k
        cache["vbuf"][:, have:total] = v
        cache["n"] = total
        cache["k"] = cache["kbuf"][:, :total]
        cache["v"] = cache["vbuf"][:, :total]

    def _heads(self, x, n_heads):
        return x.view(x.shape[0], n_heads, self.head_dim).transpose(0, 1)

    def fill_kv(self, i, k, v, pos, cache):
        """Attention cache fill from pre-RoPE K and V [tokens, kv_heads, head_dim]."""
        k_heads, v_heads = k.transpose(0, 1), v.transpose(0, 1)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, k.dtype)
        self._append_kv(cache[i], ops.apply_rope(k_heads, cos, sin), v_heads)

    def stable(self, h):
        """h itself, or a copy when h lives in a buffer that later layers reuse (tensor-parallel outputs)."""
        tp = getattr(self, "tp", None)
        return h.clone() if tp is not None and hasattr(tp, "owns") and tp.owns(h) else h

    def decode_batch(self, toks, positions, caches):
        """Next-token logits [R, V] fp32 of R independent sequences advanced by one token each: token toks[r] at
        position positions[r] over caches[r] (appended in place). This reference version runs the sequences one
        after another; the B200 model batches every projection and MLP over the R rows."""
        outs = []
        for t, p, c in zip(toks, positions, caches):
            pos = torch.tensor([int(p)], device=self.device)
            h = self.embed(torch.tensor([int(t)], device=self.device))
            for i in range(self.n_layers):
                h = self.layer(i, h, pos, c)
            outs.append(self.logits(h))
        return torch.cat(outs)

    def forward_exact(self, ids, hook=None, cache=None, keep=None, gdn_checkpoint_every=None, mix=None):
        """Exact forward over all rows. hook(i, h) sees each layer's input and hook('final', h) the
        final-norm input; mix(i, a) each layer's mixer output. keep: row indices whose logits to return."""
        if cache is None:
            cache = self.new_cache()
        positions = torch.arange(ids.shape[0], device=self.device)
        h = self.embed(ids)
        for i in range(self.n_layers):
            if hook is not None:
                hook(i, self.stable(h))
            h = self.layer(i, h, positions, cache, gdn_checkpoint_every=gdn_checkpoint_every, mix=mix)
        if hook is not None:
            hook("final", self.stable(h))
        return (None if keep is None else self.logits(h[keep])), cache


def model_class(cfg: ModelConfig, backend="torch"):
    """The class for cfg.arch and backend ('torch': this module's math on any device; 'b200': the
    sm_100a kernels). Unknown architectures never fall back to Llama's layer."""
    from . import hybrid, llama
    table = {"llama": llama.Llama, "qwen3": llama.Qwen3, "qwen3_5": hybrid.Hybrid, "qwen3_5_moe": hybrid.Hybrid}
    if backend == "b200":
        from . import b200
        table = {"llama": b200.B200Llama, "qwen3": b200.B200Llama, "qwen3_5": b200.B200Hybrid,
                 "qwen3_5_moe": b200.B200Hybrid}
    elif backend != "torch":
        raise ValueError(f"backend {backend!r} (torch | b200)")
    return table[cfg.arch]


def load(path, device="cpu", dtype=torch.bfloat16, backend="torch", verify=True, **kw):
    """The model at `path` (config.json + safetensors), files checked against <path>/SHA256SUMS when
    present (utils/integrity.py), reloaded once after dropping corrupted cached pages."""
    from ..utils import integrity
    cfg = ModelConfig.from_dir(path)
    cls = model_class(cfg, backend)
    m = cls(cfg, Checkpoint(path), device=device, dtype=dtype, **kw)
    if not verify:
        return m
    bad = integrity.verify_model(path)
    if not bad:
        return m
    m.source.files.clear()
    del m
    for name in bad:
        integrity.drop_cache(path / name if hasattr(path, "__truediv__") else f"{path}/{name}")
    m = cls(cfg, Checkpoint(path), device=device, dtype=dtype, **kw)
    bad = integrity.verify_model(path)
    if bad:
        raise integrity.IntegrityError(f"{path}: {', '.join(bad)} still read corrupted after a reload")
    return m


def from_config(cfg: ModelConfig, seed=0, device="cpu", dtype=torch.bfloat16, backend="torch", std=0.02,
                weights=None, lazy=None, **kw):
    """A random-init model of cfg. Default: every tensor drawn on the target device from a (seed, name)
    generator (RandomSource: no host copy); weights= a state dict; lazy=False: the host-generated
    random_weights (bitwise identical on every machine)."""
    cls = model_class(cfg, backend)
    if weights is not None:
        src = DictSource(weights)
    elif lazy is False:
        src = DictSource(random_weights(cfg, seed=seed, std=std))
    else:
        src = RandomSource(cfg, seed=seed, std=std)
    return cls(cfg, src, device=device, dtype=dtype, **kw)
