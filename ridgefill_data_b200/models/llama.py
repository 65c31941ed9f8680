"""Llama-3.1 (with the SwiftKV extras) and dense Qwen3 layers in plain torch: the CPU / fp32 oracle of the
layer API (the model family of code/kva/model.py:184-359).

Dense Qwen3 is the Llama layer with a per-head RMSNorm on the projected queries and keys, applied before RoPE.
Every key the model writes or exposes passes through _kv or reads, so fills and projector scoring see normed keys.
"""
from __future__ import annotations

import torch.nn.functional as F

from ..ops import oracle as ops
from .base import Model

# our weight name -> tensor name under model.layers.<i>. (the Hugging Face checkpoint layout)
_LAYER = dict(ln1="input_layernorm", ln2="post_attention_layernorm", q="self_attn.q_proj", k="self_attn.k_proj",
              v="self_attn.v_proj", o="self_attn.o_proj", gate="mlp.gate_proj", up="mlp.up_proj",
              down="mlp.down_proj")
_QK_NORM = dict(q_norm="self_attn.q_norm", k_norm="self_attn.k_norm")
_SWIFT = dict(q="q_proj_swiftkv", k="k_proj_swiftkv", v="v_proj_swiftkv")


class Llama(Model):
    def _setup(self):
        c = self.cfg
        if c.rope_type == "llama3":
            s = c.rope_llama3
            self.inv_freq = ops.inv_freq_llama3(c.rope_theta, c.head_dim, s["factor"], s["low_freq_factor"],
                                                s["high_freq_factor"], s["original_max_position_embeddings"])
        else:
            self.inv_freq = ops.inv_freq_default(c.rope_theta, c.rot_dim)
        self.swift_layers = c.swift_layers

    def _load_layer(self, i):
        base = f"{self.prefix}layers.{i}."
        names = dict(_LAYER, **(_QK_NORM if self.cfg.qk_norm else {}))
        return {ours: self._get(f"{base}{theirs}.weight") for ours, theirs in names.items()}

    def _load_extras(self):
        if self.swift_layers is None:
            return
        self.swift = {"norm": self._get(f"{self.prefix}norm_swiftkv.weight")}
        for i in range(self.swift_layers, self.n_layers):
            attn = f"{self.prefix}layers.{i}.self_attn."
            self.swift[i] = {ours: self._get(f"{attn}{theirs}.weight") for ours, theirs in _SWIFT.items()}

    def in_norm(self, x, w):
        return ops.rms_norm(x, w, self.eps)

    post_norm = in_norm

    def _rope(self, t, pos, dtype):
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, dtype)
        return ops.apply_rope(t, cos, sin)

    def _head_norm(self, t, w, which):
        return ops.rms_norm(t, w[which], self.eps) if self.cfg.qk_norm else t

    def _knorm(self, k, w):
        return self._head_norm(k, w, "k_norm")

    def _qnorm(self, q, w):
        return self._head_norm(q, w, "q_norm")

    def _kv(self, i, x, pos):
        """Post-RoPE K and V [kv_heads, n, head_dim] of normed inputs x."""
        w = self.W[i]
        k = self._knorm(self._heads(F.linear(x, w["k"]), self.n_kv), w)
        v = self._heads(F.linear(x, w["v"]), self.n_kv)
        return self._rope(k, pos, x.dtype), v

    def queries(self, i, x, pos):
        w = self.W[i]
        q = self._qnorm(self._heads(F.linear(x, w["q"]), self.n_heads), w)
        return self._rope(q, pos, x.dtype)

    def _attend_out(self, i, q, cache, at=None):
        c = cache[i]
        if at is None:
            o = ops.attend(q, c["k"], c["v"], self.scale)
        else:
            o = ops.attend_at(q, c["k"], c["v"], self.scale, at)
        return F.linear(o, self.W[i]["o"])

    def layer(self, i, h, pos, cache, mix=None, **_):
        x = self.in_norm(h, self.W[i]["ln1"])
        q = self.queries(i, x, pos)
        self._append_kv(cache[i], *self._kv(i, x, pos))
        a = self._attend_out(i, q, cache)
        if mix is not None:
            mix(i, a)
        return self.mlp(i, h + a)

    def layer_rows(self, i, h, pos, rows, cache):
        """Write cache[i] from every row's input h (an empty cache, pos = 0..n-1) and return the exact layer output
        of rows h[rows] against it, which equals layer(...)[rows]."""
        x = self.in_norm(h, self.W[i]["ln1"])
        self._append_kv(cache[i], *self._kv(i, x, pos))
        q = self.queries(i, x[rows], pos[rows])
        return self.mlp_rows(i, h[rows] + self._attend_out(i, q, cache, at=pos[rows]))

    def fill(self, i, x, pos, cache, **_):
        self._append_kv(cache[i], *self._kv(i, self.in_norm(x, self.W[i]["ln1"]), pos))
        return {}

    def reads(self, i, x):
        """K before RoPE (head-normed for Qwen3) and V: [tokens, kv_heads, head_dim] each."""
        w = self.W[i]
        x = self.in_norm(x, w["ln1"])
        n = x.shape[0]
        k = F.linear(x, w["k"]).view(n, self.n_kv, -1)
        if self.cfg.qk_norm:
            k = ops.rms_norm(k, w["k_norm"], self.eps)
        return {"k": k, "v": F.linear(x, w["v"]).view(n, self.n_kv, -1)}

    # ---- SwiftKV: late-layer K/V from norm_swiftkv(layer-split input) through the *_proj_swiftkv weights
    def swift_fill(self, i, b, pos, cache):
        sw = self.swift
        xs = ops.rms_norm(b, sw["norm"], self.eps)
        k = self._heads(F.linear(xs, sw[i]["k"]), self.n_kv)
        v = self._heads(F.linear(xs, sw[i]["v"]), self.n_kv)
        self._append_kv(cache[i], self._rope(k, pos, b.dtype), v)

    def swift_layer(self, i, h, pos, cache):
        """SwiftKV's late layer for query rows whose K/V are cached already: queries from q_proj_swiftkv, then
        attention, o_proj and the MLP of the base layer."""
        x = self.in_norm(h, self.W[i]["ln1"])
        q = self._rope(self._heads(F.linear(x, self.swift[i]["q"]), self.n_heads), pos, x.dtype)
        return self.mlp(i, h + self._attend_out(i, q, cache))


class Qwen3(Llama):
    """Dense Qwen3: the Llama layer with q_norm / k_norm (plain RMSNorm gains) ahead of RoPE."""

    def _load_extras(self):
        self.swift = None
