"""Llama-3.1 (with the SwiftKV extras) and dense Qwen3 layers in torch (code/kva/model.py:184-359).

Qwen3 is Llama's layer with a per-head RMSNorm on queries and keys after the projection and before
RoPE; every K the model writes or reads goes through _kv / reads, so fills and projector scoring
see the normed keys.
"""
from __future__ import annotations

import torch.nn.functional as F

from ..ops import oracle as ops
from .base import Model


class Llama(Model):
    def _setup(self):
        c = self.cfg
        if c.rope_type == "llama3":
            l3 = c.rope_llama3
            self.inv_freq = ops.inv_freq_llama3(c.rope_theta, c.head_dim, l3["factor"], l3["low_freq_factor"],
                                                l3["high_freq_factor"], l3["original_max_position_embeddings"])
        else:
            self.inv_freq = ops.inv_freq_default(c.rope_theta, c.rot_dim)
        self.swift_layers = c.swift_layers

    def _load_layer(self, i):
        p = f"{self.prefix}layers.{i}."
        g = self._get
        w = dict(ln1=g(p + "input_layernorm.weight"), ln2=g(p + "post_attention_layernorm.weight"),
                 q=g(p + "self_attn.q_proj.weight"), k=g(p + "self_attn.k_proj.weight"),
                 v=g(p + "self_attn.v_proj.weight"), o=g(p + "self_attn.o_proj.weight"),
                 gate=g(p + "mlp.gate_proj.weight"), up=g(p + "mlp.up_proj.weight"),
                 down=g(p + "mlp.down_proj.weight"))
        if self.cfg.qk_norm:
            w.update(q_norm=g(p + "self_attn.q_norm.weight"), k_norm=g(p + "self_attn.k_norm.weight"))
        return w

    def _load_extras(self):
        if self.swift_layers is None:
            return
        self.swift = dict(norm=self._get(f"{self.prefix}norm_swiftkv.weight"))
        for i in range(self.swift_layers, self.n_layers):
            a = f"{self.prefix}layers.{i}.self_attn."
            self.swift[i] = dict(q=self._get(a + "q_proj_swiftkv.weight"), k=self._get(a + "k_proj_swiftkv.weight"),
                                 v=self._get(a + "v_proj_swiftkv.weight"))

    def in_norm(self, x, w):
        return ops.rms_norm(x, w, self.eps)

    post_norm = in_norm

    def _knorm(self, k, w):
        return ops.rms_norm(k, w["k_norm"], self.eps) if self.cfg.qk_norm else k

    def _qnorm(self, q, w):
        return ops.rms_norm(q, w["q_norm"], self.eps) if self.cfg.qk_norm else q

    def _kv(self, i, x, pos):
        w = self.W[i]
        k = self._knorm(self._heads(F.linear(x, w["k"]), self.n_kv), w)
        v = self._heads(F.linear(x, w["v"]), self.n_kv)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, x.dtype)
        return ops.apply_rope(k, cos, sin), v

    def queries(self, i, x, pos):
        w = self.W[i]
        q = self._qnorm(self._heads(F.linear(x, w["q"]), self.n_heads), w)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, x.dtype)
        return ops.apply_rope(q, cos, sin)

    def layer(self, i, h, pos, cache, mix=None, **_):
        w = self.W[i]
        x = self.in_norm(h, w["ln1"])
        q = self.queries(i, x, pos)
        k, v = self._kv(i, x, pos)
        self._append_kv(cache[i], k, v)
        o = ops.attend(q, cache[i]["k"], cache[i]["v"], self.scale)
        a = F.linear(o, w["o"])
        if mix is not None:
            mix(i, a)
        return self.mlp(i, h + a)

    def layer_rows(self, i, h, pos, rows, cache):
        """Fill cache[i] from all rows' inputs h (an empty cache, pos = 0..n-1); return the exact layer
        output of h[rows] over that cache (= layer(...)[rows])."""
        w = self.W[i]
        x = self.in_norm(h, w["ln1"])
        k, v = self._kv(i, x, pos)
        self._append_kv(cache[i], k, v)
        q = self.queries(i, x[rows], pos[rows])
        o = ops.attend_at(q, cache[i]["k"], cache[i]["v"], self.scale, pos[rows])
        hr = h[rows] + F.linear(o, w["o"])
        return self.mlp_rows(i, hr)

    def fill(self, i, x, pos, cache, **_):
        k, v = self._kv(i, self.in_norm(x, self.W[i]["ln1"]), pos)
        self._append_kv(cache[i], k, v)
        return {}

    def reads(self, i, x):
        """Pre-RoPE K (k-normed for Qwen3) and V per KV head: [tokens, kv_heads, head_dim] each."""
        w = self.W[i]
        x = self.in_norm(x, w["ln1"])
        n = x.shape[0]
        k = F.linear(x, w["k"]).view(n, self.n_kv, -1)
        if self.cfg.qk_norm:
            k = ops.rms_norm(k, w["k_norm"], self.eps)
        return dict(k=k, v=F.linear(x, w["v"]).view(n, self.n_kv, -1))

    # ---- SwiftKV: late-layer K/V from norm_swiftkv(boundary) through *_proj_swiftkv
    def swift_fill(self, i, b, pos, cache):
        s = self.swift
        xs = ops.rms_norm(b, s["norm"], self.eps)
        k = self._heads(F.linear(xs, s[i]["k"]), self.n_kv)
        v = self._heads(F.linear(xs, s[i]["v"]), self.n_kv)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, b.dtype)
        self._append_kv(cache[i], ops.apply_rope(k, cos, sin), v)

    def swift_layer(self, i, h, pos, cache):
        """SwiftKV's late layer for query rows whose own K/V are already cached: queries through
        q_proj_swiftkv; attention, o_proj and MLP as the base layer."""
        w = self.W[i]
        x = self.in_norm(h, w["ln1"])
        q = self._heads(F.linear(x, self.swift[i]["q"]), self.n_heads)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, x.dtype)
        q = ops.apply_rope(q, cos, sin)
        o = ops.attend(q, cache[i]["k"], cache[i]["v"], self.scale)
        return self.mlp(i, h + F.linear(o, w["o"]))


class Qwen3(Llama):
    """Dense Qwen3: Llama's layer plus q_norm / k_norm (plain RMSNorm weight) before RoPE."""

    def _load_extras(self):
        self.swift = None
