"""The Qwen3.5-style hybrid in torch: Gated DeltaNet layers and gated full-attention layers
(code/kva/model.py:362-571), plus the mixture-of-experts MLP of the MoE variant (qwen3_5_moe:
softmax router, top-k renormalised, routed SwiGLU experts, a shared expert under a sigmoid gate).

Gated attention: q_proj emits [q | gate] per head; q/k get a zero-centred RMSNorm over head_dim,
partial RoPE on the first rot dims; the attention output is multiplied by sigmoid(gate).
Gated DeltaNet: in_proj_qkv -> depthwise causal conv (K=4) + SiLU -> q, k l2-normed (q scaled by
dk^-0.5), QK heads repeated to the V heads, beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias)
-> chunked delta rule -> gated RMSNorm with silu(z) -> out_proj.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import oracle as ops
from .base import GDN_ROWS, Model


class Hybrid(Model):
    def _setup(self):
        c = self.cfg
        self.inv_freq = ops.inv_freq_default(c.rope_theta, c.rot_dim)
        self.nk, self.nv, self.dk, self.dv = c.gdn_nk, c.gdn_nv, c.gdn_dk, c.gdn_dv
        self.conv_k = c.conv_k
        self.swift_layers = None

    def _load_layer(self, i):
        p = f"{self.prefix}layers.{i}."
        g = self._get
        w = dict(ln1=g(p + "input_layernorm.weight"), ln2=g(p + "post_attention_layernorm.weight"))
        if self.cfg.moe:
            m = p + "mlp."
            if m + "experts.gate_up_proj" in self.source:        # fused [E, 2F, d] / [E, d, F]
                gu, dn = g(m + "experts.gate_up_proj"), g(m + "experts.down_proj")
            else:                                                 # per-expert tensors (on-disk HF layout)
                ex = range(self.cfg.n_experts)
                gu = torch.stack([torch.cat((g(f"{m}experts.{e}.gate_proj.weight"), g(f"{m}experts.{e}.up_proj.weight")))
                                  for e in ex])
                dn = torch.stack([g(f"{m}experts.{e}.down_proj.weight") for e in ex])
            w.update(router=g(m + "gate.weight"), experts_gu=gu,
                     experts_down=dn, sh_gate=g(m + "shared_expert.gate_proj.weight"),
                     sh_up=g(m + "shared_expert.up_proj.weight"), sh_down=g(m + "shared_expert.down_proj.weight"),
                     sh_gate_w=g(m + "shared_expert_gate.weight"))
        else:
            w.update(gate=g(p + "mlp.gate_proj.weight"), up=g(p + "mlp.up_proj.weight"),
                     down=g(p + "mlp.down_proj.weight"))
        if self.layer_types[i] == "attn":
            a = p + "self_attn."
            w.update(q=g(a + "q_proj.weight"), k=g(a + "k_proj.weight"), v=g(a + "v_proj.weight"),
                     o=g(a + "o_proj.weight"), q_norm=g(a + "q_norm.weight"), k_norm=g(a + "k_norm.weight"))
        else:
            a = p + "linear_attn."
            w.update(qkv=g(a + "in_proj_qkv.weight"), z=g(a + "in_proj_z.weight"), b=g(a + "in_proj_b.weight"),
                     a=g(a + "in_proj_a.weight"), conv=g(a + "conv1d.weight").squeeze(1),
                     A_log=self._get_raw(a + "A_log"), dt_bias=self._get_raw(a + "dt_bias"),
                     norm=g(a + "norm.weight"), out=g(a + "out_proj.weight"))
        return w

    def in_norm(self, x, w):
        return ops.rms_norm_zc(x, w, self.eps)

    post_norm = in_norm

    # ---- MLP (dense or mixture of experts)
    def mlp(self, i, h):
        if not self.cfg.moe:
            return super().mlp(i, h)
        w = self.W[i]
        x = self.post_norm(h, w["ln2"])
        return h + self.moe_mlp(w, x)

    def moe_mlp(self, w, x):
        """Routed experts + gated shared expert on normed rows x [n, d]."""
        weights, experts = ops.router_topk(F.linear(x, w["router"]), self.cfg.top_k)
        out = torch.zeros_like(x)
        f = self.cfg.moe_intermediate
        for e in experts.unique().tolist():
            tok, slot = (experts == e).nonzero(as_tuple=True)
            gu = F.linear(x[tok], w["experts_gu"][e])
            y = F.linear(F.silu(gu[:, :f]) * gu[:, f:], w["experts_down"][e])
            out.index_add_(0, tok, (y * weights[tok, slot, None]).to(out.dtype))
        sh = F.linear(F.silu(F.linear(x, w["sh_gate"])) * F.linear(x, w["sh_up"]), w["sh_down"])
        return out + torch.sigmoid(F.linear(x, w["sh_gate_w"])) * sh

    # ---- gated attention
    def _attn_kv(self, i, x, pos):
        w = self.W[i]
        n = x.shape[0]
        k = ops.rms_norm_zc(F.linear(x, w["k"]).view(n, self.n_kv, self.head_dim), w["k_norm"], self.eps)
        v = F.linear(x, w["v"]).view(n, self.n_kv, self.head_dim)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, x.dtype)
        return ops.apply_rope(k.transpose(0, 1), cos, sin), v.transpose(0, 1)

    def _attn_q(self, i, x, pos):
        """Post-RoPE queries [Hq, n, d] and the output gate [n, Hq * d]."""
        w = self.W[i]
        n = x.shape[0]
        qg = F.linear(x, w["q"]).view(n, self.n_heads, 2 * self.head_dim)
        q, gate = qg[..., :self.head_dim], qg[..., self.head_dim:].reshape(n, -1)
        q = ops.rms_norm_zc(q, w["q_norm"], self.eps).transpose(0, 1)
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, x.dtype)
        return ops.apply_rope(q, cos, sin), gate

    def queries(self, i, x, pos):
        return self._attn_q(i, x, pos)[0]

    def _attn_layer(self, i, h, pos, cache):
        w = self.W[i]
        x = self.in_norm(h, w["ln1"])
        q, gate = self._attn_q(i, x, pos)
        k, v = self._attn_kv(i, x, pos)
        self._append_kv(cache[i], k, v)
        o = ops.attend(q, cache[i]["k"], cache[i]["v"], self.scale)
        return F.linear(o * torch.sigmoid(gate), w["o"])

    # ---- Gated DeltaNet
    def _gdn_inputs(self, i, x):
        w = self.W[i]
        return F.linear(x, w["qkv"]), F.linear(x, w["b"]), F.linear(x, w["a"])

    def gdn_gates(self, i, b, a):
        """beta [Hv, n] and log decay g [Hv, n] in fp32 from the b / a projections [n, Hv]."""
        w = self.W[i]
        beta = torch.sigmoid(b).float().T
        g = (-w["A_log"].float().exp() * F.softplus(a.float() + w["dt_bias"].float())).T
        return beta, g

    def gdn_qkv(self, conv_out):
        """Split conv output rows [m, C] into q (l2-normed, scaled), k (l2-normed) repeated to the V heads
        and v: [Hv, m, d] fp32 each."""
        m = conv_out.shape[0]
        kd = self.nk * self.dk
        rep = self.nv // self.nk
        q, k, v = conv_out.split([kd, kd, self.nv * self.dv], -1)
        q = q.reshape(m, self.nk, self.dk).float().repeat_interleave(rep, 1).transpose(0, 1)
        k = k.reshape(m, self.nk, self.dk).float().repeat_interleave(rep, 1).transpose(0, 1)
        v = v.reshape(m, self.nv, self.dv).float().transpose(0, 1)
        return ops.l2norm(q) * self.dk ** -0.5, ops.l2norm(k), v

    def _gdn_core(self, i, pre, b, a, cache, need_out, checkpoint_every=None, offset=0):
        """Conv + delta rule over pre-conv rows, continuing cache[i]'s conv and recurrent states, in
        GDN_ROWS segments. Returns (out [Hv, n, dv] in pre.dtype or None, checkpoints)."""
        w = self.W[i]
        c = cache[i]
        n = pre.shape[0]
        outs, ck = [], {}
        for r0 in range(0, n, GDN_ROWS):
            r1 = min(n, r0 + GDN_ROWS)
            conv_out, c["conv"] = ops.causal_conv(pre[r0:r1], c.get("conv"), w["conv"])
            q, k, v = self.gdn_qkv(conv_out)
            beta, g = self.gdn_gates(i, b[r0:r1], a[r0:r1])
            if r1 - r0 == 1 and not checkpoint_every:
                out, state = ops.delta_rule_recurrent(q, k, v, g, beta, c.get("rec"))
            else:
                out, state, part = ops.delta_rule(q, k, v, g, beta, c.get("rec"), checkpoint_every=checkpoint_every,
                                                  offset=offset + r0, need_out=need_out)
                ck.update(part)
            c["rec"] = state
            if need_out:
                outs.append(out.to(pre.dtype))
        c["len"] = c.get("len", 0) + n
        return (torch.cat(outs, 1) if need_out else None), ck

    def _gdn_out(self, i, out, x):
        """Gated RMSNorm with silu(z) and out_proj for core outputs out [Hv, n, dv] of normed rows x."""
        w = self.W[i]
        n = x.shape[0]
        z = F.linear(x, w["z"]).view(n, self.nv, self.dv)
        y = ops.rms_norm_gated(out.transpose(0, 1), z, w["norm"], self.eps).reshape(n, -1)
        return F.linear(y, w["out"])

    def _gdn_layer(self, i, h, pos, cache, checkpoint_every=None):
        x = self.in_norm(h, self.W[i]["ln1"])
        pre, b, a = self._gdn_inputs(i, x)
        out, ck = self._gdn_core(i, pre, b, a, cache, True, checkpoint_every, cache[i].get("len", 0))
        if ck:
            cache[i].setdefault("checkpoints", {}).update(ck)
        return self._gdn_out(i, out, x)

    def layer(self, i, h, pos, cache, gdn_checkpoint_every=None, mix=None):
        if self.layer_types[i] == "attn":
            a = self._attn_layer(i, h, pos, cache)
        else:
            a = self._gdn_layer(i, h, pos, cache, gdn_checkpoint_every)
        if mix is not None:
            mix(i, a)
        return self.mlp(i, h + a)

    def fill(self, i, x, pos, cache, st=None, checkpoint_every=None):
        """Cache-only fill from (predicted) inputs. GDN: conv + recurrent state over the rows, then the
        terminal-state correction st added when given (code/kva/model.py:510-523)."""
        x = self.in_norm(x, self.W[i]["ln1"])
        if self.layer_types[i] == "attn":
            k, v = self._attn_kv(i, x, pos)
            self._append_kv(cache[i], k, v)
            return {}
        pre, b, a = self._gdn_inputs(i, x)
        _, ck = self._gdn_core(i, pre, b, a, cache, False, checkpoint_every, cache[i].get("len", 0))
        if st is not None:
            cache[i]["rec"] = cache[i]["rec"] + st.to(cache[i]["rec"])
        return ck

    def fill_kv(self, i, k, v, pos, cache):
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, k.dtype)
        self._append_kv(cache[i], ops.apply_rope(k.transpose(0, 1), cos, sin), v.transpose(0, 1))

    def layer_rows(self, i, h, pos, rows, cache):
        """Fill from all rows' inputs h; return the exact output of h[rows]. GDN: the delta rule runs with
        outputs over all rows (a row's output needs the state at its position)."""
        w = self.W[i]
        x = self.in_norm(h, w["ln1"])
        xr = x[rows]
        if self.layer_types[i] == "attn":
            k, v = self._attn_kv(i, x, pos)
            self._append_kv(cache[i], k, v)
            q, gate = self._attn_q(i, xr, pos[rows])
            o = ops.attend_at(q, cache[i]["k"], cache[i]["v"], self.scale, pos[rows])
            hr = h[rows] + F.linear(o * torch.sigmoid(gate), w["o"])
        else:
            pre, b, a = self._gdn_inputs(i, x)
            out, _ = self._gdn_core(i, pre, b, a, cache, True, offset=cache[i].get("len", 0))
            hr = h[rows] + self._gdn_out(i, out[:, rows], xr)
        return self.mlp_rows(i, hr)

    def reads(self, i, x):
        """Attention: k-normed pre-RoPE K and V per KV head. GDN: pre-conv q/k/v per head and the
        beta/decay pre-activations."""
        w = self.W[i]
        x = self.in_norm(x, w["ln1"])
        n = x.shape[0]
        if self.layer_types[i] == "attn":
            k = ops.rms_norm_zc(F.linear(x, w["k"]).view(n, self.n_kv, self.head_dim), w["k_norm"], self.eps)
            return dict(k=k, v=F.linear(x, w["v"]).view(n, self.n_kv, self.head_dim))
        pre, b, a = self._gdn_inputs(i, x)
        kd = self.nk * self.dk
        q, k, v = pre.split([kd, kd, self.nv * self.dv], -1)
        return dict(q=q.reshape(n, self.nk, self.dk), k=k.reshape(n, self.nk, self.dk),
                    v=v.reshape(n, self.nv, self.dv), ba=torch.cat((b, a), -1)[:, None, :])
