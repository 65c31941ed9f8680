"""The Qwen3.5-style hybrid in plain torch, the CPU / fp32 oracle of the layer API: Gated DeltaNet layers, gated
full-attention layers (the model of code/kva/model.py:362-571) and the mixture-of-experts MLP of the MoE variant
(softmax router, renormalised top-k, routed SwiGLU experts, a shared expert behind a sigmoid gate).

Gated attention: q_proj yields [q | gate] per head; q and k get a zero-centred RMSNorm over head_dim and partial
RoPE on their first rot dims; the attention output is scaled by sigmoid(gate) before o_proj.
Gated DeltaNet: in_proj_qkv, a depthwise causal conv (width 4) with SiLU, then q and k l2-normalised (q also
scaled by dk^-1/2) with the QK heads repeated up to the V heads; beta = sigmoid(b) and the log decay
g = -exp(A_log) * softplus(a + dt_bias) drive the chunked delta rule, whose output passes a gated RMSNorm with
silu(z) and out_proj.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

from ..ops import oracle as ops
from .base import GDN_ROWS, Model

# our weight name -> tensor name under model.layers.<i>. (the Hugging Face checkpoint layout)
_NORMS = dict(ln1="input_layernorm", ln2="post_attention_layernorm")
_DENSE_MLP = dict(gate="mlp.gate_proj", up="mlp.up_proj", down="mlp.down_proj")
_SHARED = dict(router="mlp.gate", sh_gate="mlp.shared_expert.gate_proj", sh_up="mlp.shared_expert.up_proj",
               sh_down="mlp.shared_expert.down_proj", sh_gate_w="mlp.shared_expert_gate")
_ATTN = dict(q="self_attn.q_proj", k="self_attn.k_proj", v="self_attn.v_proj", o="self_attn.o_proj",
             q_norm="self_attn.q_norm", k_norm="self_attn.k_norm")
_GDN = dict(qkv="linear_attn.in_proj_qkv", z="linear_attn.in_proj_z", b="linear_attn.in_proj_b",
            a="linear_attn.in_proj_a", norm="linear_attn.norm", out="linear_attn.out_proj")


class Hybrid(Model):
    def _setup(self):
        c = self.cfg
        self.inv_freq = ops.inv_freq_default(c.rope_theta, c.rot_dim)
        self.nk, self.nv = c.gdn_nk, c.gdn_nv
        self.dk, self.dv = c.gdn_dk, c.gdn_dv
        self.conv_k = c.conv_k
        self.swift_layers = None

    def _experts(self, base):
        """(gate|up [E, 2F, d], down [E, d, F]) of the routed experts, from fused or per-expert tensors."""
        mlp = base + "mlp.experts."
        if mlp + "gate_up_proj" in self.source:
            return self._get(mlp + "gate_up_proj"), self._get(mlp + "down_proj")
        gate_up, down = [], []
        for e in range(self.cfg.n_experts):
            gate_up.append(torch.cat((self._get(f"{mlp}{e}.gate_proj.weight"), self._get(f"{mlp}{e}.up_proj.weight"))))
            down.append(self._get(f"{mlp}{e}.down_proj.weight"))
        return torch.stack(gate_up), torch.stack(down)

    def _load_layer(self, i):
        base = f"{self.prefix}layers.{i}."
        names = dict(_NORMS)
        names.update(_SHARED if self.cfg.moe else _DENSE_MLP)
        names.update(_ATTN if self.layer_types[i] == "attn" else _GDN)
        w = {ours: self._get(f"{base}{theirs}.weight") for ours, theirs in names.items()}
        if self.cfg.moe:
            w["experts_gu"], w["experts_down"] = self._experts(base)
        if self.layer_types[i] != "attn":
            gdn = base + "linear_attn."
            w["conv"] = self._get(gdn + "conv1d.weight").squeeze(1)
            w["A_log"] = self._get_raw(gdn + "A_log")          # decay parameters stay in their stored dtype
            w["dt_bias"] = self._get_raw(gdn + "dt_bias")
        return w

    def in_norm(self, x, w):
        return ops.rms_norm_zc(x, w, self.eps)

    post_norm = in_norm

    # ---- MLP (dense, or the mixture of experts)
    def mlp(self, i, h):
        if not self.cfg.moe:
            return super().mlp(i, h)
        w = self.W[i]
        return h + self.moe_mlp(w, self.post_norm(h, w["ln2"]))

    def moe_mlp(self, w, x):
        """Routed experts plus the gated shared expert on normed rows x [n, d]."""
        weights, chosen = ops.router_topk(F.linear(x, w["router"]), self.cfg.top_k)
        f = self.cfg.moe_intermediate
        routed = torch.zeros_like(x)
        for e in chosen.unique().tolist():
            rows, slot = (chosen == e).nonzero(as_tuple=True)
            gate_up = F.linear(x[rows], w["experts_gu"][e])
            y = F.linear(F.silu(gate_up[:, :f]) * gate_up[:, f:], w["experts_down"][e])
            routed.index_add_(0, rows, (y * weights[rows, slot, None]).to(routed.dtype))
        shared = F.linear(F.silu(F.linear(x, w["sh_gate"])) * F.linear(x, w["sh_up"]), w["sh_down"])
        return routed + torch.sigmoid(F.linear(x, w["sh_gate_w"])) * shared

    # ---- gated attention
    def _rope(self, t, pos, dtype):
        cos, sin = ops.rope_cos_sin(self.inv_freq, pos, dtype)
        return ops.apply_rope(t, cos, sin)

    def _k_pre(self, w, x):
        """Head-normed K before RoPE and V, [n, kv_heads, head_dim] each."""
        n = x.shape[0]
        k = F.linear(x, w["k"]).view(n, self.n_kv, self.head_dim)
        v = F.linear(x, w["v"]).view(n, self.n_kv, self.head_dim)
        return ops.rms_norm_zc(k, w["k_norm"], self.eps), v

    def _attn_kv(self, i, x, pos):
        k, v = self._k_pre(self.W[i], x)
        return self._rope(k.transpose(0, 1), pos, x.dtype), v.transpose(0, 1)

    def _attn_q(self, i, x, pos):
        """Queries after RoPE [Hq, n, d] and the output gate [n, Hq * d]."""
        w = self.W[i]
        n, d = x.shape[0], self.head_dim
        both = F.linear(x, w["q"]).view(n, self.n_heads, 2 * d)
        gate = both[..., d:].reshape(n, -1)
        q = ops.rms_norm_zc(both[..., :d], w["q_norm"], self.eps).transpose(0, 1)
        return self._rope(q, pos, x.dtype), gate

    def queries(self, i, x, pos):
        return self._attn_q(i, x, pos)[0]

    def _gated_out(self, i, o, gate):
        return F.linear(o * torch.sigmoid(gate), self.W[i]["o"])

    def _attn_layer(self, i, h, pos, cache):
        x = self.in_norm(h, self.W[i]["ln1"])
        q, gate = self._attn_q(i, x, pos)
        self._append_kv(cache[i], *self._attn_kv(i, x, pos))
        c = cache[i]
        return self._gated_out(i, ops.attend(q, c["k"], c["v"], self.scale), gate)

    # ---- Gated DeltaNet
    def _gdn_inputs(self, i, x):
        w = self.W[i]
        return F.linear(x, w["qkv"]), F.linear(x, w["b"]), F.linear(x, w["a"])

    def gdn_gates(self, i, b, a):
        """beta [Hv, n] and log decay g [Hv, n] (fp32) from the b / a projections [n, Hv]."""
        w = self.W[i]
        beta = torch.sigmoid(b).float().T
        decay = w["A_log"].float().exp()
        g = -decay * F.softplus(a.float() + w["dt_bias"].float())
        return beta, g.T

    def _split_qkv(self, rows):
        kd = self.nk * self.dk
        return rows.split([kd, kd, self.nv * self.dv], -1)

    def gdn_qkv(self, conv_out):
        """q (l2-normed and scaled), k (l2-normed), both repeated to the V heads, and v from conv output rows
        [m, C]: [Hv, m, d] fp32 each."""
        m = conv_out.shape[0]
        q, k, v = self._split_qkv(conv_out)
        rep = self.nv // self.nk

        def per_v_head(t):
            return t.reshape(m, self.nk, self.dk).float().repeat_interleave(rep, 1).transpose(0, 1)

        q, k = per_v_head(q), per_v_head(k)
        v = v.reshape(m, self.nv, self.dv).float().transpose(0, 1)
        return ops.l2norm(q) * self.dk ** -0.5, ops.l2norm(k), v

    def _gdn_core(self, i, pre, b, a, cache, need_out, checkpoint_every=None, offset=0):
        """Causal conv and delta rule over pre-conv rows `pre`, continuing cache[i]'s conv window and state, in
        segments of GDN_ROWS rows. Returns (outputs [Hv, n, dv] in pre.dtype, or None; state checkpoints)."""
        conv_w = self.W[i]["conv"]
        st = cache[i]
        n = pre.shape[0]
        outs, checkpoints = [], {}
        for lo in range(0, n, GDN_ROWS):
            hi = min(n, lo + GDN_ROWS)
            conv_out, st["conv"] = ops.causal_conv(pre[lo:hi], st.get("conv"), conv_w)
            q, k, v = self.gdn_qkv(conv_out)
            beta, g = self.gdn_gates(i, b[lo:hi], a[lo:hi])
            if hi - lo == 1 and not checkpoint_every:
                out, st["rec"] = ops.delta_rule_recurrent(q, k, v, g, beta, st.get("rec"))
            else:
                out, st["rec"], part = ops.delta_rule(q, k, v, g, beta, st.get("rec"),
                                                      checkpoint_every=checkpoint_every, offset=offset + lo,
                                                      need_out=need_out)
                checkpoints.update(part)
            if need_out:
                outs.append(out.to(pre.dtype))
        st["len"] = st.get("len", 0) + n
        return (torch.cat(outs, 1) if need_out else None), checkpoints

    def _gdn_out(self, i, out, x):
        """Gated RMSNorm with silu(z), then out_proj, of core outputs out [Hv, n, dv] for normed rows x."""
        w = self.W[i]
        n = x.shape[0]
        z = F.linear(x, w["z"]).view(n, self.nv, self.dv)
        normed = ops.rms_norm_gated(out.transpose(0, 1), z, w["norm"], self.eps)
        return F.linear(normed.reshape(n, -1), w["out"])

    def _gdn_layer(self, i, h, pos, cache, checkpoint_every=None):
        x = self.in_norm(h, self.W[i]["ln1"])
        out, ck = self._gdn_core(i, *self._gdn_inputs(i, x), cache, True, checkpoint_every,
                                 cache[i].get("len", 0))
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
        """Cache-only fill from (predicted) inputs x: attention K/V, or the GDN conv window and recurrent state
        over the rows, plus the terminal-state correction st when one is given (code/kva/model.py:510-523)."""
        x = self.in_norm(x, self.W[i]["ln1"])
        if self.layer_types[i] == "attn":
            self._append_kv(cache[i], *self._attn_kv(i, x, pos))
            return {}
        _, ck = self._gdn_core(i, *self._gdn_inputs(i, x), cache, False, checkpoint_every, cache[i].get("len", 0))
        if st is not None:
            cache[i]["rec"] = cache[i]["rec"] + st.to(cache[i]["rec"])
        return ck

    def fill_kv(self, i, k, v, pos, cache):
        self._append_kv(cache[i], self._rope(k.transpose(0, 1), pos, k.dtype), v.transpose(0, 1))

    def layer_rows(self, i, h, pos, rows, cache):
        """Write cache[i] from every row's input h and return the exact layer output of rows h[rows]. A GDN layer
        produces outputs for all rows (a row's output needs the state at its own position)."""
        x = self.in_norm(h, self.W[i]["ln1"])
        xr = x[rows]
        if self.layer_types[i] == "attn":
            self._append_kv(cache[i], *self._attn_kv(i, x, pos))
            q, gate = self._attn_q(i, xr, pos[rows])
            c = cache[i]
            mixed = self._gated_out(i, ops.attend_at(q, c["k"], c["v"], self.scale, pos[rows]), gate)
        else:
            out, _ = self._gdn_core(i, *self._gdn_inputs(i, x), cache, True, offset=cache[i].get("len", 0))
            mixed = self._gdn_out(i, out[:, rows], xr)
        return self.mlp_rows(i, h[rows] + mixed)

    def reads(self, i, x):
        """Attention: head-normed K before RoPE and V per KV head. GDN: the in-projected q / k / v per head
        (before the conv) and the beta / decay pre-activations."""
        w = self.W[i]
        x = self.in_norm(x, w["ln1"])
        n = x.shape[0]
        if self.layer_types[i] == "attn":
            k, v = self._k_pre(w, x)
            return {"k": k, "v": v}
        pre, b, a = self._gdn_inputs(i, x)
        q, k, v = self._split_qkv(pre)
        return {"q": q.reshape(n, self.nk, self.dk), "k": k.reshape(n, self.nk, self.dk),
                "v": v.reshape(n, self.nv, self.dv), "ba": torch.cat((b, a), -1).unsqueeze(1)}
