"""B200 models: the layer math of models/llama.py and models/hybrid.py on the sm_100a kernels.

Weights are packed at load for the fused kernels:
  attention   qkv_p = [q (q|gate per head when gated) ; k ; v] rows -> one tcgen05 GEMM; the K/V rows are a
              contiguous row slice (the cache-only fill's GEMM)
  GDN         in_p = [in_proj_qkv ; in_proj_b ; in_proj_a ; in_proj_z] rows: the fill GEMM uses the prefix
              without z
  MLP         gu_p = gate/up interleaved per 128-row block -> one GEMM with a SwiGLU epilogue
The torch names (q, k, v, qkv, b, a, z, ...) stay as views of the packed tensors, so the diagnostic paths
inherited from the torch models (reads, queries, layer_rows, SwiftKV) keep working on the device.

Hot path per exact layer: rmsnorm -> GEMM -> head-norm/RoPE straight into the K/V cache (or conv + gates
-> chunked delta rule) -> flash attention with the gate epilogue (or gated rmsnorm) -> GEMM with the
residual add fused -> rmsnorm -> SwiGLU GEMM -> down GEMM with the residual add fused.
"""
from __future__ import annotations

import torch

from ..ops import gemm as G
from ..ops import kernels as K
from .base import KV_RESERVE
from .hybrid import Hybrid
from .llama import Llama


class _B200:
    """Kernel-backed overrides shared by the Llama-family and hybrid models."""

    zero_centred = False
    capacity_hint = 0
    kv_pool = None     # models.kvpool.KVPool: attention caches in shared pages (multi-sequence serving)
    tp = None          # parallel.tp.TensorParallel when the weights are sharded over ranks
    ep = None          # parallel.ep.ExpertParallel when the experts are spread over ranks

    # ---- setup
    def _kernel_setup(self):
        if self.device.type != "cuda":
            raise RuntimeError("the B200 backend needs a CUDA device")
        from ..ops._ext import ext
        ext()   # fail loudly when the extension is missing
        self._rope_tables = None
        self._span_cache = {}
        self.lm_head_f = None

    def rope(self, need):
        """bf16 cos/sin tables covering positions < need (grown on demand)."""
        if self._rope_tables is None or self._rope_tables[0].shape[0] < need:
            n = max(need, 8192, 2 * (self._rope_tables[0].shape[0] if self._rope_tables else 0))
            if self._rope_tables is not None:
                # a captured decode graph keeps reading the tables it was captured with: they stay allocated
                self.__dict__.setdefault("_retired_rope_tables", []).append(self._rope_tables)
            self._rope_tables = K.rope_tables(self.inv_freq, n, self.device)
        return self._rope_tables

    def reserve(self, n_tokens):
        """Size new attention caches for n_tokens rows (prompt + decode reserve), so appends never copy."""
        self.capacity_hint = int(n_tokens)

    def _span(self, pos):
        """(first position, int32 positions or None when pos is a contiguous range)."""
        key = (pos.data_ptr(), pos.numel(), pos.device)
        ent = self._span_cache.get(key)
        hit = ent[1] if ent is not None else None
        if hit is None:
            p = pos.to("cpu", torch.long)
            p0 = int(p[0]) if p.numel() else 0
            contiguous = bool(torch.equal(p, torch.arange(p0, p0 + p.numel())))
            hit = (p0, None if contiguous else pos.to(self.device, torch.int32).contiguous())
            if len(self._span_cache) > 64:
                self._span_cache.clear()
            self._span_cache[key] = (pos, hit)   # holding pos keeps its address from being reused
        return hit

    def _norm(self, x, w):
        return K.rmsnorm(x, w, self.eps, self.zero_centred)

    # ---- common
    def embed(self, ids):
        return K.embed(self.embed_w, ids.to(self.device))

    def final_norm(self, h):
        return self._norm(h, self.norm_w)

    def logits(self, h):
        return G.linear_f32(self.final_norm(h), self.lm_head)

    def mlp(self, i, h):
        w = self.W[i]
        if "gu_p" not in w:
            return super().mlp(i, h)
        x = K.rmsnorm(h, w["ln2"], self.eps, self.zero_centred)
        act = G.swiglu_linear(x, w["gu_p"])
        if self.tp is not None:
            return self.tp.row_parallel(act, w["down"], h)
        return G.linear(act, w["down"], residual=h)

    def _pack_mlp(self, w):
        if "gate" in w and w["gate"].shape[0] % 128 == 0:
            w["gu_p"] = G.pack_gate_up(w["gate"], w["up"]).contiguous()
            del w["gate"], w["up"]

    # ---- attention
    def _kv_reserve(self, c, m, i=None):
        n = c.get("n", 0)
        if self.kv_pool is not None:
            self.kv_pool.grow(i, c, n + m, self.device)
            return n
        kb = c.get("kbuf")
        if kb is None or n + m > kb.shape[1]:
            cap = max(n + m + KV_RESERVE, self.capacity_hint)
            shape = (self.n_kv, cap, self.head_dim)
            nkb = torch.empty(shape, dtype=self.dtype, device=self.device)
            nvb = torch.empty(shape, dtype=self.dtype, device=self.device)
            if n:
                nkb[:, :n] = c["kbuf"][:, :n]
                nvb[:, :n] = c["vbuf"][:, :n]
            # rows past the ones about to be written stay zero: attention bounded by query positions (the decode
            # graph) reads whole key tiles, and a masked key's weight 0 times a NaN left in V would still be NaN
            nkb[:, n + m:].zero_()
            nvb[:, n + m:].zero_()
            c["kbuf"], c["vbuf"] = nkb, nvb
        return n

    def _commit_kv(self, c, n_new):
        c["n"] = n_new
        if self.kv_pool is not None:          # paged: no single K/V tensor of the layer
            c["k"] = c["v"] = None
            return
        c["k"], c["v"] = c["kbuf"][:, :n_new], c["vbuf"][:, :n_new]

    def _attend(self, i, q, c, nk, out, **kw):
        """tcgen05 attention over cache entry c of layer i (contiguous buffers, or the pool's pages)."""
        if self.kv_pool is not None:
            pool = self.kv_pool
            return K.attention(q, pool.k[i], pool.v[i], nk, self.scale, out, pages=c["pages_dev"], **kw)
        return K.attention(q, c["kbuf"], c["vbuf"], nk, self.scale, out, **kw)

    def _qk_mode(self):
        if not self.cfg.qk_norm:
            return -1
        return 1 if self.zero_centred else 0

    def _write_kv(self, i, kv_src, pos, c):
        """K (head norm + RoPE) and V rows of kv_src [m, 2 * hkv * hd] into cache c at its end."""
        w = self.W[i]
        m = kv_src.shape[0]
        hd, hkv = self.head_dim, self.n_kv
        p0, parr = self._span(pos)
        n0 = self._kv_reserve(c, m, i)
        tables = self.rope(p0 + m if parr is None else int(pos.max()) + 1)
        if self.kv_pool is not None:
            pool = self.kv_pool
            paged = dict(pages=c["pages_dev"], page_size=pool.page_size, page_stride=pool.page_stride, row0=n0)
            K.head_norm_rope(kv_src, hkv, hd, hd, pool.k[i], pool.page_size * hd, hd, norm_w=w.get("k_norm"),
                             norm_mode=self._qk_mode(), eps=self.eps, tables=tables, rot=self.cfg.rot_dim,
                             pos=parr, pos_offset=p0, **paged)
            K.head_norm_rope(kv_src[:, hkv * hd:], hkv, hd, hd, pool.v[i], pool.page_size * hd, hd, **paged)
            self._commit_kv(c, n0 + m)
            return n0
        kb, vb = c["kbuf"], c["vbuf"]
        cap = kb.shape[1]
        K.head_norm_rope(kv_src, hkv, hd, hd, kb[:, n0:], cap * hd, hd, norm_w=w.get("k_norm"),
                         norm_mode=self._qk_mode(), eps=self.eps, tables=tables, rot=self.cfg.rot_dim,
                         pos=parr, pos_offset=p0)
        K.head_norm_rope(kv_src[:, hkv * hd:], hkv, hd, hd, vb[:, n0:], cap * hd, hd)
        self._commit_kv(c, n0 + m)
        return n0

    def _attn_mix(self, i, h, pos, cache):
        """Attention block output added to h (new tensor) and the mixer output when asked."""
        w = self.W[i]
        x = self._norm(h, w["ln1"])
        qkv = G.linear(x, w["qkv_p"])
        o = torch.empty(h.shape[0], self.n_heads * self.head_dim, dtype=self.dtype, device=self.device)
        return self._attn_core(i, qkv, pos, cache[i], o)

    def _attn_core(self, i, qkv, pos, c, o):
        """From the projected rows qkv [n, q(+gate) | k | v] of one sequence: K/V appended to its cache c, q head
        norm + RoPE, causal attention over the cache into o [n, hq * hd] (times the gate when the model has one)."""
        w = self.W[i]
        n = qkv.shape[0]
        hd, hq = self.head_dim, self.n_heads
        gated = self.cfg.gated_attn
        qw = hq * hd * (2 if gated else 1)
        p0, parr = self._span(pos)
        if n == 1 and parr is None and c.get("n", 0) == p0 and self._attn_decode_ok():
            # a decode row (its cache row is its position): the batched decode kernel, as decode_batch's rows
            self._kv_reserve(c, 1, i)
            self.rope(p0 + 1)
            self._attn_decode(i, qkv, torch.tensor([p0], dtype=torch.int32, device=self.device), [c], o)
            self._commit_kv(c, p0 + 1)
            return o
        n0 = self._write_kv(i, qkv[:, qw:], pos, c)
        q = torch.empty(hq, n, hd, dtype=self.dtype, device=self.device)
        tables = self.rope(p0 + n if parr is None else int(pos.max()) + 1)
        K.head_norm_rope(qkv, hq, hd, 2 * hd if gated else hd, q, n * hd, hd, norm_w=w.get("q_norm"),
                         norm_mode=self._qk_mode(), eps=self.eps, tables=tables, rot=self.cfg.rot_dim, pos=parr,
                         pos_offset=p0)
        self._attend(i, q, c, n0 + n, o, q_start=n0, gate=qkv[:, hd:] if gated else None, gate_head=2 * hd)
        return o

    def decode_batch(self, toks, positions, caches):
        """R sequences advanced by one token each in one pass over the weights: the embedding, every projection,
        MLP (or MoE) and the logits run on the R stacked rows, and the per-sequence parts run for all sequences in
        two launches per layer: K/V append and attention over each sequence's cache (csrc/attention_decode.cu), the
        GDN conv and recurrent step on each sequence's state (csrc/gdn_decode.cu); shapes those kernels do not take
        run per sequence. Products of 1-16 rows take the tensor-core GEMV (csrc/gemv.cu) and larger ones the tile
        GEMMs; every kernel computes a row the same way whatever the batch, so each row equals the single-sequence
        step bitwise. The CUDA-core GEMV (set_gemv_mma(False), 1-2 rows) sums in another order than the tile GEMMs,
        so with it a single step differs from a batched row by bf16 rounding."""
        if self.tp is not None or len(toks) == 1:
            return super().decode_batch(toks, positions, caches)
        R = len(toks)
        h = self.embed(torch.tensor([int(t) for t in toks], device=self.device))
        pos = [torch.tensor([int(p)], device=self.device) for p in positions]
        pos32 = torch.tensor([int(p) for p in positions], dtype=torch.int32, device=self.device)
        for i in range(self.n_layers):
            w = self.W[i]
            x = self._norm(h, w["ln1"])
            if self.layer_types[i] == "attn":
                qkv = G.linear(x, w["qkv_p"])
                y = torch.empty(R, self.n_heads * self.head_dim, dtype=self.dtype, device=self.device)
                entries = [caches[r][i] for r in range(R)]
                if self._attn_decode_ok() and all(c.get("n", 0) == int(p) for c, p in zip(entries, positions)):
                    for c in entries:
                        self._kv_reserve(c, 1, i)
                    self.rope(max(int(p) for p in positions) + 1)
                    self._attn_decode(i, qkv, pos32, entries, y)
                    for c, p in zip(entries, positions):
                        self._commit_kv(c, int(p) + 1)
                else:
                    for r in range(R):
                        self._attn_core(i, qkv[r:r + 1], pos[r], caches[r][i], y[r:r + 1])
                wo = w["o"]
            else:
                proj = G.linear(x, w["in_p"])
                entries = [caches[r][i] for r in range(R)]
                if self._gdn_decode_ok(entries):
                    o = self._gdn_decode(i, proj, entries, in_place=False)
                    for c in entries:
                        c["len"] = c.get("len", 0) + 1
                else:
                    o = torch.cat([self._gdn_core_dev(i, proj[r:r + 1], caches[r], True) for r in range(R)])
                z = proj[:, self.conv_dim + 2 * self.nv:]
                y = K.gated_rmsnorm(o, z, w["norm"], self.nv, self.cfg.gdn_dv, self.eps)
                wo = w["out"]
            h = self.mlp(i, G.linear(y, wo, residual=h))
        return self.logits(h)

    # ---- decode on device-resident positions (one CUDA graph serves every step: engine/decode_graph.py)
    def decode_step_dev(self, tok_dev, pos_dev, caches):
        """Next-token logits [R, V] fp32 of R sequences advanced by one token each, with the tokens (int64 [R]) and
        their positions (int32 [R]: each sequence's length before the token) in device memory. K/V rows are written
        at the positions read on the device, attention bounds its keys by them (query positions), and the GDN conv
        and recurrent states are updated in place, so nothing reads a position on the host and a CUDA graph of this
        call replays for every step. The attention caches must already have room for the positions and the RoPE
        tables must reach past them; the host keeps the lengths (engine/decode_graph.py). Same kernels and
        arithmetic as decode_batch."""
        if self.tp is not None or getattr(self.cfg, "moe", False):
            raise NotImplementedError("device-position decode runs dense single-GPU models")
        R = tok_dev.shape[0]
        h = self.embed(tok_dev)
        for i in range(self.n_layers):
            w = self.W[i]
            x = self._norm(h, w["ln1"])
            if self.layer_types[i] == "attn":
                qkv = G.linear(x, w["qkv_p"])
                y = torch.empty(R, self.n_heads * self.head_dim, dtype=self.dtype, device=self.device)
                if self._attn_decode_ok():
                    self._attn_decode(i, qkv, pos_dev, [caches[r][i] for r in range(R)], y)
                else:
                    for r in range(R):
                        self._attn_step_dev(i, qkv[r:r + 1], pos_dev[r:r + 1], caches[r][i], y[r:r + 1])
                wo = w["o"]
            else:
                proj = G.linear(x, w["in_p"])
                entries = [caches[r][i] for r in range(R)]
                if self._gdn_decode_ok(entries):
                    o = self._gdn_decode(i, proj, entries, in_place=True)
                else:
                    o = torch.cat([self._gdn_step_dev(i, proj[r:r + 1], caches[r]) for r in range(R)])
                z = proj[:, self.conv_dim + 2 * self.nv:]
                y = K.gated_rmsnorm(o, z, w["norm"], self.nv, self.cfg.gdn_dv, self.eps)
                wo = w["out"]
            h = self.mlp(i, G.linear(y, wo, residual=h))
        return self.logits(h)

    def _attn_decode_ok(self):
        """Whether the batched decode attention (csrc/attention_decode.cu) serves this model's attention layers."""
        return self.tp is None and K.decode_attention_supported(self.head_dim, self.n_heads, self.n_kv,
                                                                self.cfg.rot_dim)

    def _attn_decode(self, i, qkv, pos_dev, entries, out):
        """One decode row per sequence of attention layer i in two launches for all of them: qkv [R, *] the
        projected rows, pos_dev int32 [R] the positions (a sequence's new K/V row is cache row pos), entries the
        sequences' cache entries of layer i with room for that row; the RoPE tables must reach past every
        position. Writes out [R, hq * hd]."""
        w = self.W[i]
        hd, R = self.head_dim, len(entries)
        if self.kv_pool is not None:
            pool = self.kv_pool
            k, v = [pool.k[i]] * R, [pool.v[i]] * R
            pages = [c["pages_dev"] for c in entries]
            rows = [len(c["pages"]) * pool.page_size for c in entries]
            strides, ps, pstride = [pool.page_size * hd] * R, pool.page_size, pool.page_stride
        else:
            k, v = [c["kbuf"] for c in entries], [c["vbuf"] for c in entries]
            pages, rows = [], [c["kbuf"].shape[1] for c in entries]
            strides, ps, pstride = [n * hd for n in rows], 0, 0
        K.decode_attention(qkv, pos_dev, k, v, pages, rows, strides, ps, pstride, self.n_heads, self.n_kv, hd,
                           self.cfg.gated_attn, w.get("q_norm"), w.get("k_norm"), self._qk_mode(), self.eps,
                           self._rope_tables, self.cfg.rot_dim, self.scale, out)
        return out

    def _attn_step_dev(self, i, qkv, p_dev, c, o):
        """One decode row of attention layer i: K/V written at cache row p_dev[0], the query at that position over
        keys 0 .. p_dev[0] (both read on the device)."""
        w = self.W[i]
        hd, hq, hkv = self.head_dim, self.n_heads, self.n_kv
        gated = self.cfg.gated_attn
        qw = hq * hd * (2 if gated else 1)
        tables = self._rope_tables
        if self.kv_pool is not None:
            pool = self.kv_pool
            kd, vd = pool.k[i], pool.v[i]
            rows, stride = len(c["pages"]) * pool.page_size, pool.page_size * hd
            paged = dict(pages=c["pages_dev"], page_size=pool.page_size, page_stride=pool.page_stride)
        else:
            kd, vd = c["kbuf"], c["vbuf"]
            rows, stride, paged = kd.shape[1], kd.shape[1] * hd, {}
        K.head_norm_rope(qkv[:, qw:], hkv, hd, hd, kd, stride, hd, norm_w=w.get("k_norm"), norm_mode=self._qk_mode(),
                         eps=self.eps, tables=tables, rot=self.cfg.rot_dim, pos=p_dev, row_from_pos=True,
                         dst_rows=rows, **paged)
        K.head_norm_rope(qkv[:, qw + hkv * hd:], hkv, hd, hd, vd, stride, hd, pos=p_dev, row_from_pos=True,
                         dst_rows=rows, **paged)
        q = torch.empty(hq, 1, hd, dtype=self.dtype, device=self.device)
        K.head_norm_rope(qkv, hq, hd, 2 * hd if gated else hd, q, hd, hd, norm_w=w.get("q_norm"),
                         norm_mode=self._qk_mode(), eps=self.eps, tables=tables, rot=self.cfg.rot_dim, pos=p_dev)
        K.attention(q, kd, vd, rows, self.scale, o, qpos=p_dev, gate=qkv[:, hd:] if gated else None,
                    gate_head=2 * hd, pages=c["pages_dev"] if self.kv_pool is not None else None)

    def _gdn_decode_ok(self, entries):
        """Whether the batched decode step (csrc/gdn_decode.cu) serves these cache entries of one GDN layer: one GPU
        (tensor-parallel ranks keep the per-sequence path), head dims 128, fp32 recurrent states and conv windows
        already there (a prefill made them)."""
        cfg = self.cfg
        if self.tp is not None:
            return False
        if not K.gdn_decode_supported(cfg.gdn_dk, cfg.gdn_dv, cfg.conv_k) or self.nv % self.nk:
            return False
        if self.conv_dim != 2 * self.nk * cfg.gdn_dk + self.nv * cfg.gdn_dv:
            return False
        for c in entries:
            conv, rec = c.get("conv"), c.get("rec")
            if conv is None or rec is None or rec.dtype != torch.float32 or not rec.is_contiguous() \
                    or not conv.is_contiguous():
                return False
        return True

    def _gdn_decode(self, i, proj, entries, in_place):
        """One decode row per sequence of GDN layer i in two launches for all of them (csrc/gdn_decode.cu): proj
        [R, *] the in-projection rows, entries the R sequences' cache entries of layer i. in_place: the states are
        updated where they are (the graphed step owns them); otherwise new state tensors replace the entries' ones
        (the old ones may be shared with a forked cache). Returns the delta rule's outputs [R, nv * dv]."""
        w = self.W[i]
        cfg = self.cfg
        out = torch.empty(proj.shape[0], self.vd, dtype=self.dtype, device=self.device)
        conv_src = [c["conv"] for c in entries]
        rec_src = [c["rec"] for c in entries]
        if in_place:
            conv_dst, rec_dst = conv_src, rec_src
        else:
            conv_dst = [torch.empty_like(t) for t in conv_src]
            rec_dst = [torch.empty_like(t) for t in rec_src]
        K.gdn_decode_step(proj, w["conv"], w["A_log"], w["dt_bias"], conv_src, conv_dst, rec_src, rec_dst, out,
                          self.nk, self.nv, cfg.gdn_dk, cfg.gdn_dv, self.conv_dim, self.conv_dim + self.nv)
        for c, cd, rd in zip(entries, conv_dst, rec_dst):
            c["conv"], c["rec"] = cd, rd
        return out

    def _gdn_step_dev(self, i, proj, cache):
        """One decode row of GDN layer i, its conv and recurrent states updated in place."""
        w = self.W[i]
        cfg = self.cfg
        C, nv = self.conv_dim, self.nv
        c = cache[i]
        conv_state, rec = c["conv"], c["rec"]
        q, k, v, beta, g = K.gdn_prep(proj, C, C + nv, w["conv"], conv_state, w["A_log"], w["dt_bias"], self.nk, nv,
                                      cfg.gdn_dk, cfg.gdn_dv)
        K.gdn_conv_state_update(proj, conv_state, C)
        out = torch.empty(1, self.vd, dtype=self.dtype, device=self.device)
        K.gdn_scan(q, k, v, beta, g, rec, out, groups=1)
        return out

    # ---- per-layer API
    def _mixer_out(self, i, h, pos, cache, need_out=True, checkpoint_every=None):
        if self.layer_types[i] == "attn":
            return self._attn_mix(i, h, pos, cache), self.W[i]["o"]
        return self._gdn_mix(i, h, cache, checkpoint_every), self.W[i]["out"]

    def layer(self, i, h, pos, cache, mix=None, gdn_checkpoint_every=None, **_):
        y, wo = self._mixer_out(i, h, pos, cache, checkpoint_every=gdn_checkpoint_every)
        if self.tp is not None:
            h2 = self.tp.row_parallel(y, wo, h)
            if mix is not None:
                mix(i, h2 - h)
        elif mix is not None:
            a = G.linear(y, wo)
            mix(i, a)
            h2 = h + a
        else:
            h2 = G.linear(y, wo, residual=h)
        return self.mlp(i, h2)

    def layer_rows(self, i, h, pos, rows, cache):
        """Exact rows on the kernels: cache[i] is written from every row's input h (the filled prefix with the exact
        rows' true inputs in place) and the exact layer output of rows h[rows] is returned, as the torch models'
        layer_rows (models/llama.py, models/hybrid.py; the bypass of code/kva/kva.py:392-459).
        Attention: K/V of every row, queries of the selected rows only, tcgen05 attention at their positions. GDN:
        the delta rule runs over every row (a row's output needs the state at its own position); the output norm,
        out_proj and the MLP run on the selected rows."""
        w = self.W[i]
        x = self._norm(h, w["ln1"])
        hr = h[rows]
        if self.layer_types[i] == "attn":
            hd, hq = self.head_dim, self.n_heads
            gated = self.cfg.gated_attn
            qw = hq * hd * (2 if gated else 1)
            c = cache[i]
            self._write_kv(i, G.linear(x, w["qkv_p"][qw:]), pos, c)
            p0, parr = self._span(pos)
            tables = self.rope(p0 + pos.numel() if parr is None else int(pos.max()) + 1)
            rpos = pos[rows].to(torch.int32).contiguous()
            qg = G.linear(x[rows], w["qkv_p"][:qw])
            nr = qg.shape[0]
            q = torch.empty(hq, nr, hd, dtype=self.dtype, device=self.device)
            K.head_norm_rope(qg, hq, hd, 2 * hd if gated else hd, q, nr * hd, hd, norm_w=w.get("q_norm"),
                             norm_mode=self._qk_mode(), eps=self.eps, tables=tables, rot=self.cfg.rot_dim, pos=rpos)
            y = torch.empty(nr, hq * hd, dtype=self.dtype, device=self.device)
            self._attend(i, q, c, c["n"], y, qpos=rpos, gate=qg[:, hd:] if gated else None, gate_head=2 * hd)
            wo = w["o"]
        else:
            proj = G.linear(x, w["in_p"])
            out = self._gdn_core_dev(i, proj, cache, True)
            z = proj[:, self.conv_dim + 2 * self.nv:]
            y = K.gated_rmsnorm(out[rows], z[rows], w["norm"], self.nv, self.cfg.gdn_dv, self.eps)
            wo = w["out"]
        h2 = self.tp.row_parallel(y, wo, hr) if self.tp is not None else G.linear(y, wo, residual=hr)
        return self.mlp(i, h2)

    def project_map(self, projector, i, src):
        """x_i = src W_i^T + c_i on the tcgen05 GEMM (bias epilogue); column-sharded under tensor parallelism."""
        w, c = projector.device_map(i, self.device)
        w = w if w.dtype == self.dtype else w.to(self.dtype)
        c = c if c.dtype == self.dtype else c.to(self.dtype)
        x = self.tp.map_fill(src, w, c) if self.tp is not None else G.linear(src, w, bias=c)
        projector.done_with(i)
        return x

    def fill(self, i, x, pos, cache, st=None, checkpoint_every=None, **_):
        w = self.W[i]
        xn = self._norm(x, w["ln1"])
        if self.layer_types[i] == "attn":
            qw = self.n_heads * self.head_dim * (2 if self.cfg.gated_attn else 1)
            kv = G.linear(xn, w["qkv_p"][qw:])
            self._write_kv(i, kv, pos, cache[i])
            return {}
        ck = self._gdn_fill(i, xn, cache, checkpoint_every)
        if st is not None:
            cache[i]["rec"] = cache[i]["rec"] + st.to(cache[i]["rec"])
        return ck

    def fill_batch(self, layers, b, pos, cache, projector=None):
        """Cache-only fills of every late layer from the same boundary rows b: x_i = b W_i^T + c_i (tcgen05
        GEMM with the bias epilogue; identity fill when projector is None), then the layer's fill."""
        for i in layers:
            if projector is None:
                x = b
            else:
                w, c = projector.device_map(i, self.device)
                w = w if w.dtype == self.dtype else w.to(self.dtype)
                c = c if c.dtype == self.dtype else c.to(self.dtype)
                if getattr(self.tp, "row_fill", None) is not None:
                    self.tp.row_fill.fill_layer(self, i, b, pos, cache, w, c)
                    projector.done_with(i)
                    continue
                x = self.tp.map_fill(b, w, c) if self.tp is not None else G.linear(b, w, bias=c)
                projector.done_with(i)
            self.fill(i, x, pos, cache)


class B200Llama(_B200, Llama):
    """Llama-3.1 / dense Qwen3 on the sm_100a kernels."""

    zero_centred = False

    def _setup(self):
        super()._setup()
        self._kernel_setup()

    def _load_layer(self, i):
        w = super()._load_layer(i)
        qkv = torch.cat((w["q"], w["k"], w["v"])).contiguous()
        qw, kw = w["q"].shape[0], w["k"].shape[0]
        w.update(qkv_p=qkv, q=qkv[:qw], k=qkv[qw:qw + kw], v=qkv[qw + kw:])
        self._pack_mlp(w)
        return w

    def _gdn_mix(self, i, h, cache):
        raise RuntimeError("Llama-family models have no Gated DeltaNet layers")


class B200Hybrid(_B200, Hybrid):
    """The Qwen3.5-style hybrid (and its MoE variant) on the sm_100a kernels."""

    zero_centred = True

    def _setup(self):
        super()._setup()
        self._kernel_setup()
        c = self.cfg
        self.conv_dim = c.gdn_conv_dim
        self.vd = c.gdn_nv * c.gdn_dv

    def _load_layer(self, i):
        w = super()._load_layer(i)
        if self.layer_types[i] == "attn":
            qkv = torch.cat((w["q"], w["k"], w["v"])).contiguous()
            qw, kw = w["q"].shape[0], w["k"].shape[0]
            w.update(qkv_p=qkv, q=qkv[:qw], k=qkv[qw:qw + kw], v=qkv[qw + kw:])
        else:
            C, nv = self.cfg.gdn_conv_dim, self.cfg.gdn_nv
            p = torch.cat((w["qkv"], w["b"], w["a"], w["z"])).contiguous()
            w.update(in_p=p, qkv=p[:C], b=p[C:C + nv], a=p[C + nv:C + 2 * nv], z=p[C + 2 * nv:],
                     conv=w["conv"].contiguous(), A_log=w["A_log"].float().contiguous(),
                     dt_bias=w["dt_bias"].float().contiguous())
        if self.cfg.moe:
            self._pack_moe(w)
        else:
            self._pack_mlp(w)
        return w

    def _pack_moe(self, w):
        """Router rows extended by the shared-expert gate (padded to a multiple of 8 rows), each expert's gate/up
        interleaved per 128-row block for the grouped SwiGLU GEMM, the shared expert packed like a dense MLP."""
        E, d = self.cfg.n_experts, self.hidden
        pad = (-(E + 1)) % 8
        w["router_ext"] = torch.cat((w["router"], w["sh_gate_w"],
                                     torch.zeros(pad, d, dtype=self.dtype, device=self.device))).contiguous()
        F = self.cfg.moe_intermediate
        gu = w["experts_gu"]
        w["experts_gu_p"] = torch.stack([G.pack_gate_up(gu[e, :F], gu[e, F:]) for e in range(E)]).contiguous()
        w["experts_down"] = w["experts_down"].contiguous()
        del w["experts_gu"]
        w["sh_gu_p"] = G.pack_gate_up(w["sh_gate"], w["sh_up"]).contiguous()

    def _gdn_core_dev(self, i, proj, cache, need_out):
        """Conv + gates + chunked delta rule over the rows of proj, continuing cache[i]'s states. A single row with
        output (a decode step) takes the batched decode kernel, the same arithmetic as decode_batch's rows."""
        w = self.W[i]
        cfg = self.cfg
        C, nv = self.conv_dim, self.nv
        c = cache[i]
        if proj.shape[0] == 1 and need_out and self._gdn_decode_ok([c]):
            out = self._gdn_decode(i, proj, [c], in_place=False)
            c["len"] = c.get("len", 0) + 1
            return out
        conv_state = c.get("conv")
        q, k, v, beta, g = K.gdn_prep(proj, C, C + nv, w["conv"], conv_state, w["A_log"], w["dt_bias"],
                                      self.nk, nv, cfg.gdn_dk, cfg.gdn_dv, need_q=need_out)
        new_conv = (conv_state.clone() if conv_state is not None
                    else torch.zeros(cfg.conv_k - 1, C, dtype=self.dtype, device=self.device))
        K.gdn_conv_state_update(proj, new_conv, C)
        rec = c.get("rec")
        rec = (rec.float().clone() if rec is not None
               else torch.zeros(nv, cfg.gdn_dk, cfg.gdn_dv, dtype=torch.float32, device=self.device))
        out = None
        if need_out:
            out = torch.empty(proj.shape[0], self.vd, dtype=self.dtype, device=self.device)
        K.gdn_scan(q if need_out else None, k, v, beta, g, rec, out)
        c["conv"], c["rec"] = new_conv, rec
        c["len"] = c.get("len", 0) + proj.shape[0]
        return out

    def _gdn_core_ckpt(self, i, proj, cache, need_out, every):
        """_gdn_core_dev in pieces of `every` rows (within GDN_ROWS segments, the oracle's grouping), keeping the
        fp32 recurrent state after every full piece: ({absolute position: state [nv, dk, dv]}, outputs or None).
        The states are the ones the oracle's delta_rule(checkpoint_every=...) returns (ops/oracle.py)."""
        from .base import GDN_ROWS
        if every % 64:
            raise ValueError(f"checkpoint_every={every} must be a multiple of the chunk (64)")
        n = proj.shape[0]
        offset = cache[i].get("len", 0)
        outs, cks = [], {}
        for lo in range(0, n, GDN_ROWS):
            hi = min(n, lo + GDN_ROWS)
            for s in range(lo, hi, every):
                e = min(hi, s + every)
                o = self._gdn_core_dev(i, proj[s:e], cache, need_out)
                if need_out:
                    outs.append(o)
                if e - s == every:
                    cks[offset + e] = cache[i]["rec"].clone()
        return cks, (torch.cat(outs) if need_out else None)

    def _gdn_mix(self, i, h, cache, checkpoint_every=None):
        w = self.W[i]
        x = self._norm(h, w["ln1"])
        proj = G.linear(x, w["in_p"])
        if checkpoint_every:
            ck, o = self._gdn_core_ckpt(i, proj, cache, True, checkpoint_every)
            if ck:
                cache[i].setdefault("checkpoints", {}).update(ck)
        else:
            o = self._gdn_core_dev(i, proj, cache, True)
        z = proj[:, self.conv_dim + 2 * self.nv:]
        return K.gated_rmsnorm(o, z, w["norm"], self.nv, self.cfg.gdn_dv, self.eps)

    def _gdn_fill(self, i, xn, cache, checkpoint_every=None):
        """State-only fill: the q projection is needed only for the last conv_k - 1 rows (the conv window the next
        rows continue from), so the in-projection GEMM skips the q rows of every other row."""
        w = self.W[i]
        C, nv = self.conv_dim, self.nv
        qd = self.nk * self.cfg.gdn_dk
        rows = xn.shape[0]
        proj = torch.empty(rows, C + 2 * nv, dtype=self.dtype, device=self.device)
        G.linear(xn, w["in_p"][qd:C + 2 * nv], out=proj[:, qd:])
        last = min(rows, self.cfg.conv_k - 1)
        if last:
            G.linear(xn[rows - last:], w["in_p"][:qd], out=proj[rows - last:, :qd])
        if checkpoint_every:
            return self._gdn_core_ckpt(i, proj, cache, False, checkpoint_every)[0]
        self._gdn_core_dev(i, proj, cache, False)
        return {}

    def mlp(self, i, h):
        if self.cfg.moe:
            return self._moe_mlp(i, h)
        return _B200.mlp(self, i, h)

    def _moe_mlp(self, i, h):
        """Routed experts on the expert-grouped tcgen05 GEMM plus the gated shared expert, combined with the
        residual in one pass (ops/moe.py)."""
        from ..ops import moe as MO
        w = self.W[i]
        E, k = self.cfg.n_experts, self.cfg.top_k
        x = K.rmsnorm(h, w["ln2"], self.eps, self.zero_centred)
        logits = G.linear_f32(x, w["router_ext"])
        if self.ep is not None:
            return self.ep.moe(self, w, h, x, logits)
        idx, wts = MO.router_topk(logits, E, k)
        xp, pos, seg, tiles = MO.align(idx, E, x)
        act = MO.grouped(xp, w["experts_gu_p"], seg, tiles, swiglu=True)
        y = MO.grouped(act, w["experts_down"], seg, tiles, swiglu=False)
        ys = G.linear(G.swiglu_linear(x, w["sh_gu_p"]), w["sh_down"])
        return MO.combine(h, y, pos, wts, ys, logits[:, E])
