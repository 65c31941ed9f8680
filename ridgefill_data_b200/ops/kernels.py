"""Tensor-level wrappers of the sm_100a kernels (csrc/norm.cu, attention.cu, gdn.cu).

Every wrapper requires CUDA bf16 tensors in the layouts documented per function and raises if the
extension is missing: there is no PyTorch fallback on the device path.
"""
from __future__ import annotations

import torch

from ._ext import ext

BF16 = torch.bfloat16


def rmsnorm(x, w, eps, zero_centred, out=None):
    """RMSNorm of rows x [n, d] (plain: HF order; zero-centred: (1 + w))."""
    if out is None:
        out = torch.empty(x.shape[0], x.shape[1], dtype=BF16, device=x.device)
    ext().rmsnorm(x, w, out, float(eps), bool(zero_centred))
    return out


def rope_tables(inv_freq, max_pos, device, dtype=BF16):
    """cos/sin [max_pos, rot/2]: angles pos * inv_freq in fp32, cast to the activation dtype (the same
    values the oracle's rope_cos_sin produces, stored once per half)."""
    pos = torch.arange(max_pos, device=device, dtype=torch.float32)
    ang = pos[:, None] * inv_freq.to(device=device, dtype=torch.float32)[None, :]
    return ang.cos().to(dtype).contiguous(), ang.sin().to(dtype).contiguous()


def head_norm_rope(src, n_heads, head_dim, head_stride, dst, dst_head_stride, dst_row_stride, norm_w=None,
                   norm_mode=-1, eps=1e-6, tables=None, rot=0, pos=None, pos_offset=0, pages=None, page_size=0,
                   page_stride=0, row0=0, row_from_pos=False, dst_rows=0):
    """Per (row, head) of src [n, *] (head h at column h * head_stride): optional head RMSNorm, RoPE on the
    first rot dims at positions pos (int32 [n]) or pos_offset + row; written to dst + h * dst_head_stride +
    row * dst_row_stride (element strides). With pages (int32 page ids): row t is cache row row0 + t, stored in
    page pages[(row0 + t) // page_size] of the pool dst (page_stride elements apart) at row (row0 + t) % page_size.
    row_from_pos: row t goes to cache row pos[t] instead (read on the device), rows >= dst_rows not written."""
    cos, sin = tables if tables is not None else (None, None)
    ext().head_norm_rope(src, src.stride(0), head_stride, n_heads, head_dim, src.shape[0], norm_w, norm_mode,
                         float(eps), cos, sin, rot, pos, pos_offset, dst, dst_head_stride, dst_row_stride,
                         pages, page_size, page_stride, row0, bool(row_from_pos), int(dst_rows))


def gated_rmsnorm(o, z, w, heads, dv, eps, out=None):
    """Gated DeltaNet output norm: o [n, heads * dv], z [n, heads * dv] (any row pitch)."""
    if out is None:
        out = torch.empty(o.shape[0], heads * dv, dtype=BF16, device=o.device)
    ext().gated_rmsnorm(o, z, z.stride(0), w, out, heads, dv, float(eps))
    return out


def embed(table, ids):
    out = torch.empty(ids.numel(), table.shape[1], dtype=BF16, device=table.device)
    ext().embed_gather(table, ids.to(table.device, torch.long).contiguous(), out)
    return out


ATTN_IMPL = {"auto": 0, "mma": 1, "tcgen05": 2}


def attention(q, k_cache, v_cache, nk, scale, out, q_start=0, qpos=None, gate=None, gate_head=0, impl="auto",
              pages=None):
    """Causal GQA attention. q [hq, nq, hd] (any head pitch, row pitch hd); k_cache/v_cache [hkv, cap, hd]
    (the first nk rows valid); queries at positions q_start + row (or qpos int32 [nq]); out [nq, hq * hd];
    gate: a [nq, *] view whose head h starts at column h * gate_head (o * sigmoid(gate)).
    pages (int32 page ids, tcgen05 kernel only): k_cache / v_cache are page pools [num_pages, hkv, page_size, hd]
    and key row j lives in page pages[j // page_size]."""
    hq, nq, hd = q.shape
    if pages is None:
        hkv = k_cache.shape[0]
        ext().flash_attention(q, q.stride(0), k_cache, v_cache, k_cache.stride(0), out, hq, hkv, hd, nq, nk, qpos,
                              q_start, float(scale), gate, gate.stride(0) if gate is not None else 0, gate_head,
                              ATTN_IMPL[impl], ext().error_word(q.device.index or 0))
        return out
    n_pages, hkv, page_size, _ = k_cache.shape
    ext().flash_attention(q, q.stride(0), k_cache, v_cache, page_size * hd, out, hq, hkv, hd, nq, nk, qpos, q_start,
                          float(scale), gate, gate.stride(0) if gate is not None else 0, gate_head, ATTN_IMPL[impl],
                          ext().error_word(q.device.index or 0), kv_pages=pages, page_size=page_size,
                          num_pages=n_pages)
    return out


def gdn_prep(proj, b_off, a_off, conv_w, conv_state, A_log, dt_bias, nk, nv, dk, dv, need_q=True):
    """Conv + SiLU + l2norm + gates for the rows of proj [n, *]: returns q, k [nk, n, dk], v [nv, n, dv]
    (bf16) and beta, g [nv, n] (fp32). need_q False (a state-only fill): q is None and its columns of proj are
    not read."""
    n = proj.shape[0]
    dev = proj.device
    q = torch.empty(nk, n, dk, dtype=BF16, device=dev) if need_q else None
    k = torch.empty(nk, n, dk, dtype=BF16, device=dev)
    v = torch.empty(nv, n, dv, dtype=BF16, device=dev)
    beta = torch.empty(nv, n, dtype=torch.float32, device=dev)
    g = torch.empty(nv, n, dtype=torch.float32, device=dev)
    ext().gdn_prep(proj, b_off, a_off, conv_w, conv_state, A_log, dt_bias, n, nk, nv, dk, dv, conv_w.shape[1],
                   q, k, v, beta, g)
    return q, k, v, beta, g


def gdn_conv_state_update(proj, state, channels):
    ext().gdn_conv_state_update(proj, state, proj.shape[0], channels, state.shape[0] + 1)


def gdn_decode_supported(dk, dv, conv_k):
    """Shapes the batched decode step (csrc/gdn_decode.cu) takes: head dims 128, 2-8 conv taps."""
    return dk == 128 and dv == 128 and 2 <= conv_k <= 8


def gdn_decode_step(proj, conv_w, A_log, dt_bias, conv_src, conv_dst, rec_src, rec_dst, out, nk, nv, dk, dv,
                    b_off, a_off):
    """One decode row of a GDN layer for R sequences in two launches (csrc/gdn_decode.cu): proj [R, *] in-projection
    rows ([q | k | v] conv channels, b at b_off, a at a_off), per-sequence conv states [K-1, C] bf16 and recurrent
    states [nv, dk, dv] fp32 read from *_src and written to *_dst (the same tensors for an update in place), out
    [R, nv * dv] bf16 (the delta rule's outputs before the gated norm)."""
    ext().gdn_decode_step(proj, conv_w, A_log, dt_bias, list(conv_src), list(conv_dst), list(rec_src), list(rec_dst),
                          out, int(b_off), int(a_off), int(nk), int(nv), int(dk), int(dv), int(conv_w.shape[1]))
    return out


DEC_SPLITS = 64   # key splits per (sequence, KV head) of the decode attention (kDecSplits)


def decode_attention_supported(hd, hq, hkv, rot):
    """Shapes the batched decode attention (csrc/attention_decode.cu) takes: head_dim 64 / 128 / 256, 1, 2, 4, 6 or 8
    query heads per KV head, rotary dims a multiple of 2 hd / 32."""
    if hd not in (64, 128, 256) or hkv <= 0 or hq % hkv or hq // hkv not in (1, 2, 4, 6, 8):
        return False
    return rot == 0 or (rot <= hd and rot % (2 * (hd // 32)) == 0)


def decode_attention(qkv, pos, k, v, pages, rows, head_stride, page_size, page_stride, hq, hkv, hd, gated, q_norm,
                     k_norm, norm_mode, eps, tables, rot, scale, out):
    """One decode row of an attention layer for R sequences in two launches (csrc/attention_decode.cu): qkv [R, *]
    projected rows (q heads, each [q | gate] when gated, then k and v heads), pos int32 [R] each sequence's position
    (its new K/V row goes to cache row pos), k / v per sequence its contiguous [hkv, rows, hd] buffers or the pool's
    tensors, pages [] (contiguous) or one int32 page table per sequence, rows / head_stride per sequence; out
    [R, hq * hd] bf16."""
    R = qkv.shape[0]
    dev = qkv.device
    G = hq // hkv
    part_o = torch.empty(R * hkv * DEC_SPLITS * G * hd, dtype=torch.float32, device=dev)
    part_ml = torch.empty(R * hkv * DEC_SPLITS * G * 2, dtype=torch.float32, device=dev)
    cos, sin = tables if (tables is not None and rot) else (None, None)
    ext().decode_attention(qkv, pos, list(k), list(v), list(pages), [int(x) for x in rows],
                           [int(x) for x in head_stride], int(page_size), int(page_stride), q_norm, k_norm,
                           int(norm_mode), float(eps), cos, sin, int(rot), float(scale), int(hq), int(hkv), int(hd),
                           bool(gated), out, part_o, part_ml, ext().error_word(dev.index or 0))
    return out


def scan_groups(nv, dv, n, sms=148):
    """Chunk groups of the two-level delta-rule scan: enough (value head, 64-row slice, group) CTAs to fill about two
    waves when the heads alone leave the GPU mostly idle (tensor parallelism shrinks the heads per GPU); 1 (the
    sequential scan) when the heads already fill it."""
    n_chunks = (n + 63) // 64
    per_group_ctas = nv * 2 * (dv // 64)
    groups = (2 * sms) // max(1, per_group_ctas)
    return groups if groups > 1 and n_chunks >= 2 * groups else 1


def gdn_scan(q, k, v, beta, g, state, out=None, groups=None):
    """Chunked gated delta rule continuing `state` [nv, dk, dv] fp32 (updated in place). q None: fill
    mode (state only). out [n, nv * dv] bf16 (output mode). groups: chunk groups of the two-level scan
    (None: scan_groups' choice; 1: sequential)."""
    nk, n, dk = k.shape
    nv, _, dv = v.shape
    n_pad = (n + 63) // 64 * 64
    w_buf = torch.empty(nv, n_pad, dk, dtype=BF16, device=k.device)
    u_buf = torch.empty(nv, n_pad, dv, dtype=BF16, device=k.device)
    # chunk-start states and V' in memory only for the split output path (the fused state pass writes O itself)
    split = q is not None and (not ext().gdn_fused_output() or out.data_ptr() % 16 != 0 or out.stride(0) % 8 != 0)
    s_buf = torch.empty(nv, n_pad // 64, dv, dk, dtype=BF16, device=k.device) if split else None
    vt_buf = torch.empty(nv, n_pad, dv, dtype=BF16, device=k.device) if split else None
    if groups is None:
        groups = scan_groups(nv, dv, n) if dv == dk else 1
    grp_buf = start_buf = None
    if groups > 1:
        grp_buf = torch.empty(2, nv, groups, dv, dk, dtype=torch.float32, device=k.device)
        start_buf = torch.empty(nv, groups, dv, dk, dtype=torch.float32, device=k.device) if q is not None else None
    err = ext().error_word(k.device.index or 0)
    ext().gdn_chunk_scan(q, k, v, beta, g, state, out, w_buf, u_buf, s_buf, vt_buf, n, nk, nv, dk, dv, err,
                         groups, grp_buf, start_buf)
    return out


def score_rows(logits, targets=None, ref=None):
    """Vocabulary reductions of fp32 logits rows [rows, V] on the device (csrc/score.cu): dict(lse fp64, argmax
    int32, logprob fp64 of `targets` (int64 [rows]) when given, and with `ref` (the reference arm's logits of
    the same rows) kl = KL(ref || logits) fp64 and ref_argmax)."""
    logits = logits.float().contiguous()
    rows = logits.shape[0]
    dev = logits.device
    f64 = dict(dtype=torch.float64, device=dev)
    i32 = dict(dtype=torch.int32, device=dev)
    out = dict(lse=torch.empty(rows, **f64), argmax=torch.empty(rows, **i32),
               logprob=torch.empty(rows, **f64), kl=torch.empty(rows, **f64), ref_argmax=torch.empty(rows, **i32))
    tg = None if targets is None else targets.to(dev, torch.int64).contiguous()
    rf = None if ref is None else ref.float().contiguous()
    ext().score_rows(logits, rf, tg, out["logprob"], out["lse"], out["argmax"], out["ref_argmax"], out["kl"])
    if targets is None:
        del out["logprob"]
    if ref is None:
        del out["kl"], out["ref_argmax"]
    return out


def row_cosine(a, b, eps=1e-8):
    """Cosine similarity of matching rows of a, b [..., d] (bf16) in fp32 on the device (csrc/reduce.cu)."""
    d = a.shape[-1]
    a2, b2 = a.reshape(-1, d), b.reshape(-1, d)
    if a2.dtype != BF16:
        a2, b2 = a2.to(BF16), b2.to(BF16)
    a2, b2 = a2.contiguous() if a2.stride(-1) != 1 else a2, b2.contiguous() if b2.stride(-1) != 1 else b2
    out = torch.empty(a2.shape[0], dtype=torch.float32, device=a.device)
    ext().row_cosine(a2, b2, out, float(eps))
    return out.view(a.shape[:-1])


def window_mass(q, k, qpos, scale, mass=None):
    """Attention mass [n] (fp64) that window queries q [hq, w, hd] at positions qpos [w] give every key of
    k [hkv, n, hd] (causal, summed over heads and window rows); added into `mass` when given."""
    hq, w, hd = q.shape
    n = k.shape[1]
    nblk = (n + 63) // 64
    dev = q.device
    f32 = dict(dtype=torch.float32, device=dev)
    if mass is None:
        mass = torch.zeros(n, dtype=torch.float64, device=dev)
    ext().window_mass(q, k, qpos.to(dev, torch.int32).contiguous(), float(scale), mass,
                      torch.empty(hq * w * nblk, **f32), torch.empty(hq * w * nblk, **f32),
                      torch.empty(hq * w, **f32), torch.empty(hq * w, **f32))
    return mass
