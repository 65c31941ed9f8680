"""CPU oracle: the numerical building blocks in plain PyTorch (fp32/fp64 capable), restating the
semantics of the reference's ops module (code/kva/ops.py) so the sm_100a kernels have an
independent ground truth.

Layouts: activations [tokens, features]; per-head tensors [heads, tokens, dim]; the Gated DeltaNet
recurrent state [value_heads, key_dim, value_dim] in fp32; the conv state the last kernel-1 pre-conv
rows [kernel-1, channels].

Norm rounding follows Hugging Face's order (code/kva/ops.py:14-37): normalise in fp32, cast to the
activation dtype, then scale; the zero-centred variant scales by (1 + w) in fp32 before the cast.
"""
import math

import torch
import torch.nn.functional as F

# --------------------------------------------------------------------------------------- norms


def _inv_rms(xf, eps):
    return torch.rsqrt(xf.square().mean(-1, keepdim=True) + eps)


def rms_norm(x, weight, eps):
    """Llama RMSNorm (code/kva/ops.py:14-18)."""
    xf = x.float()
    return weight * (xf * _inv_rms(xf, eps)).to(x.dtype)


def rms_norm_zc(x, weight, eps):
    """Zero-centred RMSNorm, (1 + w) applied in fp32 (code/kva/ops.py:21-25)."""
    xf = x.float()
    return (xf * _inv_rms(xf, eps) * (1.0 + weight.float())).to(x.dtype)


def rms_norm_gated(x, gate, weight, eps):
    """Gated DeltaNet output norm: per-head RMSNorm, scale, then times silu(gate) in fp32
    (code/kva/ops.py:28-33)."""
    xf = x.float()
    y = weight * (xf * _inv_rms(xf, eps)).to(x.dtype)
    return (y * F.silu(gate.float())).to(x.dtype)


def l2norm(x, eps=1e-6):
    return x * torch.rsqrt(x.square().sum(-1, keepdim=True) + eps)


# ---------------------------------------------------------------------------------------- RoPE


def inv_freq_default(theta, rot_dim):
    exps = torch.arange(0, rot_dim, 2, dtype=torch.float32) / rot_dim
    return 1.0 / (theta ** exps)


def inv_freq_llama3(theta, dim, factor, low_freq_factor, high_freq_factor, original_max):
    """Llama-3.1 frequency rescaling: long wavelengths divided by `factor`, short ones kept, the band
    between blended linearly in 1/wavelength (code/kva/ops.py:46-56)."""
    base = inv_freq_default(theta, dim)
    wavelen = 2 * math.pi / base
    lo_w = original_max / low_freq_factor
    hi_w = original_max / high_freq_factor
    scaled = torch.where(wavelen > lo_w, base / factor, base)
    t = (original_max / wavelen - low_freq_factor) / (high_freq_factor - low_freq_factor)
    blended = (1 - t) * scaled / factor + t * scaled
    in_band = (wavelen >= hi_w) & (wavelen <= lo_w)
    return torch.where(in_band, blended, scaled)


def rope_cos_sin(inv_freq, positions, dtype):
    """cos/sin [tokens, rot_dim]: angles in fp32, cast to the activation dtype."""
    ang = positions.float()[:, None] * inv_freq.to(positions.device)[None, :]
    ang = torch.cat((ang, ang), -1)
    return ang.cos().to(dtype), ang.sin().to(dtype)


def apply_rope(x, cos, sin):
    """Rotate-half RoPE on the first cos.shape[-1] dims of x [heads, tokens, head_dim]."""
    rot = cos.shape[-1]
    xr = x[..., :rot]
    half = rot // 2
    rotated = torch.cat((-xr[..., half:], xr[..., :half]), -1)
    out = xr * cos + rotated * sin
    if rot == x.shape[-1]:
        return out
    return torch.cat((out, x[..., rot:]), -1)


# ----------------------------------------------------------------------------------- attention

ATTN_BLOCK_SCORES = 1 << 26   # fp32 scores held per query block


def query_block(hq, nk):
    return max(16, ATTN_BLOCK_SCORES // (hq * nk))


def _attend_rows(q, k_t, v, scale, qpos):
    """q [Hq, m, d] at positions qpos [m] over keys k_t = K^T fp32 [Hkv, d, nk] (key j at position j).
    GQA without expanding K/V; scores/softmax fp32, probabilities cast to V's dtype."""
    hq, m, d = q.shape
    hkv, _, nk = k_t.shape
    rep = hq // hkv
    s = torch.matmul(q.reshape(hkv, rep * m, d).float(), k_t) * scale
    mask = torch.arange(nk, device=q.device)[None, :] > qpos[:, None]
    s.view(hkv, rep, m, nk).masked_fill_(mask, float("-inf"))
    p = torch.softmax(s, -1).to(v.dtype)
    return torch.matmul(p, v).view(hq, m, -1)


def attend_at(q, k, v, scale, qpos):
    """Causal attention of queries at sorted positions qpos over keys 0..nk-1 (query t sees keys
    j <= qpos[t]); query-blocked. Returns [nq, Hq * d] (code/kva/ops.py:128-152)."""
    hq, nq, _ = q.shape
    k_t = k.float().transpose(1, 2)
    rows = query_block(hq, k.shape[1])
    parts = []
    for a in range(0, nq, rows):
        b = min(nq, a + rows)
        end = int(qpos[b - 1]) + 1
        parts.append(_attend_rows(q[:, a:b], k_t[:, :, :end], v[:, :end], scale, qpos[a:b]))
    return torch.cat(parts, 1).transpose(0, 1).reshape(nq, -1)


def attend(q, k, v, scale):
    """The last nq positions of a sequence attending causally over all nk keys (bottom-right
    aligned). Returns [nq, Hq * d] (code/kva/ops.py:107-125)."""
    nq, nk = q.shape[1], k.shape[1]
    qpos = torch.arange(nk - nq, nk, device=q.device)
    return attend_at(q, k, v, scale, qpos)


# ------------------------------------------------------------------------------ Gated DeltaNet


def causal_conv(x, state, weight):
    """Depthwise causal conv (kernel K) + SiLU continuing from `state` [K-1, C] (None: zeros).
    x [n, C]; weight [C, K]. Returns (out [n, C] in x.dtype, new state [K-1, C])."""
    n, channels = x.shape
    width = weight.shape[1]
    history = x.new_zeros(width - 1, channels) if state is None else state.to(x.dtype)
    window = torch.cat([history, x], 0)                          # [width - 1 + n, C]
    taps = weight.float()
    acc = torch.zeros(n, channels, dtype=torch.float32, device=x.device)
    for j in range(width):                                       # oldest tap first (the accumulation order)
        acc += window[j:j + n].float() * taps[:, j]
    return F.silu(acc).to(x.dtype), window[window.shape[0] - (width - 1):].clone()


def unit_lower_inverse(a):
    """(I + A)^-1 for strictly lower-triangular A [..., C, C] by forward substitution."""
    c = a.shape[-1]
    t = torch.zeros_like(a)
    eye = torch.eye(c, dtype=a.dtype, device=a.device)
    # row i of T = e_i - sum_{j<i} A[i, j] T[j]
    for i in range(c):
        row = eye[i].expand_as(t[..., i, :]).clone()
        if i:
            row = row - (a[..., i, :i, None] * t[..., :i, :]).sum(-2)
        t[..., i, :] = row
    return t


def _initial_state(state, h, dk, dv, device):
    if state is None:
        return torch.zeros(h, dk, dv, dtype=torch.float32, device=device)
    return state.float().clone()


def delta_rule(q, k, v, g, beta, state=None, chunk=64, checkpoint_every=None, offset=0, need_out=True):
    """Chunked gated delta rule in fp32, continuing from `state`.

    q, k [H, n, dk] (l2-normed, q pre-scaled), v [H, n, dv], g (log decay) and beta [H, n].
    Per token: S <- e^g S;  S <- S + k (beta (v - S^T k))^T;  o = S^T q.
    Within a chunk of C tokens (cumulative log decay gamma): A = strictly-lower(beta_i k_i.k_j e^(gamma_i - gamma_j)),
    T = (I + A)^-1, u = T (beta v), w = T (beta e^gamma k); per chunk v' = u - w S,
    o = (q e^gamma) S + (q k^T * decay) v', S <- e^(gamma_C) S + (k e^(gamma_C - gamma))^T v'
    (code/kva/ops.py:199-262). checkpoint_every: also return {offset + t: S_t} at chunk ends t that are
    multiples of it. Returns (out [H, n, dv] fp32 or None, state [H, dk, dv], checkpoints)."""
    h, n, dk = k.shape
    dv = v.shape[-1]
    if checkpoint_every and checkpoint_every % chunk:
        raise ValueError(f"checkpoint_every={checkpoint_every} must be a multiple of the chunk ({chunk})")
    S = _initial_state(state, h, dk, dv, k.device)
    out = torch.empty(h, n, dv, dtype=torch.float32, device=k.device) if need_out else None
    cks = {}
    tri = torch.ones(chunk, chunk, dtype=torch.bool, device=k.device).tril()
    for c0 in range(0, n, chunk):
        c1 = min(n, c0 + chunk)
        m = c1 - c0

        def take(x):
            part = x[:, c0:c1].float()
            if m == chunk:
                return part
            return F.pad(part, (0, chunk - m) if part.dim() == 2 else (0, 0, 0, chunk - m))

        qc, kc, vc, gc, bc = (take(x) for x in (q, k, v, g, beta))
        gam = gc.cumsum(-1)
        rel = gam[:, :, None] - gam[:, None, :]
        decay = torch.where(tri, rel, torch.full_like(rel, -math.inf)).exp()
        a = (bc[:, :, None] * (kc @ kc.transpose(-1, -2)) * decay).tril(-1)
        t = unit_lower_inverse(a)
        u = t @ (bc[:, :, None] * vc)
        w = t @ (bc[:, :, None] * gam.exp()[:, :, None] * kc)
        vn = u - w @ S
        if need_out:
            o = (qc * gam.exp()[:, :, None]) @ S + ((qc @ kc.transpose(-1, -2)) * decay) @ vn
            out[:, c0:c1] = o[:, :m]
        last = gam[:, -1]
        kd = kc * (last[:, None] - gam).exp()[:, :, None]
        S = S * last.exp()[:, None, None] + kd.transpose(-1, -2) @ vn
        if checkpoint_every and c1 == c0 + chunk and c1 % checkpoint_every == 0:
            cks[offset + c1] = S.clone()
    return out, S, cks


def delta_rule_recurrent(q, k, v, g, beta, state=None):
    """Token-by-token gated delta rule (the definition; decode and tests)."""
    h, n, dk = k.shape
    dv = v.shape[-1]
    S = _initial_state(state, h, dk, dv, k.device)
    out = torch.empty(h, n, dv, dtype=torch.float32, device=k.device)
    for t in range(n):
        S = S * g[:, t].float().exp()[:, None, None]                     # decay
        key, val = k[:, t].float(), v[:, t].float()
        correction = (val - torch.einsum("hkv,hk->hv", S, key)) * beta[:, t].float()[:, None]
        S = S + key[:, :, None] * correction[:, None, :]                 # delta-rule write
        out[:, t] = torch.einsum("hkv,hk->hv", S, q[:, t].float())       # read
    return out, S


# ---------------------------------------------------------------------------------------- MoE


def router_topk(logits, k, norm_topk=True):
    """Softmax router with top-k selection (fp32): returns (weights [n, k], experts [n, k]).
    norm_topk renormalises the k selected probabilities to sum to one."""
    p = torch.softmax(logits.float(), -1)
    w, idx = torch.topk(p, k, dim=-1)
    if norm_topk:
        w = w / w.sum(-1, keepdim=True)
    return w, idx
