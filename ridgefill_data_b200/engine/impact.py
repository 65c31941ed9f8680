"""Fill impact: how much the scored loss would move if a prefix row's late-layer K/V were exact instead of
filled, to first order (code/kva/impact.py:1-18), plus the per-row lookup features used by the sensitivity
selectors and the weighted fit.

    impact_j = sum over late attention layers l of <dL/dK_l[j], K_l^true[j] - K_l^fill[j]>
                                                  + <dL/dV_l[j], V_l^true[j] - V_l^fill[j]>

L is the mean NLL of the scored targets, its gradient taken at the filled cache. K is the cached post-RoPE key
(RoPE is a rotation, so the inner product is the pre-RoPE one). GDN layers enter through their conv and
recurrent state at P, held constant: impact covers the attention K/V only.

The inference path writes caches in place and never keeps the fp32 probabilities, so this module carries its
own differentiable tail path for the late layers: attention as an autograd function whose backward recomputes
the probabilities one (KV head, query block) at a time, and a chunked delta rule built from out-of-place ops
(the unit lower inverse as a triangular solve); each layer is checkpointed.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..ops import oracle as ops


class CausalAttention(torch.autograd.Function):
    """ops.attend (bottom-right causal GQA; q [Hq, nq, d], k/v [Hkv, nk, d] -> [nq, Hq d]) with a backward that
    recomputes the softmax per KV head and query block, so only one block of scores is alive. The forward's
    bf16 cast of the probabilities counts as the identity in the backward."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        out = ops.attend(q, k, v, scale)
        ctx.save_for_backward(q, k, v, out)
        ctx.scale = scale
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out = ctx.saved_tensors
        scale = ctx.scale
        hq, nq, d = q.shape
        hkv, nk, dv = v.shape
        rep = hq // hkv
        g_o = grad_out.reshape(nq, hq, dv).transpose(0, 1).float()                 # [hq, nq, dv]
        o = out.reshape(nq, hq, dv).transpose(0, 1).float()
        delta = (g_o * o).sum(-1)                                                      # rowsum(dO * O)
        gq = torch.zeros(hq, nq, d, device=q.device)
        gk = torch.zeros(hkv, nk, d, device=q.device)
        gv = torch.zeros(hkv, nk, dv, device=q.device)
        block = ops.query_block(rep, nk)
        keys = torch.arange(nk, device=q.device)
        for h in range(hkv):
            heads = slice(h * rep, (h + 1) * rep)
            for a in range(0, nq, block):
                b = min(nq, a + block)
                end = nk - nq + b                                                      # keys the block can see
                qpos = torch.arange(nk - nq + a, nk - nq + b, device=q.device)
                kf, vf = k[h, :end].float(), v[h, :end].float()
                qf = q[heads, a:b].float()
                s = (qf @ kf.T) * scale
                s.masked_fill_(keys[None, :end] > qpos[:, None], -math.inf)
                p = torch.softmax(s, -1)
                dp = g_o[heads, a:b] @ vf.T
                ds = p * (dp - delta[heads, a:b, None])
                gq[heads, a:b] = (ds @ kf) * scale
                gk[h, :end] += (ds.transpose(1, 2) @ qf).sum(0) * scale
                gv[h, :end] += (p.transpose(1, 2) @ g_o[heads, a:b]).sum(0)
        return gq.to(q.dtype), gk.to(k.dtype), gv.to(v.dtype), None


def delta_rule_diff(q, k, v, g, beta, state, chunk=64):
    """The chunked gated delta rule of ops.delta_rule (same chunk grid and formulas) written with out-of-place
    ops only, so autograd runs through it. Returns out [H, n, dv] fp32."""
    h, n, dk = k.shape
    dv = v.shape[-1]
    pad = (-n) % chunk
    nc = (n + pad) // chunk

    def chunks(x):
        x = x.float()
        if pad:
            x = F.pad(x, (0, 0, 0, pad) if x.dim() == 3 else (0, pad))
        return x.reshape(h, nc, chunk, *x.shape[2:])

    qc, kc, vc, bc = chunks(q), chunks(k), chunks(v), chunks(beta)
    gam = chunks(g).cumsum(-1)                                                         # [h, nc, C]
    lower = torch.ones(chunk, chunk, dtype=torch.bool, device=k.device).tril()
    gap = gam[..., :, None] - gam[..., None, :]
    decay = torch.where(lower, gap, torch.full_like(gap, -math.inf)).exp()
    a = (bc[..., None] * (kc @ kc.transpose(-1, -2)) * decay).tril(-1)
    eye = torch.eye(chunk, device=k.device).expand_as(a)
    t = torch.linalg.solve_triangular(a + eye, eye, upper=False, unitriangular=True)
    u = t @ (bc[..., None] * vc)
    w = t @ (bc[..., None] * gam.exp()[..., None] * kc)
    intra = (qc @ kc.transpose(-1, -2)) * decay
    q_in = qc * gam.exp()[..., None]
    k_out = kc * (gam[..., -1:] - gam).exp()[..., None]
    s = state.float()
    outs = []
    for c in range(nc):
        vn = u[:, c] - w[:, c] @ s
        outs.append(q_in[:, c] @ s + intra[:, c] @ vn)
        s = s * gam[:, c, -1].exp()[:, None, None] + k_out[:, c].transpose(-1, -2) @ vn
    return torch.cat(outs, 1)[:, :n]


# ------------------------------------------------------------------------------------- late layers

def attn_kv(model, i, x, pos):
    """Post-RoPE K, V [Hkv, n, d] of attention layer i for normed rows x, as the cache holds them."""
    return model._attn_kv(i, x, pos) if hasattr(model, "_attn_kv") else model._kv(i, x, pos)


def _attn_queries(model, i, x, pos):
    if hasattr(model, "_attn_q"):
        return model._attn_q(i, x, pos)
    return model.queries(i, x, pos), None


def _late_attn(model, i, h, pos, k_pre, v_pre):
    """Attention layer i for rows h over [prefix K/V; the rows' own K/V] (= model.layer)."""
    w = model.W[i]
    x = model.in_norm(h, w["ln1"])
    q, gate = _attn_queries(model, i, x, pos)
    k, v = attn_kv(model, i, x, pos)
    o = CausalAttention.apply(q, torch.cat((k_pre, k), 1), torch.cat((v_pre, v), 1), model.scale)
    if gate is not None:
        o = o * torch.sigmoid(gate)
    return model.mlp(i, h + F.linear(o, w["o"]))


def _late_gdn(model, i, h, conv, rec):
    """GDN layer i for rows h continuing the conv / recurrent state (held constant) (= model.layer)."""
    w = model.W[i]
    x = model.in_norm(h, w["ln1"])
    pre, b, a = model._gdn_inputs(i, x)
    conv_out, _ = ops.causal_conv(pre, conv, w["conv"])
    q, k, v = model.gdn_qkv(conv_out)
    beta, g = model.gdn_gates(i, b, a)
    out = delta_rule_diff(q, k, v, g, beta, rec).to(pre.dtype)
    return model.mlp(i, h + model._gdn_out(i, out, x))


def tail_loss(model, split, h0, pos, kv, gdn, rows, targets, recompute=True):
    """Mean NLL (fp32) of `targets` at tail rows `rows`, running the tail rows (split-layer inputs h0 at
    positions pos) through layers >= split over the prefix caches kv {i: (K, V)} and gdn {i: {conv, rec}}.
    recompute: checkpoint each layer (recompute it in the backward)."""
    h = h0
    for i in range(split, model.n_layers):
        if model.layer_types[i] == "attn":
            fn, args = _late_attn, (model, i, h, pos, *(t.to(h.device) for t in kv[i]))
        else:
            fn, args = _late_gdn, (model, i, h, gdn[i]["conv"], gdn[i]["rec"])
        h = checkpoint(fn, *args, use_reentrant=False) if recompute and torch.is_grad_enabled() else fn(*args)
    return F.cross_entropy(model.logits(h[rows]), targets)


@torch.no_grad()
def exact_late(model, h_split, split, P, rows, targets, final=False, hook=None):
    """Exact late layers over all rows from the split-layer inputs. Returns ({attention layer: (K, V) of rows
    [0, P) on the CPU, post-RoPE}, exact loss over `rows`) and, when final, the last layer's output rows.
    hook(i, h) sees each late layer's input rows."""
    n = h_split.shape[0]
    pos = torch.arange(n, device=h_split.device)
    cache = model.new_cache()
    true = {}
    h = h_split
    for i in range(split, model.n_layers):
        if hook is not None:
            hook(i, h)
        h = model.layer(i, h, pos, cache)
        if model.layer_types[i] == "attn":
            true[i] = (cache[i]["k"][:, :P].cpu(), cache[i]["v"][:, :P].cpu())
        cache[i] = {}
    loss = float(F.cross_entropy(model.logits(h[rows]), targets))
    return (true, loss, h) if final else (true, loss)


@torch.no_grad()
def fill_late(model, split, P, fill_x):
    """Prefix fill of every late layer from inputs fill_x(i) [P, d], as the prefill's fill step does. Returns
    ({attention layer: (K, V)}, {GDN layer: {conv, rec}})."""
    dev = fill_x(split).device
    pos = torch.arange(P, device=dev)
    cache = model.new_cache()
    kv, gdn = {}, {}
    for i in range(split, model.n_layers):
        model.fill(i, fill_x(i), pos, cache)
        if model.layer_types[i] == "attn":
            kv[i] = (cache[i]["k"], cache[i]["v"])
        else:
            gdn[i] = dict(conv=cache[i]["conv"], rec=cache[i]["rec"])
        cache[i] = {}
    return kv, gdn


def impact(model, split, h_tail, P, kv, true_kv, gdn, rows, targets):
    """Backward through the tail at the filled cache. Per prefix row (fp64, CPU): the signed first-order impact,
    the relative fill error (mean over late attention layers of (|dK|/|K| + |dV|/|V|) / 2) and the gradient norm
    over all late attention K/V. Each leaf's gradient is folded into the per-row sums as soon as it has been
    accumulated, then dropped. Returns (dict of [P] tensors, loss at the fill)."""
    dev = h_tail.device
    pos = torch.arange(P, P + h_tail.shape[0], device=dev)
    sums = {name: torch.zeros(P, dtype=torch.float64, device=dev) for name in ("impact", "err", "grad2")}

    def fold(i, which):
        def hook(leaf):
            true = true_kv[i][which].to(dev).float()
            diff = true - leaf.detach().float()
            g = leaf.grad.float()
            sums["impact"] += (g * diff).sum((0, 2)).double()
            sums["grad2"] += g.square().sum((0, 2)).double()
            ref = true.square().sum((0, 2)).sqrt().clamp_min(1e-6)
            sums["err"] += 0.5 * (diff.square().sum((0, 2)).sqrt() / ref).double()
            leaf.grad = None
        return hook

    leaves = {}
    for i, (k, v) in kv.items():
        leaves[i] = (k.detach().requires_grad_(), v.detach().requires_grad_())
        for which, leaf in enumerate(leaves[i]):
            leaf.register_post_accumulate_grad_hook(fold(i, which))
    with torch.enable_grad():
        loss = tail_loss(model, split, h_tail, pos, leaves, gdn, rows, targets)
        loss.backward()
    sums["err"] /= max(1, len(kv))
    return dict(impact=sums["impact"].cpu(), err=sums["err"].cpu(), grad_norm=sums["grad2"].sqrt().cpu()), \
        float(loss.detach())


# ------------------------------------------------------------------------------ lookup statistics

def _blocks(q, k, scale, stride=1):
    """Yield (kv head, query positions, causal softmax probabilities [rep, m, b]) over query blocks."""
    hq, n, _ = q.shape
    hkv = k.shape[0]
    rep = hq // hkv
    block = ops.query_block(rep, n) * stride
    keys = torch.arange(n, device=q.device)
    for h in range(hkv):
        kf = k[h].float()
        for a in range(0, n, block):
            b = min(n, a + block)
            qpos = keys[a:b:stride]
            s = (q[h * rep:(h + 1) * rep, qpos].float() @ kf[:b].T) * scale
            s.masked_fill_(keys[None, :b] > qpos[:, None], -math.inf)
            yield qpos, b, torch.softmax(s, -1)


@torch.no_grad()
def received_mass(q, k, scale, rows_below=None, stride=1, entropy=False):
    """Attention mass each key row receives from strictly later query rows, summed over query heads (causal
    column sums, H2O style) (code/kva/impact.py:234-268). q [Hq, n, d] post-RoPE, k [Hkv, n, d]. rows_below:
    also the mass from query rows < rows_below only. stride s > 1: every s-th query row, scaled by s (unbiased
    in expectation at ~1/s the cost). entropy: also each query row's attention entropy in nats summed over
    heads (stride 1 only). Returns fp64 CPU [n] (then [n] for rows_below, then [n] for entropy)."""
    if entropy and stride != 1:
        raise ValueError("entropy needs every query row (stride 1)")
    n = q.shape[1]
    tot, low, ent = (torch.zeros(n, dtype=torch.float64, device=q.device) for _ in range(3))
    for qpos, b, p in _blocks(q, k, scale, stride):
        if entropy:
            ent[qpos] += torch.special.entr(p).sum((0, 2)).double()
        keys = torch.arange(b, device=q.device)
        p = p.masked_fill(keys[None, :] == qpos[:, None], 0.0)
        per_query = p.sum(0) * stride                                                  # [m, b]
        tot[:b] += per_query.sum(0).double()
        if rows_below is not None:
            low[:b] += per_query[qpos < rows_below].sum(0).double()
    out = (tot.cpu(),) + ((low.cpu(),) if rows_below is not None else ()) + ((ent.cpu(),) if entropy else ())
    return out if len(out) > 1 else out[0]


@torch.no_grad()
def row_stats(q, k, scale, local=64):
    """Each query row's own lookup, averaged over query heads: entropy (nats), mass on row 0 (the sink) and
    mass on the `local` most recent keys, itself included. Three fp64 CPU [n]."""
    hq, n, _ = q.shape
    ent, sink, near = (torch.zeros(n, dtype=torch.float64, device=q.device) for _ in range(3))
    for qpos, b, p in _blocks(q, k, scale):
        keys = torch.arange(b, device=q.device)
        ent[qpos] += torch.special.entr(p).sum(-1).sum(0).double()
        sink[qpos] += p[..., 0].sum(0).double()
        recent = (qpos[:, None] - keys[None, :] < local) & (keys[None, :] <= qpos[:, None])
        near[qpos] += (p * recent).sum(-1).sum(0).double()
    return (ent / hq).cpu(), (sink / hq).cpu(), (near / hq).cpu()


def leverage_map(stats_state, lam):
    """(mean, L) such that |(x - mean) L|^2 is the ridge hat value of a split state x under the projector's own
    calibration scatter (Cxx + lam s I, as EigenFit fits it): how far a row lies outside the fit's data.
    CPU fp64."""
    from ..ridge.fit import EigenFit
    fit = EigenFit(stats_state)
    return fit.mean_x, fit.evecs / (fit.evals + lam * fit.scale).sqrt()[None, :]


# ------------------------------------------------------------------- per-row features of [n, d] states
ROWS = 4096


def by_rows(fn, n, chunk=None):
    """torch.cat of fn(row slice) over row chunks (fp64 CPU): per-row features of [n, d] states with chunk x d
    temporaries only."""
    chunk = chunk or ROWS
    return torch.cat([fn(slice(a, min(n, a + chunk))).double().cpu() for a in range(0, n, chunk)])


def row_norm(x):
    return by_rows(lambda s: x[s].float().norm(dim=-1), x.shape[0])


def velocity(x, prev):
    """|x - prev| / |prev| per row: how far the last layers moved each row."""
    def f(s):
        p = prev[s].float()
        return (x[s].float() - p).norm(dim=-1) / p.norm(dim=-1).clamp_min(1e-6)
    return by_rows(f, x.shape[0])


def log_leverage(x, mean, L):
    mean, L = mean.to(x.device, torch.float32), L.to(x.device, torch.float32)
    return by_rows(lambda s: ((x[s].float() - mean) @ L).square().sum(-1), x.shape[0]).clamp_min(1e-30).log()


def log_max_act(x):
    """log max |x| over each row: massive-activation (sink-like) rows."""
    return by_rows(lambda s: x[s].float().abs().amax(-1), x.shape[0]).clamp_min(1e-30).log()


@torch.no_grad()
def gdn_gates(model, i, h):
    """Per row at GDN layer i: the write strength sigmoid(b) and the log decay, each a mean over value heads.
    Two fp64 CPU [n]."""
    w = model.W[i]

    def f(s):
        _, b, a = model._gdn_inputs(i, model.in_norm(h[s], w["ln1"]))
        beta, g = model.gdn_gates(i, b, a)
        return torch.stack((beta.mean(0), g.mean(0)), -1)
    out = by_rows(f, h.shape[0])
    return out[:, 0], out[:, 1]


def repetition(ids, cap):
    """Per token: log distance to the previous occurrence of the same id (cap for first occurrences), a
    first-occurrence flag, and whether the (previous, current) pair occurred before. Three fp64 lists."""
    last, pairs = {}, set()
    dist, first, bigram = [], [], []
    prev = None
    for j, t in enumerate(ids):
        seen = t in last
        dist.append(math.log(max(1, min(j - last[t] if seen else cap, cap))))
        first.append(0.0 if seen else 1.0)
        pair = (prev, t) if j else None
        bigram.append(1.0 if pair in pairs else 0.0)
        if pair is not None:
            pairs.add(pair)
        last[t] = j
        prev = t
    return dist, first, bigram
