"""Fill impact: to first order, how much the scored loss would move if one prefix row's late-layer K/V were exact
instead of filled (the measure of code/kva/impact.py:1-18), plus the per-row lookup features that the
sensitivity selectors and the weighted fit read.

    impact_j = sum over late attention layers l of  <dL/dK_l[j], K_l^true[j] - K_l^fill[j]>
                                                 + <dL/dV_l[j], V_l^true[j] - V_l^fill[j]>

L is the mean NLL of the scored targets, differentiated at the filled cache; K is the cached key after RoPE (a
rotation, so the inner product equals the one before RoPE). A GDN layer enters through its conv window and
recurrent state at P, held constant: the impact covers attention K/V only.

The inference path writes caches in place and keeps no fp32 probabilities, so the late layers get their own
differentiable path here: attention as an autograd function whose backward recomputes the probabilities per
(KV head, query block), and the chunked delta rule written with out-of-place operations (the chunk's unit lower
triangular system solved by a triangular solve). Each layer is checkpointed.
"""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F
from torch.utils.checkpoint import checkpoint

from ..ops import oracle as ops

NEG_INF = -math.inf


def _causal_mask_(scores, key_pos, q_pos):
    """Mask keys after each query (in place) and return the scores."""
    return scores.masked_fill_(key_pos[None, :] > q_pos[:, None], NEG_INF)


class CausalAttention(torch.autograd.Function):
    """ops.attend (bottom-right causal GQA: q [Hq, nq, d], k / v [Hkv, nk, d] -> [nq, Hq * d]) with a backward
    that rebuilds the softmax one (KV head, query block) at a time, so one block of scores is alive at once. The
    forward's bf16 rounding of the probabilities is treated as the identity in the backward."""

    @staticmethod
    def forward(ctx, q, k, v, scale):
        out = ops.attend(q, k, v, scale)
        ctx.scale = scale
        ctx.save_for_backward(q, k, v, out)
        return out

    @staticmethod
    def backward(ctx, grad_out):
        q, k, v, out = ctx.saved_tensors
        scale = ctx.scale
        n_q_heads, nq, d = q.shape
        n_kv_heads, nk, dv = v.shape
        group = n_q_heads // n_kv_heads
        dev = q.device
        dout = grad_out.reshape(nq, n_q_heads, dv).transpose(0, 1).float()          # [Hq, nq, dv]
        rowdot = (dout * out.reshape(nq, n_q_heads, dv).transpose(0, 1).float()).sum(-1)
        dq = torch.zeros(n_q_heads, nq, d, device=dev)
        dk = torch.zeros(n_kv_heads, nk, d, device=dev)
        dvv = torch.zeros(n_kv_heads, nk, dv, device=dev)
        step = ops.query_block(group, nk)
        key_pos = torch.arange(nk, device=dev)
        offset = nk - nq                                                                 # bottom-right alignment
        for kv in range(n_kv_heads):
            hs = slice(kv * group, (kv + 1) * group)
            for lo in range(0, nq, step):
                hi = min(nq, lo + step)
                visible = offset + hi
                keys_f, vals_f = k[kv, :visible].float(), v[kv, :visible].float()
                q_f = q[hs, lo:hi].float()
                scores = _causal_mask_((q_f @ keys_f.T) * scale, key_pos[:visible],
                                       torch.arange(offset + lo, offset + hi, device=dev))
                probs = torch.softmax(scores, -1)
                dscores = probs * (dout[hs, lo:hi] @ vals_f.T - rowdot[hs, lo:hi, None])
                dq[hs, lo:hi] = (dscores @ keys_f) * scale
                dk[kv, :visible] += (dscores.transpose(1, 2) @ q_f).sum(0) * scale
                dvv[kv, :visible] += (probs.transpose(1, 2) @ dout[hs, lo:hi]).sum(0)
        return dq.to(q.dtype), dk.to(k.dtype), dvv.to(v.dtype), None


def _pad_rows(x, pad):
    """Zero rows appended along dim 1 of [H, n] or [H, n, d]."""
    if not pad:
        return x
    return F.pad(x, (0, pad) if x.dim() == 2 else (0, 0, 0, pad))


def delta_rule_diff(q, k, v, g, beta, state, chunk=64):
    """The chunked gated delta rule of ops.delta_rule (same chunk grid, same formulas) built from out-of-place
    operations only, so that autograd runs through it. Returns out [H, n, dv] fp32."""
    heads, n, _ = k.shape
    n_chunks = -(-n // chunk)
    pad = n_chunks * chunk - n

    def split(x):
        x = _pad_rows(x.float(), pad)
        return x.reshape(heads, n_chunks, chunk, *x.shape[2:])

    qc, kc, vc, bc = split(q), split(k), split(v), split(beta)
    cum = split(g).cumsum(-1)                                                              # [H, nc, C]
    causal = torch.ones(chunk, chunk, dtype=torch.bool, device=k.device).tril()
    rel = cum[..., :, None] - cum[..., None, :]
    decay = torch.where(causal, rel, torch.full_like(rel, NEG_INF)).exp()
    strict = (bc[..., None] * (kc @ kc.transpose(-1, -2)) * decay).tril(-1)
    identity = torch.eye(chunk, device=k.device).expand_as(strict)
    inv = torch.linalg.solve_triangular(strict + identity, identity, upper=False, unitriangular=True)
    u = inv @ (bc[..., None] * vc)
    w = inv @ (bc[..., None] * cum.exp()[..., None] * kc)
    within = (qc @ kc.transpose(-1, -2)) * decay
    q_scaled = qc * cum.exp()[..., None]
    k_to_end = kc * (cum[..., -1:] - cum).exp()[..., None]
    s = state.float()
    pieces = []
    for c in range(n_chunks):
        v_new = u[:, c] - w[:, c] @ s
        pieces.append(q_scaled[:, c] @ s + within[:, c] @ v_new)
        s = s * cum[:, c, -1].exp()[:, None, None] + k_to_end[:, c].transpose(-1, -2) @ v_new
    return torch.cat(pieces, 1)[:, :n]


# ------------------------------------------------------------------------------------- late layers
def attn_kv(model, i, x, pos):
    """K and V after RoPE [Hkv, n, d] of attention layer i for normed rows x, as the cache holds them."""
    kv = getattr(model, "_attn_kv", None) or model._kv
    return kv(i, x, pos)


def _queries_and_gate(model, i, x, pos):
    if hasattr(model, "_attn_q"):
        return model._attn_q(i, x, pos)
    return model.queries(i, x, pos), None


def _late_attn(model, i, h, pos, k_pre, v_pre):
    """Attention layer i for rows h over [prefix K/V, the rows' own K/V] (model.layer's result)."""
    x = model.in_norm(h, model.W[i]["ln1"])
    q, gate = _queries_and_gate(model, i, x, pos)
    k_own, v_own = attn_kv(model, i, x, pos)
    o = CausalAttention.apply(q, torch.cat([k_pre, k_own], 1), torch.cat([v_pre, v_own], 1), model.scale)
    if gate is not None:
        o = o * torch.sigmoid(gate)
    return model.mlp(i, h + F.linear(o, model.W[i]["o"]))


def _late_gdn(model, i, h, conv, rec):
    """GDN layer i for rows h continuing a (constant) conv window and recurrent state (model.layer's result)."""
    x = model.in_norm(h, model.W[i]["ln1"])
    pre, b, a = model._gdn_inputs(i, x)
    mixed, _ = ops.causal_conv(pre, conv, model.W[i]["conv"])
    beta, g = model.gdn_gates(i, b, a)
    out = delta_rule_diff(*model.gdn_qkv(mixed), g, beta, rec).to(pre.dtype)
    return model.mlp(i, h + model._gdn_out(i, out, x))


def tail_loss(model, split, h0, pos, kv, gdn, rows, targets, recompute=True):
    """Mean NLL (fp32) of `targets` at tail rows `rows`: the tail rows (layer-split inputs h0 at positions pos)
    run through layers >= split over the prefix caches kv {i: (K, V)} and gdn {i: {conv, rec}}. recompute:
    checkpoint every layer (recomputed in the backward)."""
    use_checkpoint = recompute and torch.is_grad_enabled()
    h = h0
    for i in range(split, model.n_layers):
        if model.layer_types[i] == "attn":
            k_pre, v_pre = (t.to(h.device) for t in kv[i])
            fn, args = _late_attn, (model, i, h, pos, k_pre, v_pre)
        else:
            fn, args = _late_gdn, (model, i, h, gdn[i]["conv"], gdn[i]["rec"])
        h = checkpoint(fn, *args, use_reentrant=False) if use_checkpoint else fn(*args)
    return F.cross_entropy(model.logits(h[rows]), targets)


@torch.no_grad()
def exact_late(model, h_split, split, P, rows, targets, final=False, hook=None):
    """The exact late layers over every row from the layer-split inputs. Returns ({attention layer: (K, V) of
    rows [0, P) after RoPE, on the host}, the exact loss over `rows`), plus the last layer's output when final.
    hook(i, h) sees each late layer's input rows."""
    pos = torch.arange(h_split.shape[0], device=h_split.device)
    scratch = model.new_cache()
    true_kv = {}
    h = h_split
    for i in range(split, model.n_layers):
        if hook is not None:
            hook(i, h)
        h = model.layer(i, h, pos, scratch)
        if model.layer_types[i] == "attn":
            true_kv[i] = tuple(scratch[i][name][:, :P].cpu() for name in ("k", "v"))
        scratch[i] = {}
    loss = F.cross_entropy(model.logits(h[rows]), targets).item()
    if final:
        return true_kv, loss, h
    return true_kv, loss


@torch.no_grad()
def fill_late(model, split, P, fill_x):
    """Prefix fill of every late layer from inputs fill_x(i) [P, d], as prefill's fill step writes it. Returns
    ({attention layer: (K, V)}, {GDN layer: {conv, rec}})."""
    pos = torch.arange(P, device=fill_x(split).device)
    scratch = model.new_cache()
    kv, gdn = {}, {}
    for i in range(split, model.n_layers):
        model.fill(i, fill_x(i), pos, scratch)
        entry = scratch[i]
        if model.layer_types[i] == "attn":
            kv[i] = (entry["k"], entry["v"])
        else:
            gdn[i] = {"conv": entry["conv"], "rec": entry["rec"]}
        scratch[i] = {}
    return kv, gdn


class _RowSums:
    """Per-row sums folded from each K/V leaf's gradient the moment it is complete (the gradient is then freed)."""

    def __init__(self, P, device, true_kv):
        self.true_kv, self.device = true_kv, device
        zeros = lambda: torch.zeros(P, dtype=torch.float64, device=device)      # noqa: E731
        self.impact, self.err, self.grad2 = zeros(), zeros(), zeros()

    def hook(self, layer, which):
        def fold(leaf):
            true = self.true_kv[layer][which].to(self.device).float()
            diff = true - leaf.detach().float()
            grad = leaf.grad.float()
            self.impact += (grad * diff).sum((0, 2)).double()
            self.grad2 += grad.square().sum((0, 2)).double()
            scale = true.square().sum((0, 2)).sqrt().clamp_min(1e-6)
            self.err += 0.5 * (diff.square().sum((0, 2)).sqrt() / scale).double()
            leaf.grad = None
        return fold


def impact(model, split, h_tail, P, kv, true_kv, gdn, rows, targets):
    """Backward through the tail at the filled cache. Per prefix row (fp64, host): the signed first-order
    impact, the relative fill error (the mean over late attention layers of (|dK|/|K| + |dV|/|V|) / 2) and the
    gradient norm over every late attention K/V. Returns (dict of [P] tensors, the loss at the fill)."""
    dev = h_tail.device
    pos = torch.arange(P, P + h_tail.shape[0], device=dev)
    sums = _RowSums(P, dev, true_kv)
    leaves = {}
    for i, pair in kv.items():
        leaves[i] = tuple(t.detach().requires_grad_() for t in pair)
        for which, leaf in enumerate(leaves[i]):
            leaf.register_post_accumulate_grad_hook(sums.hook(i, which))
    with torch.enable_grad():
        loss = tail_loss(model, split, h_tail, pos, leaves, gdn, rows, targets)
        loss.backward()
    err = sums.err / max(1, len(kv))
    result = {"impact": sums.impact.cpu(), "err": err.cpu(), "grad_norm": sums.grad2.sqrt().cpu()}
    return result, float(loss.detach())


# ------------------------------------------------------------------------------ lookup statistics
def _blocks(q, k, scale, stride=1):
    """(query positions, keys visible, causal probabilities [group, m, visible]) per KV head and query block."""
    n_q_heads, n, _ = q.shape
    group = n_q_heads // k.shape[0]
    step = ops.query_block(group, n) * stride
    pos = torch.arange(n, device=q.device)
    for kv in range(k.shape[0]):
        keys_f = k[kv].float()
        heads = slice(kv * group, (kv + 1) * group)
        for lo in range(0, n, step):
            hi = min(n, lo + step)
            q_pos = pos[lo:hi:stride]
            scores = _causal_mask_((q[heads, q_pos].float() @ keys_f[:hi].T) * scale, pos[:hi], q_pos)
            yield q_pos, hi, torch.softmax(scores, -1)


@torch.no_grad()
def received_mass(q, k, scale, rows_below=None, stride=1, entropy=False):
    """Attention mass each key row receives from strictly later query rows, summed over query heads (causal
    column sums in the manner of H2O; code/kva/impact.py:234-268). q [Hq, n, d] after RoPE, k [Hkv, n, d].
    rows_below: also the mass from query rows < rows_below alone. stride s > 1: every s-th query row, scaled by
    s (unbiased in expectation at about 1/s of the cost). entropy: also each query row's attention entropy in
    nats, summed over heads (stride 1 only). Returns host fp64 [n] tensors: the total, then the rows_below part,
    then the entropy, as requested."""
    if entropy and stride != 1:
        raise ValueError("the entropy reads every query row: use stride 1")
    n = q.shape[1]
    total, below, ent = (torch.zeros(n, dtype=torch.float64, device=q.device) for _ in range(3))
    for q_pos, visible, probs in _blocks(q, k, scale, stride):
        if entropy:
            ent[q_pos] += torch.special.entr(probs).sum((0, 2)).double()
        own = torch.arange(visible, device=q.device)[None, :] == q_pos[:, None]
        per_query = probs.masked_fill(own, 0.0).sum(0) * stride                        # [m, visible]
        total[:visible] += per_query.sum(0).double()
        if rows_below is not None:
            below[:visible] += per_query[q_pos < rows_below].sum(0).double()
    out = [total.cpu()]
    if rows_below is not None:
        out.append(below.cpu())
    if entropy:
        out.append(ent.cpu())
    return tuple(out) if len(out) > 1 else out[0]


@torch.no_grad()
def row_stats(q, k, scale, local=64):
    """Each query row's own lookup, averaged over query heads: entropy in nats, the mass on row 0 (the sink) and
    the mass on its `local` most recent keys, itself included. Three host fp64 [n]."""
    n_q_heads, n, _ = q.shape
    ent, sink, near = (torch.zeros(n, dtype=torch.float64, device=q.device) for _ in range(3))
    for q_pos, visible, probs in _blocks(q, k, scale):
        keys = torch.arange(visible, device=q.device)[None, :]
        back = q_pos[:, None] - keys
        window = (back < local) & (back >= 0)
        ent[q_pos] += torch.special.entr(probs).sum(-1).sum(0).double()
        sink[q_pos] += probs[..., 0].sum(0).double()
        near[q_pos] += (probs * window).sum(-1).sum(0).double()
    return tuple((t / n_q_heads).cpu() for t in (ent, sink, near))


def leverage_map(stats_state, lam):
    """(mean, L) with |(x - mean) L|^2 the ridge hat value of a split state x under the map's own calibration
    scatter (Cxx + lam s I, as EigenFit fits it): how far a row lies outside the fit's data. Host fp64."""
    from ..ridge.fit import EigenFit
    fit = EigenFit(stats_state)
    whiten = (fit.evals + lam * fit.scale).sqrt()
    return fit.mean_x, fit.evecs / whiten.unsqueeze(0)


# ------------------------------------------------------------------- per-row features of [n, d] states
ROWS = 4096


def by_rows(fn, n, chunk=None):
    """fn(row slice) over row chunks, concatenated on the host in fp64: per-row features of [n, d] states with
    [chunk, d] temporaries only."""
    step = chunk or ROWS
    parts = [fn(slice(lo, min(n, lo + step))).double().cpu() for lo in range(0, n, step)]
    return torch.cat(parts)


def row_norm(x):
    return by_rows(lambda s: x[s].float().norm(dim=-1), x.shape[0])


def velocity(x, prev):
    """|x - prev| / |prev| per row: how far the last layers moved each row."""
    def moved(s):
        before = prev[s].float()
        return (x[s].float() - before).norm(dim=-1) / before.norm(dim=-1).clamp_min(1e-6)
    return by_rows(moved, x.shape[0])


def _log_floor(t):
    return t.clamp_min(1e-30).log()


def log_leverage(x, mean, L):
    mean = mean.to(x.device, torch.float32)
    L = L.to(x.device, torch.float32)
    return _log_floor(by_rows(lambda s: ((x[s].float() - mean) @ L).square().sum(-1), x.shape[0]))


def log_max_act(x):
    """log of max |x| over each row: massive-activation (sink-like) rows."""
    return _log_floor(by_rows(lambda s: x[s].float().abs().amax(-1), x.shape[0]))


@torch.no_grad()
def gdn_gates(model, i, h):
    """Per row at GDN layer i: the write strength sigmoid(b) and the log decay, each averaged over the value
    heads. Two host fp64 [n]."""
    ln = model.W[i]["ln1"]

    def gates(s):
        _, b, a = model._gdn_inputs(i, model.in_norm(h[s], ln))
        beta, g = model.gdn_gates(i, b, a)
        return torch.stack([beta.mean(0), g.mean(0)], dim=-1)
    both = by_rows(gates, h.shape[0])
    return both[:, 0], both[:, 1]


def repetition(ids, cap):
    """Per token: the log distance to the previous occurrence of the same id (cap at a first occurrence), a
    first-occurrence flag, and whether the (previous, current) pair occurred before. Three lists of floats."""
    ids = list(ids)
    last_at, seen_pairs = {}, set()
    dist, first, bigram = [], [], []
    for j, t in enumerate(ids):
        gap = j - last_at[t] if t in last_at else cap
        dist.append(math.log(max(1, min(gap, cap))))
        first.append(0.0 if t in last_at else 1.0)
        pair = (ids[j - 1], t) if j else None
        bigram.append(1.0 if pair in seen_pairs else 0.0)
        if pair is not None:
            seen_pairs.add(pair)
        last_at[t] = j
    return dist, first, bigram
