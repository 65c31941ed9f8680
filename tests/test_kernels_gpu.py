"""sm_100a kernels vs the plain PyTorch fp32 oracle of the same op (ops/oracle.py)."""
import pytest
import torch
import torch.nn.functional as F

from ridgefill_data_b200.ops import kernels as K
from ridgefill_data_b200.ops import oracle as O

pytestmark = pytest.mark.gpu
dev = "cuda"


def _rel(a, b):
    return ((a.float() - b.float()).norm() / b.float().norm().clamp_min(1e-30)).item()


@pytest.mark.parametrize("zc", [False, True])
def test_rmsnorm(zc):
    torch.manual_seed(0)
    x = torch.randn(37, 5120, device=dev).bfloat16()
    w = (torch.randn(5120, device=dev) * 0.1 + (0 if zc else 1)).bfloat16()
    got = K.rmsnorm(x, w, 1e-6, zc)
    ref = (O.rms_norm_zc if zc else O.rms_norm)(x, w, 1e-6)
    assert (got.float() - ref.float()).abs().max().item() <= 2 * ref.float().abs().max().item() / 128


@pytest.mark.parametrize("hd,rot,mode", [(128, 128, 0), (256, 64, 1), (128, 128, -1)])
def test_head_norm_rope(hd, rot, mode):
    torch.manual_seed(1)
    n, h = 50, 3
    src = torch.randn(n, h * hd, device=dev).bfloat16()
    w = (torch.randn(hd, device=dev) * 0.1 + (1 if mode == 0 else 0)).bfloat16()
    inv = O.inv_freq_default(1e6, rot)
    tables = K.rope_tables(inv, 4096, dev)
    dst = torch.empty(h, n, hd, device=dev, dtype=torch.bfloat16)
    K.head_norm_rope(src, h, hd, hd, dst, n * hd, hd, norm_w=w if mode >= 0 else None, norm_mode=mode, eps=1e-6,
                     tables=tables, rot=rot, pos_offset=100)
    x = src.view(n, h, hd)
    if mode == 0:
        x = O.rms_norm(x, w, 1e-6)
    elif mode == 1:
        x = O.rms_norm_zc(x, w, 1e-6)
    cos, sin = O.rope_cos_sin(inv, torch.arange(100, 100 + n, device=dev), torch.bfloat16)
    ref = O.apply_rope(x.transpose(0, 1), cos, sin)
    assert _rel(dst, ref) < 1e-2


@pytest.mark.parametrize("impl", ["mma", "auto"])
@pytest.mark.parametrize("hd,hq,hkv,nq,nk,gated", [(128, 8, 2, 300, 300, False), (256, 6, 1, 200, 700, True),
                                                    (64, 4, 4, 1, 513, False), (128, 4, 1, 130, 130, True),
                                                    (256, 3, 1, 1000, 1000, True), (128, 4, 2, 64, 2000, False),
                                                    (256, 2, 2, 129, 4100, False)])
def test_flash_attention(hd, hq, hkv, nq, nk, gated, impl):
    torch.manual_seed(2)
    q = torch.randn(hq, nq, hd, device=dev).bfloat16()
    k = torch.randn(hkv, nk + 64, hd, device=dev).bfloat16()
    v = torch.randn(hkv, nk + 64, hd, device=dev).bfloat16()
    gate = torch.randn(nq, hq * 2 * hd, device=dev).bfloat16()
    out = torch.empty(nq, hq * hd, device=dev, dtype=torch.bfloat16)
    k[:, nk:] = float("nan")           # rows past nk must never be read into the result
    v[:, nk:] = float("nan")
    K.attention(q, k, v, nk, hd ** -0.5, out, q_start=nk - nq, gate=gate[:, hd:] if gated else None,
                gate_head=2 * hd, impl=impl)
    ref = O.attend(q, k[:, :nk], v[:, :nk], hd ** -0.5)
    if gated:
        g = gate.view(nq, hq, 2 * hd)[..., hd:].reshape(nq, -1)
        ref = ref * torch.sigmoid(g)
    assert _rel(out, ref) < 2e-2
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("impl,hd,nk,nsel,gated", [("mma", 128, 400, 90, False), ("tcgen05", 128, 400, 90, False),
                                                  ("tcgen05", 256, 1000, 300, True), ("tcgen05", 128, 2100, 700, False)])
def test_flash_attention_qpos(impl, hd, nk, nsel, gated):
    """Queries at arbitrary ascending positions (the exact rows of a bypass arm) against the fp32 oracle."""
    torch.manual_seed(3)
    hq, hkv = 4, 2
    qpos = torch.tensor(sorted(set(torch.randint(0, nk, (nsel,)).tolist())), device=dev)
    nq = qpos.numel()
    q = torch.randn(hq, nq, hd, device=dev).bfloat16()
    k = torch.randn(hkv, nk, hd, device=dev).bfloat16()
    v = torch.randn(hkv, nk, hd, device=dev).bfloat16()
    gate = torch.randn(nq, hq * 2 * hd, device=dev).bfloat16() if gated else None
    out = torch.empty(nq, hq * hd, device=dev, dtype=torch.bfloat16)
    K.attention(q, k, v, nk, hd ** -0.5, out, qpos=qpos.int(), gate=gate[:, hd:] if gated else None,
                gate_head=2 * hd, impl=impl)
    ref = O.attend_at(q, k, v, hd ** -0.5, qpos)
    if gated:
        ref = ref * torch.sigmoid(gate.view(nq, hq, 2 * hd)[..., hd:].reshape(nq, -1).float())
    assert _rel(out, ref) < 2e-2
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("n,need_out,with_state", [(200, True, False), (64, True, True), (333, False, True),
                                                   (1, True, True)])
def test_gdn_prep_and_scan(n, need_out, with_state):
    torch.manual_seed(4)
    nk, nv, dk, dv, kk = 2, 6, 128, 128, 4
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(n, C + 2 * nv, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, kk, device=dev) / 2).bfloat16()
    A_log = torch.empty(nv, device=dev).uniform_(0, 2.7)
    dt = torch.randn(nv, device=dev) * 0.1
    conv_state = (torch.randn(kk - 1, C, device=dev) * 0.5).bfloat16() if with_state else None
    state = torch.randn(nv, dk, dv, device=dev) * 0.1 if with_state else torch.zeros(nv, dk, dv, device=dev)
    q, k, v, beta, g = K.gdn_prep(proj, C, C + nv, conv_w, conv_state, A_log, dt, nk, nv, dk, dv)
    # oracle
    co, new_state = O.causal_conv(proj[:, :C], conv_state, conv_w)
    rep = nv // nk
    qo, ko, vo = co.split([nk * dk, nk * dk, nv * dv], -1)
    qo = O.l2norm(qo.reshape(n, nk, dk).float()).transpose(0, 1) * dk ** -0.5
    ko = O.l2norm(ko.reshape(n, nk, dk).float()).transpose(0, 1)
    vo = vo.reshape(n, nv, dv).float().transpose(0, 1)
    bo = torch.sigmoid(proj[:, C:C + nv]).float().T
    go = (-A_log.exp() * F.softplus(proj[:, C + nv:].float() + dt)).T
    assert _rel(q, qo) < 1e-2 and _rel(k, ko) < 1e-2 and _rel(v, vo) < 1e-2
    assert _rel(beta, bo) < 1e-2 and _rel(g, go) < 1e-3
    cs = conv_state.clone() if conv_state is not None else torch.zeros(kk - 1, C, device=dev, dtype=torch.bfloat16)
    K.gdn_conv_state_update(proj, cs, C)
    assert torch.equal(cs, new_state)
    out = torch.empty(n, nv * dv, device=dev, dtype=torch.bfloat16) if need_out else None
    st = state.clone()
    K.gdn_scan(q if need_out else None, k, v, beta, g, st, out)
    ro, rs, _ = O.delta_rule(qo.repeat_interleave(rep, 0), ko.repeat_interleave(rep, 0), vo, go, bo, state)
    assert _rel(st, rs) < 3e-2
    if need_out:
        assert _rel(out.view(n, nv, dv).transpose(0, 1), ro) < 3e-2
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("n,dv,groups", [(1000, 128, 1), (1000, 128, 4), (333, 64, 1), (64, 128, 1)])
def test_gdn_fused_output_pass_matches_split_and_oracle(n, dv, groups):
    """Output mode computed inside the state pass (no chunk-start states in memory), on tcgen05 with the state in
    TMEM and on mma.sync, against the split form (state pass storing chunk states and V', then the parallel output
    pass) and the fp32 oracle: sequential and two-level scans, a partial last chunk and dv 64 (mma.sync only)."""
    from ridgefill_data_b200.ops._ext import check_errors, ext
    torch.manual_seed(17)
    nk, nv, dk = 1, 3, 128
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(n, C + 2 * nv, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, 4, device=dev) / 2).bfloat16()
    A_log = torch.empty(nv, device=dev).uniform_(0, 2.7)
    dt = torch.randn(nv, device=dev) * 0.1
    state = torch.randn(nv, dk, dv, device=dev) * 0.1
    q, k, v, beta, g = K.gdn_prep(proj, C, C + nv, conv_w, None, A_log, dt, nk, nv, dk, dv)
    outs, states = {}, {}
    # 2: fused on tcgen05 (state in TMEM, where dk = dv = 128), 1: fused on mma.sync, 0: split passes
    for mode in (2, 1, 0):
        was_f = ext().set_gdn_fused_output(1 if mode else 0)
        was_t = ext().set_gdn_state_tc(1 if mode == 2 else 0)
        try:
            out = torch.empty(n, nv * dv, device=dev, dtype=torch.bfloat16)
            st = state.clone()
            K.gdn_scan(q, k, v, beta, g, st, out, groups=groups)
            outs[mode], states[mode] = out, st
        finally:
            ext().set_gdn_fused_output(was_f)
            ext().set_gdn_state_tc(was_t)
        torch.cuda.synchronize()
        check_errors()
    assert _rel(states[1], states[0]) < 1e-4    # same recurrence, fp32 contraction order may differ
    assert _rel(outs[1].float(), outs[0].float()) < 1e-2
    assert _rel(states[2], states[0]) < 1e-2    # tcgen05: bf16 state operand rounded at other points
    assert _rel(outs[2].float(), outs[0].float()) < 1e-2
    co, _ = O.causal_conv(proj[:, :C], None, conv_w)
    qo, ko, vo = co.split([nk * dk, nk * dk, nv * dv], -1)
    qo = O.l2norm(qo.reshape(n, nk, dk).float()).transpose(0, 1) * dk ** -0.5
    ko = O.l2norm(ko.reshape(n, nk, dk).float()).transpose(0, 1)
    vo = vo.reshape(n, nv, dv).float().transpose(0, 1)
    bo = torch.sigmoid(proj[:, C:C + nv]).float().T
    go = (-A_log.exp() * F.softplus(proj[:, C + nv:].float() + dt)).T
    ro, rs, _ = O.delta_rule(qo.repeat_interleave(nv, 0), ko.repeat_interleave(nv, 0), vo, go, bo, state)
    for mode in (2, 1):
        assert _rel(outs[mode].view(n, nv, dv).transpose(0, 1), ro) < 3e-2
        assert _rel(states[mode], rs) < 3e-2


@pytest.mark.parametrize("groups", [3, 8])
@pytest.mark.parametrize("need_out", [False, True])
def test_gdn_two_level_scan_matches_sequential_and_oracle(groups, need_out):
    """The chunk-parallel scan (group end states from zero, group transfer matrices, sequential propagation with
    split-bf16 products, then the per-group rerun for outputs) against the sequential scan and the fp32 oracle."""
    torch.manual_seed(5)
    n, nk, nv, dk, dv = 1500, 1, 2, 128, 128
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(n, C + 2 * nv, device=dev) * 0.5).bfloat16()
    conv_w = (torch.randn(C, 4, device=dev) / 2).bfloat16()
    A_log = torch.empty(nv, device=dev).uniform_(0, 2.7)
    dt = torch.randn(nv, device=dev) * 0.1
    state = torch.randn(nv, dk, dv, device=dev) * 0.1
    q, k, v, beta, g = K.gdn_prep(proj, C, C + nv, conv_w, None, A_log, dt, nk, nv, dk, dv)
    outs, states = {}, {}
    for grp in (1, groups):
        out = torch.empty(n, nv * dv, device=dev, dtype=torch.bfloat16) if need_out else None
        st = state.clone()
        K.gdn_scan(q if need_out else None, k, v, beta, g, st, out, groups=grp)
        outs[grp], states[grp] = out, st
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()
    assert _rel(states[groups], states[1]) < 5e-3
    if need_out:
        assert _rel(outs[groups].float(), outs[1].float()) < 1e-2
    co, _ = O.causal_conv(proj[:, :C], None, conv_w)
    qo, ko, vo = co.split([nk * dk, nk * dk, nv * dv], -1)
    qo = O.l2norm(qo.reshape(n, nk, dk).float()).transpose(0, 1) * dk ** -0.5
    ko = O.l2norm(ko.reshape(n, nk, dk).float()).transpose(0, 1)
    vo = vo.reshape(n, nv, dv).float().transpose(0, 1)
    bo = torch.sigmoid(proj[:, C:C + nv]).float().T
    go = (-A_log.exp() * F.softplus(proj[:, C + nv:].float() + dt)).T
    ro, rs, _ = O.delta_rule(qo.repeat_interleave(nv, 0), ko.repeat_interleave(nv, 0), vo, go, bo, state)
    assert _rel(states[groups], rs) < 3e-2
    if need_out:
        assert _rel(outs[groups].view(n, nv, dv).transpose(0, 1), ro) < 3e-2


@pytest.mark.parametrize("variant", [("set_attn_softmax_groups", 2), ("set_attn_s_buffers", 2),
                                     ("set_attn_s_buffers", 3), ("set_attn_p_buffers", 1), ("set_attn_rotate", 1),
                                     ("set_attn_q_tmem", 1)])
@pytest.mark.parametrize("hd", [128, 256])
def test_flash_attention_pipeline_variants(variant, hd):
    """The tcgen05 attention's pipeline variants (two softmax warpgroups swapping the row max per tile, two or
    three TMEM S buffers, one P buffer, key tiles in a per-CTA rotated order, Q read from TMEM by the S product) against the fp32 oracle and the default build, causal over 300 rows with
    keys past the last query tile."""
    from ridgefill_data_b200.ops._ext import check_errors, ext
    setter, value = variant
    torch.manual_seed(13)
    hq, hkv, nq = 4, 2, 300
    q = torch.randn(hq, nq, hd, device=dev).bfloat16()
    k = torch.randn(hkv, nq, hd, device=dev).bfloat16()
    v = torch.randn(hkv, nq, hd, device=dev).bfloat16()
    ref = O.attend(q, k, v, hd ** -0.5)
    outs = {}
    for mode in ("default", "variant"):
        was = getattr(ext(), setter)(value) if mode == "variant" else None
        try:
            out = torch.empty(nq, hq * hd, device=dev, dtype=torch.bfloat16)
            K.attention(q, k, v, nq, hd ** -0.5, out, impl="tcgen05")
            outs[mode] = out
        finally:
            if was is not None:
                getattr(ext(), setter)(was)
    check_errors(dev)
    assert _rel(outs["variant"], ref) < 2e-2
    assert _rel(outs["variant"], outs["default"]) < 5e-3


@pytest.mark.parametrize("poly", [2, 4])
@pytest.mark.parametrize("hd", [128, 256])
def test_flash_attention_with_fma_exponentials(poly, hd):
    """Part of every row's exponentials on the FMA pipe (range-reduced cubic, csrc/attention_tc.cu exp2_fma): the
    result stays within the same tolerance of the fp32 oracle as the special-function path, and close to it."""
    from ridgefill_data_b200.ops._ext import ext
    torch.manual_seed(9)
    hq, hkv, nq = 4, 2, 300
    q = torch.randn(hq, nq, hd, device=dev).bfloat16()
    k = torch.randn(hkv, nq, hd, device=dev).bfloat16()
    v = torch.randn(hkv, nq, hd, device=dev).bfloat16()
    ref = O.attend(q, k, v, hd ** -0.5)
    outs = {}
    for mode in (0, poly):
        was = ext().set_attn_poly(mode)
        try:
            out = torch.empty(nq, hq * hd, device=dev, dtype=torch.bfloat16)
            K.attention(q, k, v, nq, hd ** -0.5, out, impl="tcgen05")
            outs[mode] = out
        finally:
            ext().set_attn_poly(was)
    assert _rel(outs[poly], ref) < 2e-2
    assert _rel(outs[poly], outs[0]) < 5e-3
