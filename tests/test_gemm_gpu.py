"""tcgen05 GEMM vs a plain PyTorch fp32 reference of the same op."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _ref(x, w):
    return x.float() @ w.float().T


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 512), (1000, 384, 200), (37, 4096, 4096),
                                   (4096, 4096, 4096), (300, 128, 1024)])
def test_linear(m, n, k):
    from ridgefill_data_b200.ops import gemm
    torch.manual_seed(0)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    got = gemm.linear(x, w).float()
    ref = _ref(x, w)
    err = (got - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err


def test_linear_bias_residual_inplace():
    from ridgefill_data_b200.ops import gemm
    torch.manual_seed(1)
    m, n, k = 513, 768, 320
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    h = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    ref = _ref(x, w) + b.float() + h.float()
    gemm.linear(x, w, bias=b, residual=h, out=h)
    err = (h.float() - ref).abs().max().item() / ref.abs().max().item()
    assert err < 1e-2, err


def test_linear_bn128_and_f32():
    from ridgefill_data_b200.ops import gemm
    torch.manual_seed(2)
    x = torch.randn(640, 512, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(200, 512, device="cuda", dtype=torch.bfloat16)
    ref = _ref(x, w)
    got = gemm.linear_f32(x, w, bn=128)
    assert torch.allclose(got, ref, rtol=1e-4, atol=1e-2)
    got16 = gemm.linear(x, w, bn=128).float()
    assert (got16 - ref).abs().max().item() / ref.abs().max().item() < 1e-2


def test_swiglu():
    from ridgefill_data_b200.ops import gemm
    torch.manual_seed(3)
    m, f, k = 700, 512, 256
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    g = torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.1
    u = torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.1
    got = gemm.swiglu_linear(x, gemm.pack_gate_up(g, u)).float()
    gr, ur = _ref(x, g), _ref(x, u)
    ref = torch.nn.functional.silu(gr) * ur
    assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-2


def test_gram_fp64_split_k():
    from ridgefill_data_b200.ops import gemm
    torch.manual_seed(4)
    n, dx, dy = 5000, 384, 256
    x = torch.randn(n, dx, device="cuda", dtype=torch.bfloat16)
    y = torch.randn(n, dy, device="cuda", dtype=torch.bfloat16)
    acc = torch.zeros(dx, dy, device="cuda", dtype=torch.float64)
    gemm.gram_acc(acc, x, y, k_chunk=1024)
    ref = x.double().T @ y.double()
    assert (acc - ref).abs().max().item() < 1e-3 * ref.abs().max().item()
    gemm.gram_acc(acc, x, y, k_chunk=8192)
    assert (acc - 2 * ref).abs().max().item() < 2e-3 * ref.abs().max().item()


def test_no_error_recorded():
    from ridgefill_data_b200.ops._ext import check_errors
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("m,n,k", [(256, 256, 64), (300, 1000, 200), (1024, 5120, 5120), (4100, 2304, 1024)])
def test_two_sm_gemm_matches_one_sm_and_fp32(m, n, k):
    """The cta_group::2 kernel (256 x 256 tiles over an SM pair) against the fp32 reference and the one-SM kernel,
    with bias and residual, and the SwiGLU epilogue."""
    from ridgefill_data_b200.ops import gemm
    from ridgefill_data_b200.ops._ext import check_errors, ext
    torch.manual_seed(5)
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    h = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    ref = _ref(x, w) + b.float() + h.float()
    outs = {}
    for two in (True, False):
        was = ext().set_gemm_2sm(two)
        try:
            outs[two] = gemm.linear(x, w, bias=b, residual=h, bn=256).float()
        finally:
            ext().set_gemm_2sm(was)
    for two, got in outs.items():
        err = (got - ref).abs().max().item() / ref.abs().max().item()
        assert err < 1e-2, (two, err)
    assert (outs[True] - outs[False]).abs().max().item() <= 1e-2 * ref.abs().max().item()
    if n % 256 == 0:
        g = torch.randn(n // 2, k, device="cuda", dtype=torch.bfloat16) * 0.05
        u = torch.randn(n // 2, k, device="cuda", dtype=torch.bfloat16) * 0.05
        act = gemm.swiglu_linear(x, gemm.pack_gate_up(g, u)).float()
        rg, ru = _ref(x, g), _ref(x, u)
        want = torch.nn.functional.silu(rg) * ru
        assert (act - want).abs().max().item() / want.abs().max().item() < 2e-2
    torch.cuda.synchronize()
    check_errors()


@pytest.mark.parametrize("m", [1, 2, 3, 5, 8, 9, 13, 16])
@pytest.mark.parametrize("kernel", ["mma", "simt"])
def test_small_m_gemv_epilogues_match_fp32_and_tile_gemm(m, kernel):
    """1-16 row products (a decode step) take a GEMV kernel (csrc/gemv.cu; the tensor-core one for 1-16 rows, the
    CUDA-core one for 1-8): store with bias + residual written in place, fp32, and the packed SwiGLU, against the
    fp32 reference and the tile GEMM (gemv switched off)."""
    from ridgefill_data_b200.ops import gemm
    from ridgefill_data_b200.ops._ext import check_errors, ext
    if kernel == "simt" and m > 8:
        pytest.skip("the CUDA-core GEMV takes at most 8 rows")
    torch.manual_seed(11 + m)
    k, n, f = 1000, 1000, 256          # k not a multiple of the 32-wide k block; n not a multiple of 16 columns
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.05
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    h = torch.randn(m, n, device="cuda", dtype=torch.bfloat16)
    g = torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.1
    u = torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.1
    gu = gemm.pack_gate_up(g, u)
    outs = {}
    rows_was = ext().set_gemv_max_rows(16)                 # every row count of the test on the GEMV
    mma_was = ext().set_gemv_mma(kernel == "mma")
    for on in (True, False):
        was = ext().set_gemv(on)
        try:
            hh = h.clone()
            n0 = ext().launch_count()
            gemm.linear(x, w, bias=b, residual=hh, out=hh)
            outs[on] = (hh.float(), gemm.linear_f32(x, w), gemm.swiglu_linear(x, gu).float())
            launches = ext().launch_count() - n0
        finally:
            ext().set_gemv(was)
    ext().set_gemv_mma(mma_was)
    ext().set_gemv_max_rows(rows_was)
    torch.cuda.synchronize()
    check_errors()
    assert launches == 3
    ref_store = _ref(x, w) + b.float() + h.float()
    ref_f32 = _ref(x, w)
    ref_sw = torch.nn.functional.silu(_ref(x, g)) * _ref(x, u)
    for got, ref in zip(outs[True], (ref_store, ref_f32, ref_sw)):
        assert (got - ref).abs().max().item() / ref.abs().max().item() < 1e-2
    for a, b2 in zip(outs[True], outs[False]):
        assert (a - b2).abs().max().item() / b2.abs().max().item() < 1e-2


def test_mma_gemv_rows_do_not_depend_on_the_batch():
    """The tensor-core GEMV sums every row in one fixed order (its k blocks per warp, the warps in turn), so a row's
    result is the same bits whether it runs alone or with up to 15 other rows, on every epilogue."""
    from ridgefill_data_b200.ops import gemm
    from ridgefill_data_b200.ops._ext import check_errors, ext
    torch.manual_seed(5)
    k, n, f = 5120, 1024, 512
    x = torch.randn(16, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02
    b = torch.randn(n, device="cuda", dtype=torch.bfloat16)
    gu = gemm.pack_gate_up(torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.02,
                           torch.randn(f, k, device="cuda", dtype=torch.bfloat16) * 0.02)
    rows_was, mma_was, on_was = ext().set_gemv_max_rows(16), ext().set_gemv_mma(True), ext().set_gemv(True)
    try:
        full = (gemm.linear(x, w, bias=b), gemm.linear_f32(x, w), gemm.swiglu_linear(x, gu))
        for m in (1, 2, 3, 7, 8, 9, 15):
            part = (gemm.linear(x[-m:], w, bias=b), gemm.linear_f32(x[-m:], w), gemm.swiglu_linear(x[-m:], gu))
            for a, ref in zip(part, full):
                assert torch.equal(a, ref[-m:]), (m, (a.float() - ref[-m:].float()).abs().max())
    finally:
        ext().set_gemv(on_was)
        ext().set_gemv_mma(mma_was)
        ext().set_gemv_max_rows(rows_was)
    torch.cuda.synchronize()
    check_errors()