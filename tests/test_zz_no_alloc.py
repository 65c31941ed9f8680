"""The allocation-free Gated DeltaNet entry point, called through its exported C symbol.

rf_gdn_chunk_scan_noalloc serves callers that may not allocate device memory while they run (a server
that gives each request a fixed slice of a reserved pool, a runtime whose own allocator must own every
byte, a latency-critical loop that cannot afford cudaMalloc's synchronisation). It takes its scratch from
a fixed device array inside the library, so it must produce exactly what the allocating entry point
(ops.kernels.gdn_scan) produces, call after call, and refuse shapes that do not fit the array.
This file is collected last so a failure here never hides the rest of the suite.
"""
import ctypes

import pytest
import torch

pytestmark = pytest.mark.gpu

C_VOIDP, C_INT, C_LONG = ctypes.c_void_p, ctypes.c_int, ctypes.c_long


def _lib():
    import ridgefill_data_b200._C as ext
    lib = ctypes.CDLL(ext.__file__)
    f = lib.rf_gdn_chunk_scan_noalloc
    f.restype = C_INT
    f.argtypes = [C_VOIDP, C_VOIDP, C_VOIDP, C_VOIDP, C_VOIDP, C_VOIDP, C_VOIDP, C_LONG,
                  C_INT, C_INT, C_INT, C_INT, C_INT, C_VOIDP]
    lib.rf_gdn_noalloc_scratch_bytes.restype = ctypes.c_size_t
    lib.rf_gdn_noalloc_scratch_bytes.argtypes = [C_INT] * 6
    lib.rf_gdn_noalloc_capacity.restype = ctypes.c_size_t
    lib.rf_gdn_noalloc_strerror.restype = ctypes.c_char_p
    lib.rf_gdn_noalloc_strerror.argtypes = [C_INT]
    lib.rf_gdn_noalloc_last_error.restype = C_INT
    lib.rf_gdn_noalloc_last_error.argtypes = [ctypes.POINTER(C_INT), C_VOIDP]
    return lib


def _last_error(lib, stream):
    code = C_INT(-1)
    rc = lib.rf_gdn_noalloc_last_error(ctypes.byref(code), stream)
    return rc, code.value


def _inputs(n, nk, nv, dk, dv, seed):
    from ridgefill_data_b200.ops import kernels as K
    g = torch.Generator(device="cuda").manual_seed(seed)
    C = 2 * nk * dk + nv * dv
    proj = (torch.randn(n, C + 2 * nv, device="cuda", generator=g) * 0.5).bfloat16()
    conv_w = (torch.randn(C, 4, device="cuda", generator=g) / 2).bfloat16()
    A_log = torch.rand(nv, device="cuda", generator=g) * 2.7
    dt = torch.randn(nv, device="cuda", generator=g) * 0.1
    state = torch.randn(nv, dk, dv, device="cuda", generator=g) * 0.1
    return K.gdn_prep(proj, C, C + nv, conv_w, None, A_log, dt, nk, nv, dk, dv), state


def _ptr(t):
    return None if t is None else t.data_ptr()


def _largest_n(lib, nk, nv, dk, dv, output_mode):
    """The longest sequence (a multiple of 64) whose scratch fits the fixed array."""
    cap, n = lib.rf_gdn_noalloc_capacity(), 64
    while lib.rf_gdn_noalloc_scratch_bytes(n + 64, nk, nv, dk, dv, output_mode) <= cap:
        n += 64
    return n


@pytest.mark.parametrize("output_mode", [True, False])
@pytest.mark.parametrize("shape", ["n300_dv128", "n300_dv64", "at_capacity"])
def test_noalloc_matches_allocating_entry_point_twice(output_mode, shape):
    from ridgefill_data_b200.ops import kernels as K
    lib = _lib()
    n, nk, nv, dk, dv = 300, 2, 4, 128, 128
    if shape == "n300_dv64":
        dv = 64
    elif shape == "at_capacity":               # the largest call the array admits; 64 more tokens are refused
        n = _largest_n(lib, nk, nv, dk, dv, int(output_mode))
        cap = lib.rf_gdn_noalloc_capacity()
        assert lib.rf_gdn_noalloc_scratch_bytes(n, nk, nv, dk, dv, int(output_mode)) <= cap
        assert lib.rf_gdn_noalloc_scratch_bytes(n + 64, nk, nv, dk, dv, int(output_mode)) > cap
    stream = torch.cuda.current_stream().cuda_stream
    for call, seed in enumerate((11, 12)):          # two calls in a row share the scratch array
        (q, k, v, beta, g), state = _inputs(n, nk, nv, dk, dv, seed)
        ref_state = state.clone()
        ref_out = torch.empty(n, nv * dv, device="cuda", dtype=torch.bfloat16) if output_mode else None
        K.gdn_scan(q if output_mode else None, k, v, beta, g, ref_state, ref_out, groups=1)   # sequential scan
        dut_state = state.clone()
        dut_out = torch.full((n, nv * dv), float("nan"), device="cuda", dtype=torch.bfloat16) if output_mode else None
        rc = lib.rf_gdn_chunk_scan_noalloc(_ptr(q) if output_mode else None, _ptr(k), _ptr(v), _ptr(beta), _ptr(g),
                                          _ptr(dut_state), _ptr(dut_out), nv * dv, n, nk, nv, dk, dv, stream)
        assert rc == 0, lib.rf_gdn_noalloc_strerror(rc)
        assert _last_error(lib, stream) == (0, 0)   # no kernel recorded an error
        torch.cuda.synchronize()
        rel = ((dut_state - ref_state).norm() / ref_state.norm()).item()
        assert rel < 1e-6, (call, rel)
        assert torch.isfinite(dut_state).all()
        if output_mode:
            assert torch.isfinite(dut_out.float()).all()
            rel_o = ((dut_out.float() - ref_out.float()).norm() / ref_out.float().norm()).item()
            assert rel_o < 1e-6, (call, rel_o)


def test_noalloc_rejects_shapes_beyond_the_array():
    lib = _lib()
    cap = lib.rf_gdn_noalloc_capacity()
    n, nk, nv, dk, dv = 65536, 16, 48, 128, 128
    assert lib.rf_gdn_noalloc_scratch_bytes(n, nk, nv, dk, dv, 1) > cap
    dummy = torch.zeros(8, device="cuda")
    p = dummy.data_ptr()
    rc = lib.rf_gdn_chunk_scan_noalloc(p, p, p, p, p, p, p, nv * dv, n, nk, nv, dk, dv,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 2 and b"16 MiB" in lib.rf_gdn_noalloc_strerror(rc)
    rc = lib.rf_gdn_chunk_scan_noalloc(p, p, p, p, p, p, p, nv * dv, 100, nk, nv, 64, dv,
                                      torch.cuda.current_stream().cuda_stream)
    assert rc == 1
