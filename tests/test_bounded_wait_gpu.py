"""A bounded device wait that runs out: the kernel records the timeout in the error word, returns, and leaves the
context usable; the host reads the code (ops._ext.check_errors raises KernelError).

The wait is made to expire without any fault: one CUDA block waits, with a 2 ms limit, on flags in this GPU's own
memory that nothing ever sets (the shape of a peer rank that never arrives). This is the failure-detection path
of every peer-flag wait in csrc/comm.cu, csrc/nvls.cu and the fused GEMM epilogues."""
import time

import pytest
import torch

pytestmark = pytest.mark.gpu


def test_peer_wait_times_out_and_the_context_survives():
    from ridgefill_data_b200.ops import kernels as K
    from ridgefill_data_b200.ops._ext import KernelError, check_errors, ext
    x = ext()
    dev = torch.cuda.current_device()
    check_errors(dev)                                   # start from a clear word
    flags = torch.zeros(8, dtype=torch.int32, device="cuda")
    err = x.error_word(dev)
    torch.cuda.synchronize()
    t0 = time.perf_counter()
    x.comm_wait(flags.data_ptr(), 0, 2, 1, err, limit_ns=2_000_000)    # two "ranks" that never arrive
    torch.cuda.synchronize()
    waited = time.perf_counter() - t0
    assert waited < 5.0                                 # returned at its own limit, far below the 10 s default
    with pytest.raises(KernelError) as e:
        check_errors(dev)
    assert e.value.code == 4                            # kErrTimeoutPeer
    check_errors(dev)                                   # the word was cleared
    # the context still runs kernels and gives right answers
    a = torch.randn(64, 256, device="cuda").bfloat16()
    w = torch.ones(256, device="cuda").bfloat16()
    y = K.rmsnorm(a, w, 1e-6, False).float()
    ref = a.float() * torch.rsqrt(a.float().pow(2).mean(-1, keepdim=True) + 1e-6)
    torch.testing.assert_close(y, ref, atol=2e-2, rtol=2e-2)


def test_peer_wait_returns_at_once_when_the_flags_are_set():
    from ridgefill_data_b200.ops._ext import check_errors, ext
    x = ext()
    dev = torch.cuda.current_device()
    flags = torch.full((8,), 7, dtype=torch.int32, device="cuda")
    x.comm_wait(flags.data_ptr(), 2, 4, 7, x.error_word(dev), limit_ns=2_000_000)
    torch.cuda.synchronize()
    check_errors(dev)                                   # no error recorded
