"""fp64 ridge solve on the device (csrc/linalg.cu): blocked Cholesky of (A + shift I) and blocked triangular
solves for all right-hand sides at once."""
from __future__ import annotations

import torch

from ._ext import check_errors, ext


def ridge_solve(a, b, shift):
    """X = (a + shift I)^-1 b for symmetric positive definite a [n, n] (fp64, CUDA) and b [n, R]."""
    A = a.double().contiguous().clone()
    X = b.double().contiguous().clone()
    err = ext().error_word(A.device.index or 0)
    ext().cholesky_solve(A, X, float(shift), err)
    torch.cuda.synchronize(A.device)
    code = int(err.item())
    if code:
        err.zero_()
        raise ValueError("ridge_solve: the shifted scatter is not positive definite (raise lambda)")
    check_errors(A.device)
    return X
