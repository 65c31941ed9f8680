"""fp64 ridge solves X = (A + shift I)^-1 B for symmetric positive semi-definite A.

CPU tensors: torch.linalg (LAPACK) Cholesky + triangular solves. CUDA tensors: the sm_100a fp64
kernels of csrc/linalg.cu (blocked right-looking Cholesky, then blocked forward and backward
substitution over all right-hand sides at once).
"""
from __future__ import annotations

import torch


def ridge_solve(a, b, shift):
    a = a.double()
    b = b.double()
    if a.is_cuda:
        from ..ops import linalg
        return linalg.ridge_solve(a, b, float(shift))
    m = a + shift * torch.eye(a.shape[0], dtype=a.dtype, device=a.device)
    chol = torch.linalg.cholesky(m)
    return torch.cholesky_solve(b, chol)
