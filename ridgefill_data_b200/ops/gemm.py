"""tcgen05 GEMM entry points (csrc/gemm.cu).

linear(x, w)        x @ w.T (+ bias) (+ residual), bf16 out: the F.linear layout of every projection
swiglu_linear(x, w) silu(x @ g.T) * (x @ u.T) with w the gate/up rows interleaved per 128-row block
                    (pack_gate_up builds it)
gram_acc(acc, x, y) acc += x.T @ y in fp64, fp32 per k-chunk of rows (ridge sufficient statistics)
"""
import torch

from ._ext import ext

EPI_STORE, EPI_SWIGLU, EPI_F32, EPI_F64ACC = 0, 1, 2, 3


def _bn(n):
    return 256 if n >= 2048 or n % 256 == 0 else 128


def linear(x, w, bias=None, residual=None, out=None, bn=None, max_ctas=0):
    """x [M, K] bf16, w [N, K] bf16 -> [M, N] bf16 = x w^T + bias (+ residual, which may be `out`). max_ctas > 0: the
    GEMM keeps to that many SMs (the others stay free for a kernel running beside it on another stream)."""
    m, n = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.bfloat16, device=x.device)
    ext().gemm(x, w, out, bias, residual, EPI_STORE, bn or _bn(n), False, False, 1, 0, int(max_ctas))
    return out


def linear_f32(x, w, out=None, bn=None):
    m, n = x.shape[0], w.shape[0]
    if out is None:
        out = torch.empty(m, n, dtype=torch.float32, device=x.device)
    ext().gemm(x, w, out, None, None, EPI_F32, bn or _bn(n), False, False, 1, 0, 0)
    return out


def pack_gate_up(gate, up, block=128):
    """[2F, K] with rows [gate block j ; up block j] for every 128-row block j (F % block == 0)."""
    f, k = gate.shape
    assert f % block == 0, f"FFN width {f} must be a multiple of {block}"
    return torch.stack((gate.view(f // block, block, k), up.view(f // block, block, k)), 1).reshape(2 * f, k)


def swiglu_linear(x, w_gu, out=None, block=128):
    """x [M, K], w_gu = pack_gate_up(gate, up) [2F, K] -> silu(x g^T) * (x u^T) [M, F]."""
    m, n2 = x.shape[0], w_gu.shape[0]
    if out is None:
        out = torch.empty(m, n2 // 2, dtype=torch.bfloat16, device=x.device)
    ext().gemm(x, w_gu, out, None, None, EPI_SWIGLU, 2 * block, False, False, 1, 0, 0)
    return out


def gram_acc(acc, x, y, k_chunk=8192):
    """acc [dx, dy] fp64 += x^T y for x [n, dx], y [n, dy] bf16 (row-major, read MN-major by the kernel).
    Rows are summed in fp32 within each k_chunk block and the blocks added in fp64."""
    n = x.shape[0]
    k_chunk = max(64, (k_chunk // 64) * 64)
    splits = max(1, (n + k_chunk - 1) // k_chunk)
    ext().gemm(x, y, acc, None, None, EPI_F64ACC, 256 if acc.shape[1] >= 256 else 128, True, True, splits,
               k_chunk if splits > 1 else 0, 0)
    return acc
