// fp64 ridge solve on the device: X = (A + shift I)^-1 B for symmetric positive definite A [n, n] and many
// right-hand sides B [n, R] (every late layer's cross-moments at once).
//
//  blocked right-looking Cholesky A = L L^T (block 64):
//    potrf_block   the 64 x 64 diagonal block factored in shared memory (one CTA)
//    trsm_panel    rows below: L_ij = A_ij L_jj^-T, one thread per row (forward substitution)
//    gemm_sub      trailing update A_ik -= L_ij L_kj^T (lower triangle), tiled fp64 FMA
//  forward solve L Y = B and backward solve L^T X = Y, blocked the same way:
//    trsm_rhs      the 64-row block of the right-hand sides through L_jj (or L_jj^T), one thread per column
//    gemm_sub      the rest of the right-hand sides updated with the solved block
// A non-positive pivot records kErrBadShape in the error word (the caller raises).
#include "kernels.h"
#include "ptx.cuh"

namespace rf {

constexpr int LB = 64;   // block size

// shift the diagonal and copy the lower triangle of A (row-major, lda) into L (in place allowed)
__global__ void shift_diag_kernel(double* a, int n, long lda, double shift) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i < n) a[(long)i * lda + i] += shift;
}

__global__ void potrf_block_kernel(double* a, int n, long lda, int j0, int* err) {
  __shared__ double s[LB][LB + 1];
  const int nb = min(LB, n - j0);
  for (int v = threadIdx.x; v < nb * nb; v += blockDim.x) s[v / nb][v % nb] = a[(long)(j0 + v / nb) * lda + j0 + v % nb];
  __syncthreads();
  for (int k = 0; k < nb; ++k) {
    if (threadIdx.x == 0) {
      const double d = s[k][k];
      if (!(d > 0.0)) {
        record_error(err, kErrBadShape);
        s[k][k] = 1.0;
      } else {
        s[k][k] = sqrt(d);
      }
    }
    __syncthreads();
    const double piv = s[k][k];
    for (int i = k + 1 + threadIdx.x; i < nb; i += blockDim.x) s[i][k] /= piv;
    __syncthreads();
    for (int v = threadIdx.x; v < (nb - k - 1) * (nb - k - 1); v += blockDim.x) {
      const int i = k + 1 + v / (nb - k - 1), j = k + 1 + v % (nb - k - 1);
      if (j <= i) s[i][j] -= s[i][k] * s[j][k];
    }
    __syncthreads();
  }
  for (int v = threadIdx.x; v < nb * nb; v += blockDim.x) {
    const int i = v / nb, j = v % nb;
    a[(long)(j0 + i) * lda + j0 + j] = j <= i ? s[i][j] : 0.0;
  }
}

// rows i >= j0 + nb: L[i, j0:j0+nb] = A[i, j0:j0+nb] L_jj^-T
__global__ void trsm_panel_kernel(double* a, int n, long lda, int j0) {
  __shared__ double l[LB][LB + 1];
  const int nb = min(LB, n - j0);
  for (int v = threadIdx.x; v < nb * nb; v += blockDim.x) l[v / nb][v % nb] = a[(long)(j0 + v / nb) * lda + j0 + v % nb];
  __syncthreads();
  const int i = j0 + nb + blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  double x[LB];
  double* row = a + (long)i * lda + j0;
  for (int j = 0; j < nb; ++j) {
    double v = row[j];
    for (int m = 0; m < j; ++m) v -= x[m] * l[j][m];
    x[j] = v / l[j][j];
  }
  for (int j = 0; j < nb; ++j) row[j] = x[j];
}

// C[M, N] -= A[M, K] B[K, N] with element strides (row, col) for each operand; lower: only C entries with
// (row0 + i) >= (col0 + j) (trailing Cholesky update). 64 x 64 tiles, 256 threads, 4 x 4 per thread.
struct DgemmArgs {
  int M, N, K;
  const double* A;
  long a_r, a_c;
  const double* B;
  long b_r, b_c;
  double* C;
  long c_r, c_c;
  int lower;
  long row_off, col_off;   // global indices of C's origin (for the lower test)
};

__global__ void __launch_bounds__(256) dgemm_sub_kernel(DgemmArgs g) {
  __shared__ double As[16][64 + 1];
  __shared__ double Bs[16][64 + 1];
  const int bm = blockIdx.y * 64, bn = blockIdx.x * 64;
  if (g.lower && (g.row_off + bm + 63) < (g.col_off + bn)) return;   // tile strictly above the diagonal
  const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
  double acc[4][4] = {};
  for (int k0 = 0; k0 < g.K; k0 += 16) {
    for (int v = threadIdx.x; v < 16 * 64; v += 256) {
      const int kk = v / 64, mm = v % 64;
      const int gm = bm + mm, gk = k0 + kk;
      As[kk][mm] = (gm < g.M && gk < g.K) ? g.A[(long)gm * g.a_r + (long)gk * g.a_c] : 0.0;
      const int gn = bn + mm;
      Bs[kk][mm] = (gn < g.N && gk < g.K) ? g.B[(long)gk * g.b_r + (long)gn * g.b_c] : 0.0;
    }
    __syncthreads();
#pragma unroll
    for (int kk = 0; kk < 16; ++kk) {
      double a[4], b[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) a[i] = As[kk][ty * 4 + i];
#pragma unroll
      for (int j = 0; j < 4; ++j) b[j] = Bs[kk][tx * 4 + j];
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) acc[i][j] = fma(a[i], b[j], acc[i][j]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int m = bm + ty * 4 + i;
    if (m >= g.M) continue;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int nn = bn + tx * 4 + j;
      if (nn >= g.N) continue;
      if (g.lower && g.row_off + m < g.col_off + nn) continue;
      g.C[(long)m * g.c_r + (long)nn * g.c_c] -= acc[i][j];
    }
  }
}

static void dgemm_sub(const DgemmArgs& g, cudaStream_t s) {
  if (g.M <= 0 || g.N <= 0 || g.K <= 0) return;
  dim3 grid((g.N + 63) / 64, (g.M + 63) / 64);
  dgemm_sub_kernel<<<grid, 256, 0, s>>>(g);
  count_launch();
}

// Right-hand sides: rows [j0, j0 + nb) of B [n, R] through L_jj (forward: solve L_jj Y = B) or its transpose
// (backward: solve L_jj^T X = Y); one thread per column.
__global__ void trsm_rhs_kernel(const double* l_mat, long lda, double* b, long ldb, int n, int R, int j0, int upper) {
  __shared__ double l[LB][LB + 1];
  const int nb = min(LB, n - j0);
  for (int v = threadIdx.x; v < nb * nb; v += blockDim.x) l[v / nb][v % nb] = l_mat[(long)(j0 + v / nb) * lda + j0 + v % nb];
  __syncthreads();
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= R) return;
  double x[LB];
  for (int j = 0; j < nb; ++j) x[j] = b[(long)(j0 + j) * ldb + c];
  if (!upper) {
    for (int j = 0; j < nb; ++j) {
      double v = x[j];
      for (int m = 0; m < j; ++m) v -= l[j][m] * x[m];
      x[j] = v / l[j][j];
    }
  } else {
    for (int j = nb - 1; j >= 0; --j) {
      double v = x[j];
      for (int m = j + 1; m < nb; ++m) v -= l[m][j] * x[m];
      x[j] = v / l[j][j];
    }
  }
  for (int j = 0; j < nb; ++j) b[(long)(j0 + j) * ldb + c] = x[j];
}

void cholesky_solve(double* a, int n, long lda, double shift, double* b, long ldb, int R, int* err,
                    cudaStream_t s) {
  if (n <= 0) return;
  shift_diag_kernel<<<(n + 255) / 256, 256, 0, s>>>(a, n, lda, shift);
  count_launch();
  for (int j0 = 0; j0 < n; j0 += LB) {
    const int nb = min(LB, n - j0);
    potrf_block_kernel<<<1, 256, 0, s>>>(a, n, lda, j0, err);
    const int rest = n - j0 - nb;
    count_launch();
    if (rest > 0) {
      trsm_panel_kernel<<<(rest + 127) / 128, 128, 0, s>>>(a, n, lda, j0);
      count_launch();
      // A[j0+nb:, j0+nb:] -= L[j0+nb:, j0:j0+nb] L[j0+nb:, j0:j0+nb]^T (lower)
      DgemmArgs g{rest, rest, nb, a + (long)(j0 + nb) * lda + j0, lda, 1, a + (long)(j0 + nb) * lda + j0, 1, lda,
                  a + (long)(j0 + nb) * lda + j0 + nb, lda, 1, 1, 0, 0};
      dgemm_sub(g, s);
    }
  }
  // forward: L Y = B
  for (int j0 = 0; j0 < n; j0 += LB) {
    const int nb = min(LB, n - j0);
    trsm_rhs_kernel<<<(R + 127) / 128, 128, 0, s>>>(a, lda, b, ldb, n, R, j0, 0);
    count_launch();
    const int rest = n - j0 - nb;
    if (rest > 0) {   // B[j0+nb:] -= L[j0+nb:, j0:j0+nb] Y[j0:j0+nb]
      DgemmArgs g{rest, R, nb, a + (long)(j0 + nb) * lda + j0, lda, 1, b + (long)j0 * ldb, ldb, 1,
                  b + (long)(j0 + nb) * ldb, ldb, 1, 0, 0, 0};
      dgemm_sub(g, s);
    }
  }
  // backward: L^T X = Y
  const int last = ((n - 1) / LB) * LB;
  for (int j0 = last; j0 >= 0; j0 -= LB) {
    trsm_rhs_kernel<<<(R + 127) / 128, 128, 0, s>>>(a, lda, b, ldb, n, R, j0, 1);
    count_launch();
    if (j0 > 0) {   // Y[:j0] -= L[j0:j0+nb, :j0]^T X[j0:j0+nb]
      const int nb = min(LB, n - j0);
      DgemmArgs g{j0, R, nb, a + (long)j0 * lda, 1, lda, b + (long)j0 * ldb, ldb, 1, b, ldb, 1, 0, 0, 0};
      dgemm_sub(g, s);
    }
  }
}

}  // namespace rf
