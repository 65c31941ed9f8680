// Small reductions of the fit and the selectors.
//
//  row_cosine    cosine similarity of every row pair of two [rows][d] bf16 tensors (one warp per row, fp32):
//                the held-out read cosine of the lambda selection (code/scripts/fit_sweep.py:301-318)
//  window_mass   attention mass the last w query rows give every key, summed over query heads and window rows,
//                causal (key j visible to the query at position p when j <= p) (code/kva/select.py:223-244):
//                pass 1 scores each 64-key block against every window query on the tensor cores and keeps the
//                block's running max and exp-sum per query; a combine step gives each query its softmax
//                normaliser; pass 2 recomputes the scores and sums exp(s - m) / l down each key column, the
//                column sums of the 4 warps meet in shared memory and every block adds its 64 masses into the
//                fp64 output (one add per key per KV head).
#include "kernels.h"
#include "mma.cuh"
#include "ptx.cuh"

#include <cfloat>

namespace rf {

__global__ void row_cosine_kernel(const __nv_bfloat16* a, long lda, const __nv_bfloat16* b, long ldb, long rows, int d,
                                  float eps, float* out) {
  const long r = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
  const int lane = threadIdx.x & 31;
  if (r >= rows) return;
  const __nv_bfloat16* x = a + r * lda;
  const __nv_bfloat16* y = b + r * ldb;
  float xy = 0.f, xx = 0.f, yy = 0.f;
  for (int c = lane; c < d; c += 32) {
    const float u = __bfloat162float(x[c]), v = __bfloat162float(y[c]);
    xy = fmaf(u, v, xy);
    xx = fmaf(u, u, xx);
    yy = fmaf(v, v, yy);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    xy += __shfl_xor_sync(0xffffffffu, xy, o);
    xx += __shfl_xor_sync(0xffffffffu, xx, o);
    yy += __shfl_xor_sync(0xffffffffu, yy, o);
  }
  if (lane == 0) out[r] = xy / sqrtf(fmaxf(xx * yy, eps * eps));
}

void row_cosine(const __nv_bfloat16* a, long lda, const __nv_bfloat16* b, long ldb, long rows, int d, float eps,
                float* out, cudaStream_t stream) {
  if (rows <= 0) return;
  row_cosine_kernel<<<(unsigned)((rows + 7) / 8), 256, 0, stream>>>(a, lda, b, ldb, rows, d, eps, out);
  count_launch();
}

// ------------------------------------------------------------------------------------------ window mass
constexpr int WM_KEYS = 64;       // keys per block
constexpr int WM_Q = 64;          // window query rows per pass over the block (4 warps x 16)

struct WmSmem {
  __nv_bfloat16 k[WM_KEYS * (256 + 8)];
  __nv_bfloat16 q[WM_Q * (256 + 8)];
  float col[WM_KEYS];
};

// Scores of this warp's 16 query rows (rows r0.. of the staged Q chunk) against the 64 staged keys:
// s[j][0..3] = C fragment of n-tile j (keys 8j + 2t, +1; rows g, g + 8).
__device__ __forceinline__ void wm_scores(float (&s)[8][4], const WmSmem& sm, int pitch, int hd, int r0, int lane) {
#pragma unroll
  for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
  for (int k0 = 0; k0 < hd; k0 += 16) {
    uint32_t a[4];
    lda_row(a, sm.q, pitch, r0, k0, lane);
#pragma unroll
    for (int j2 = 0; j2 < 4; ++j2) {
      uint32_t b[4];
      ldb_nk(b, sm.k, pitch, j2 * 16, k0, lane);
      mma_bf16(s[2 * j2], a, b[0], b[1]);
      mma_bf16(s[2 * j2 + 1], a, b[2], b[3]);
    }
  }
}

template <int PASS>
__global__ void __launch_bounds__(128) window_mass_kernel(WindowMassArgs a) {
  extern __shared__ __align__(16) uint8_t wm_raw[];
  WmSmem& sm = *reinterpret_cast<WmSmem*>(wm_raw);
  const int blk = blockIdx.x, gh = blockIdx.y;           // key block, KV head
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, g = lane >> 2, t = lane & 3;
  const int pitch = a.hd + 8;
  const int key0 = blk * WM_KEYS;
  const int nblk = (a.n + WM_KEYS - 1) / WM_KEYS;
  const int rep = a.hq / a.hkv;
  const int nq = rep * a.w;                               // window queries of this KV head
  // stage the key block (zero rows past n)
  for (int v = tid; v < WM_KEYS * (a.hd / 8); v += 128) {
    const int r = v / (a.hd / 8), c = (v % (a.hd / 8)) * 8;
    const bool ok = key0 + r < a.n;
    uint4 x = make_uint4(0, 0, 0, 0);
    if (ok) x = *reinterpret_cast<const uint4*>(a.k + gh * a.k_head_stride + (long)(key0 + r) * a.k_row_stride + c);
    *reinterpret_cast<uint4*>(&sm.k[r * pitch + c]) = x;
  }
  if (PASS == 2)
    for (int v = tid; v < WM_KEYS; v += 128) sm.col[v] = 0.f;
  for (int qb = 0; qb < nq; qb += WM_Q) {
    __syncthreads();
    for (int v = tid; v < WM_Q * (a.hd / 8); v += 128) {
      const int r = v / (a.hd / 8), c = (v % (a.hd / 8)) * 8;
      const int qi = qb + r;
      uint4 x = make_uint4(0, 0, 0, 0);
      if (qi < nq) {
        const int hh = gh * rep + qi / a.w, wr = qi % a.w;
        x = *reinterpret_cast<const uint4*>(a.q + hh * a.q_head_stride + (long)wr * a.q_row_stride + c);
      }
      *reinterpret_cast<uint4*>(&sm.q[r * pitch + c]) = x;
    }
    __syncthreads();
    float s[8][4];
    wm_scores(s, sm, pitch, a.hd, warp * 16, lane);
    // the two query rows of this thread
    int qrow[2], qpos[2];
    bool qok[2];
#pragma unroll
    for (int h2 = 0; h2 < 2; ++h2) {
      const int qi = qb + warp * 16 + g + 8 * h2;
      qok[h2] = qi < nq;
      qrow[h2] = qok[h2] ? (gh * rep + qi / a.w) * a.w + qi % a.w : 0;   // global window-query index
      qpos[h2] = qok[h2] ? a.qpos[qi % a.w] : -1;
    }
    if constexpr (PASS == 1) {
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        float m = -FLT_MAX;
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = key0 + j * 8 + 2 * t + e;
            if (key < a.n && key <= qpos[h2]) m = fmaxf(m, s[j][2 * h2 + e] * a.scale);
          }
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 1));
        m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, 2));
        float l = 0.f;
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = key0 + j * 8 + 2 * t + e;
            if (key < a.n && key <= qpos[h2]) l += __expf(s[j][2 * h2 + e] * a.scale - m);
          }
        l += __shfl_xor_sync(0xffffffffu, l, 1);
        l += __shfl_xor_sync(0xffffffffu, l, 2);
        if (t == 0 && qok[h2]) {
          a.part_m[(long)qrow[h2] * nblk + blk] = l > 0.f ? m : -FLT_MAX;
          a.part_l[(long)qrow[h2] * nblk + blk] = l;
        }
      }
    } else {
      float col[8][2];
#pragma unroll
      for (int j = 0; j < 8; ++j) col[j][0] = col[j][1] = 0.f;
#pragma unroll
      for (int h2 = 0; h2 < 2; ++h2) {
        if (!qok[h2]) continue;
        const float m = a.qm[qrow[h2]], inv = 1.f / a.ql[qrow[h2]];
#pragma unroll
        for (int j = 0; j < 8; ++j)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int key = key0 + j * 8 + 2 * t + e;
            if (key < a.n && key <= qpos[h2]) col[j][e] += __expf(s[j][2 * h2 + e] * a.scale - m) * inv;
          }
      }
      // sum the 8 row groups (lanes with the same t) of the warp, then the warps in shared memory
#pragma unroll
      for (int j = 0; j < 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          float v = col[j][e];
          v += __shfl_xor_sync(0xffffffffu, v, 4);
          v += __shfl_xor_sync(0xffffffffu, v, 8);
          v += __shfl_xor_sync(0xffffffffu, v, 16);
          if (g == 0) atomicAdd(&sm.col[j * 8 + 2 * t + e], v);
        }
    }
  }
  if constexpr (PASS == 2) {
    __syncthreads();
    for (int v = tid; v < WM_KEYS; v += 128)
      if (key0 + v < a.n) atomicAdd(a.mass + key0 + v, (double)sm.col[v]);
  }
}

__global__ void window_mass_combine_kernel(WindowMassArgs a, int nq_total, int nblk) {
  const int qi = blockIdx.x * blockDim.x + threadIdx.x;
  if (qi >= nq_total) return;
  float m = -FLT_MAX;
  for (int b = 0; b < nblk; ++b) m = fmaxf(m, a.part_m[(long)qi * nblk + b]);
  float l = 0.f;
  for (int b = 0; b < nblk; ++b) {
    const float lb = a.part_l[(long)qi * nblk + b];
    if (lb > 0.f) l += lb * __expf(a.part_m[(long)qi * nblk + b] - m);
  }
  a.qm[qi] = m;
  a.ql[qi] = l > 0.f ? l : 1.f;
}

void window_mass(const WindowMassArgs& a, cudaStream_t stream) {
  if (a.n <= 0 || a.w <= 0) return;
  static PerDeviceOnce once;
  once([] {
    cudaFuncSetAttribute(window_mass_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(WmSmem));
    cudaFuncSetAttribute(window_mass_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(WmSmem));
  });
  const int nblk = (a.n + WM_KEYS - 1) / WM_KEYS;
  const dim3 grid(nblk, a.hkv);
  window_mass_kernel<1><<<grid, 128, sizeof(WmSmem), stream>>>(a);
  const int nq_total = a.hq * a.w;
  window_mass_combine_kernel<<<(nq_total + 127) / 128, 128, 0, stream>>>(a, nq_total, nblk);
  window_mass_kernel<2><<<grid, 128, sizeof(WmSmem), stream>>>(a);
  count_launch(3);
}

}  // namespace rf
