// One Gated DeltaNet decode token for R sequences in two launches per layer.
//
// Decode advances every sequence by one row. Run through the prefill kernels, that row costs four launches per
// sequence and layer: the prep kernel (conv, SiLU, l2norm, gates), the conv-state update, and the chunk scan's WY and
// state passes, the last two on a 64-row chunk that holds one live row. Here:
//
// gdn_decode_step_kernel   grid (value head, sequence), 256 threads. The CTA computes the conv + SiLU of its key
//                          head's q and k channels and its value head's v channels from the sequence's conv state
//                          (K - 1 previous rows, oldest first) and the new in-projection row; q and k are
//                          l2-normalised (q times dk^-0.5) and, like v, rounded to bf16 as the prep kernel stores
//                          them; beta = sigmoid(b) (rounded to bf16), g = -exp(A_log) softplus(a + dt_bias). Then the
//                          recurrent step of the delta rule on the fp32 state S [dk, dv] of the value head:
//                          S <- e^g S;  S <- S + k ((v - S^T k) beta)^T;  o = S^T q.
//                          Thread (p, j) keeps rows [p RPT, (p + 1) RPT) of state column j in registers (P = 256 / dv
//                          row parts of RPT rows); the column sums S^T k and S^T q are added over the parts in part
//                          order through shared memory.
// gdn_decode_conv_kernel   the conv states move one row on: rows 1 .. K - 2 up, the new row last (one thread per
//                          channel). It runs after the step kernel, because the q and k channels of a key head are
//                          read by the CTAs of all its value heads.
//
// States are read from `*_src` and written to `*_dst` (the same pointers for an in-place update; each thread reads
// every element it writes first). The sequences' pointers travel in the kernel arguments (up to kDecodeSeqs per
// launch), so a CUDA graph of the step holds them and nothing is copied to the device per step. The arithmetic is
// the oracle's token-by-token form (code/kva/ops.py's recurrent definition of the gated delta rule); every row of
// a batch is computed alike whatever the batch, so a batched decode row equals its single-sequence step bitwise.
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <stdexcept>

namespace rf {

namespace {

constexpr int kDecodeThreads = 256;

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16(x)); }
__device__ __forceinline__ float softplus_d(float x) { return x > 20.f ? x : log1pf(expf(x)); }

template <int DK, int DV>
__global__ void __launch_bounds__(kDecodeThreads) gdn_decode_step_kernel(GdnDecodeArgs a, int r0) {
  constexpr int P = kDecodeThreads / DV;   // row parts of a state column
  constexpr int RPT = DK / P;              // state rows per thread
  static_assert(P * DV == kDecodeThreads && RPT * P == DK, "state split");
  __shared__ float ys[2 * DK + DV];        // conv + SiLU outputs: q | k | v
  __shared__ float qs[DK], ks[DK];
  __shared__ float red_kv[P][DV], red_o[P][DV];
  __shared__ float gate[2];                // beta, e^g
  const int h = blockIdx.x, r = blockIdx.y + r0;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int kh = h / (a.nv / a.nk);
  const int C = 2 * a.nk * DK + a.nv * DV;
  const int K1 = a.K - 1;
  const __nv_bfloat16* prow = a.proj + (long)r * a.proj_row;
  const __nv_bfloat16* cst = a.conv_src[blockIdx.y];
  for (int i = tid; i < 2 * DK + DV; i += kDecodeThreads) {
    const int ch = i < DK ? kh * DK + i
                 : i < 2 * DK ? a.nk * DK + kh * DK + (i - DK)
                 : 2 * a.nk * DK + h * DV + (i - 2 * DK);
    const __nv_bfloat16* w = a.conv_w + (long)ch * a.K;
    float acc = 0.f;
    for (int tap = 0; tap < K1; ++tap) acc += __bfloat162float(cst[(long)tap * C + ch]) * __bfloat162float(w[tap]);
    acc += __bfloat162float(prow[ch]) * __bfloat162float(w[K1]);
    ys[i] = bf16_round(acc / (1.f + __expf(-acc)));
  }
  if (tid == 0) {
    const float b = __bfloat162float(prow[a.b_off + h]);
    const float av = __bfloat162float(prow[a.a_off + h]);
    gate[0] = bf16_round(1.f / (1.f + expf(-b)));
    gate[1] = expf(-expf(a.A_log[h]) * softplus_d(av + a.dt_bias[h]));
  }
  __syncthreads();
  if (warp < 2) {   // warp 0: q, warp 1: k; channel lane + 32 j, squares summed over j, then across the warp
    const float* y = ys + warp * DK;
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < DK / 32; ++j) ss += y[j * 32 + lane] * y[j * 32 + lane];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
    const float scale = rsqrtf(ss + 1e-6f) * (warp == 0 ? rsqrtf((float)DK) : 1.f);
    float* dst = warp == 0 ? qs : ks;
#pragma unroll
    for (int j = 0; j < DK / 32; ++j) dst[j * 32 + lane] = bf16_round(y[j * 32 + lane] * scale);
  }
  __syncthreads();
  const int j = tid % DV, p = tid / DV;
  const float beta = gate[0], decay = gate[1];
  const float* src = a.rec_src[blockIdx.y] + (long)h * DK * DV + (long)p * RPT * DV + j;
  float* dst = a.rec_dst[blockIdx.y] + (long)h * DK * DV + (long)p * RPT * DV + j;
  float s[RPT];
#pragma unroll
  for (int i = 0; i < RPT; ++i) s[i] = src[(long)i * DV] * decay;
  float kv = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; ++i) kv = fmaf(s[i], ks[p * RPT + i], kv);
  red_kv[p][j] = kv;
  __syncthreads();
  kv = 0.f;
#pragma unroll
  for (int q = 0; q < P; ++q) kv += red_kv[q][j];
  const float corr = (ys[2 * DK + j] - kv) * beta;
  float o = 0.f;
#pragma unroll
  for (int i = 0; i < RPT; ++i) {
    s[i] = fmaf(ks[p * RPT + i], corr, s[i]);
    o = fmaf(s[i], qs[p * RPT + i], o);
    dst[(long)i * DV] = s[i];
  }
  red_o[p][j] = o;
  __syncthreads();
  if (p == 0) {
    o = 0.f;
#pragma unroll
    for (int q = 0; q < P; ++q) o += red_o[q][j];
    a.out[(long)r * a.out_row + (long)h * DV + j] = __float2bfloat16(o);
  }
}

template <int K1>
__global__ void gdn_decode_conv_kernel(GdnDecodeArgs a, int r0, int C) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  const __nv_bfloat16* src = a.conv_src[blockIdx.y];
  __nv_bfloat16* dst = a.conv_dst[blockIdx.y];
  __nv_bfloat16 tmp[K1];
#pragma unroll
  for (int i = 0; i + 1 < K1; ++i) tmp[i] = src[(long)(i + 1) * C + c];
  tmp[K1 - 1] = a.proj[(long)(blockIdx.y + r0) * a.proj_row + c];
#pragma unroll
  for (int i = 0; i < K1; ++i) dst[(long)i * C + c] = tmp[i];
}

}  // namespace

bool gdn_decode_supported(int dk, int dv, int K) { return dk == 128 && dv == 128 && K >= 2 && K <= 8; }

void gdn_decode_step(const GdnDecodeArgs& a, int r0, int rows, cudaStream_t stream) {
  if (rows <= 0) return;
  if (rows > kDecodeSeqs || !gdn_decode_supported(a.dk, a.dv, a.K) || a.nv % a.nk != 0)
    throw std::runtime_error("gdn_decode_step: unsupported shape");
  const int C = 2 * a.nk * a.dk + a.nv * a.dv;
  gdn_decode_step_kernel<128, 128><<<dim3(a.nv, rows), kDecodeThreads, 0, stream>>>(a, r0);
  count_launch();
  const dim3 grid((C + 255) / 256, rows);
  switch (a.K - 1) {
    case 1: gdn_decode_conv_kernel<1><<<grid, 256, 0, stream>>>(a, r0, C); break;
    case 2: gdn_decode_conv_kernel<2><<<grid, 256, 0, stream>>>(a, r0, C); break;
    case 3: gdn_decode_conv_kernel<3><<<grid, 256, 0, stream>>>(a, r0, C); break;
    case 4: gdn_decode_conv_kernel<4><<<grid, 256, 0, stream>>>(a, r0, C); break;
    case 5: gdn_decode_conv_kernel<5><<<grid, 256, 0, stream>>>(a, r0, C); break;
    case 6: gdn_decode_conv_kernel<6><<<grid, 256, 0, stream>>>(a, r0, C); break;
    default: gdn_decode_conv_kernel<7><<<grid, 256, 0, stream>>>(a, r0, C); break;
  }
  count_launch();
}

}  // namespace rf
