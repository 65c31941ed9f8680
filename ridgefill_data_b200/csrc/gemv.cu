// Products with at most 8 rows (a decode step's R sequences) as bandwidth-bound GEMVs.
//
// The tile GEMMs give such a product one 128- or 256-column tile per CTA, so a 5120-wide projection streams its
// weights through 20 SMs and a 27B decode step reads its 54 GB of weights far below HBM bandwidth (21 ms of device
// time for one sequence against an 8 ms floor). Here every warp owns 2 (1-2 rows) or 4 (3-8 rows) output columns (for
// SwiGLU, output features and their gate and up rows): its lanes stream those weight rows once in 16-byte pieces (non-allocating
// loads: the weights are read once) against the activation rows (read through L1, shared by the warp's columns), and
// the dot products are summed across the warp. 128-thread CTAs, as many as the columns need (thousands for the
// large projections), so every SM keeps enough loads in flight to stream at HBM rate without a persistent schedule.
// Epilogues as the tile GEMMs': kEpiStore (bf16, + bias[n], + residual[m, n]), kEpiSwiGLU (silu(gate) * up of the
// packed gate/up rows, blocks of `half` rows), kEpiF32 (fp32).
#include "gemm.h"
#include "kernels.h"

#include <cuda_bf16.h>

namespace rf {

namespace {

constexpr int kGemvThreads = 128;

__device__ __forceinline__ uint4 ld_stream(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ void to_f32x8(const uint4& v, float (&f)[8]) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 t = __bfloat1622float2(h[i]);
    f[2 * i] = t.x;
    f[2 * i + 1] = t.y;
  }
}

__device__ __forceinline__ float warp_sum_f(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

// MT: rows the kernel is compiled for (1, 2, 4, 8; rows >= M are skipped); EPI: epilogue; C: output columns per warp
// (the weight pieces are converted once per 16-byte step and reused by every row; each activation piece by every
// column). The k-steps of a lane's rows are summed in the order k, k + 256, k + 512, ...; the lanes' sums by a
// butterfly.
template <int MT, int EPI, int C>
__global__ void __launch_bounds__(kGemvThreads) gemv_kernel(const __nv_bfloat16* __restrict__ A, long lda,
                                                           const __nv_bfloat16* __restrict__ B, long ldb,
                                                           GemmArgs args, int half) {
  constexpr int NW = EPI == kEpiSwiGLU ? 2 * C : C;   // weight rows per warp
  const int warp = (blockIdx.x * kGemvThreads + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int M = args.M, K = args.K;
  const int n_out = EPI == kEpiSwiGLU ? args.N / 2 : args.N;
  const int c0 = warp * C;   // first output column of this warp
  if (c0 >= n_out) return;
  // weight rows: store / f32 -> columns c0 ..; SwiGLU -> the gate and up rows of features c0 ..
  const __nv_bfloat16* wrow[NW];
  bool wok[NW];
#pragma unroll
  for (int j = 0; j < C; ++j) {
    const int c = c0 + j;
    const bool ok = c < n_out;
    if constexpr (EPI == kEpiSwiGLU) {
      const int g = (c / half) * 2 * half + c % half;
      wrow[2 * j] = B + (long)(ok ? g : 0) * ldb;
      wrow[2 * j + 1] = B + (long)(ok ? g + half : 0) * ldb;
      wok[2 * j] = wok[2 * j + 1] = ok;
    } else {
      wrow[j] = B + (long)(ok ? c : 0) * ldb;
      wok[j] = ok;
    }
  }
  float acc[NW][MT];
#pragma unroll
  for (int j = 0; j < NW; ++j)
#pragma unroll
    for (int r = 0; r < MT; ++r) acc[j][r] = 0.f;
  const int k8 = K / 8;
#pragma unroll 2
  for (int kc = lane; kc < k8; kc += 32) {
    uint4 w[NW];
#pragma unroll
    for (int j = 0; j < NW; ++j) w[j] = wok[j] ? ld_stream(wrow[j] + 8 * kc) : make_uint4(0, 0, 0, 0);
    float wf[NW][8];
#pragma unroll
    for (int j = 0; j < NW; ++j) to_f32x8(w[j], wf[j]);
#pragma unroll
    for (int r = 0; r < MT; ++r) {
      if (r < M) {
        float xf[8];
        to_f32x8(__ldg(reinterpret_cast<const uint4*>(A + (long)r * lda + 8 * kc)), xf);
#pragma unroll
        for (int j = 0; j < NW; ++j)
#pragma unroll
          for (int e = 0; e < 8; ++e) acc[j][r] = fmaf(xf[e], wf[j][e], acc[j][r]);
      }
    }
  }
#pragma unroll
  for (int j = 0; j < NW; ++j)
#pragma unroll
    for (int r = 0; r < MT; ++r) acc[j][r] = warp_sum_f(acc[j][r]);
  // lane r * C + j writes output row r, column c0 + j
#pragma unroll
  for (int r = 0; r < MT; ++r) {
#pragma unroll
    for (int j = 0; j < C; ++j) {
      const int c = c0 + j;
      if (lane != (r * C + j) % 32 || r >= M || c >= n_out) continue;
      if constexpr (EPI == kEpiSwiGLU) {
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
        out[(long)r * args.ldo + c] = __float2bfloat16(silu_f(acc[2 * j][r]) * acc[2 * j + 1][r]);
      } else if constexpr (EPI == kEpiF32) {
        reinterpret_cast<float*>(args.out)[(long)r * args.ldo + c] = acc[j][r];
      } else {
        float v = acc[j][r];
        if (args.bias != nullptr) v += __bfloat162float(args.bias[c]);
        if (args.residual != nullptr) v += __bfloat162float(args.residual[(long)r * args.ldr + c]);
        reinterpret_cast<__nv_bfloat16*>(args.out)[(long)r * args.ldo + c] = __float2bfloat16(v);
      }
    }
  }
}

template <int MT, int C>
void launch_gemv(const GemmOperands& op, const GemmArgs& args, int epi, int half, cudaStream_t stream) {
  const int n_out = epi == kEpiSwiGLU ? args.N / 2 : args.N;
  const long warps = (n_out + C - 1) / C;
  const int blocks = (int)((warps * 32 + kGemvThreads - 1) / kGemvThreads);
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(op.A);
  const auto* B = reinterpret_cast<const __nv_bfloat16*>(op.B);
  if (epi == kEpiSwiGLU)
    gemv_kernel<MT, kEpiSwiGLU, C><<<blocks, kGemvThreads, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  else if (epi == kEpiF32)
    gemv_kernel<MT, kEpiF32, C><<<blocks, kGemvThreads, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  else
    gemv_kernel<MT, kEpiStore, C><<<blocks, kGemvThreads, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  count_launch();
}

}  // namespace

bool gemv_enabled = true;

// Rows routed here by default: 1-2. Measured on the 27B decode step (one B200, device time per token): 1 row 14.7 ms
// here against 22.8 ms on the tile GEMMs; 3 rows 29.0 against 28.9; 8 rows 61.3 against 44.0 (the FMAs of 8 rows per
// weight piece and the activation conversions then cost more than the tile GEMMs' idle SMs).
int gemv_max_rows = 2;

bool gemm_bf16_gemv(const GemmOperands& op, const GemmArgs& args, int epi, int bn, cudaStream_t stream) {
  if (!gemv_enabled || args.M < 1 || args.M > gemv_max_rows || args.M > 8 || op.a_mn || op.b_mn || args.k_splits != 1)
    return false;
  if (epi != kEpiStore && epi != kEpiSwiGLU && epi != kEpiF32) return false;
  if (args.K % 8 != 0 || op.lda % 8 != 0 || op.ldb % 8 != 0) return false;   // 16-byte pieces of every row
  if (reinterpret_cast<uintptr_t>(op.A) % 16 || reinterpret_cast<uintptr_t>(op.B) % 16) return false;
  const int half = bn / 2;
  if (epi == kEpiSwiGLU && (half <= 0 || args.N % (2 * half) != 0)) return false;
  if (args.M == 1) launch_gemv<1, 2>(op, args, epi, half, stream);
  else if (args.M == 2) launch_gemv<2, 2>(op, args, epi, half, stream);
  else if (args.M <= 4) launch_gemv<4, 4>(op, args, epi, half, stream);
  else launch_gemv<8, 4>(op, args, epi, half, stream);
  return true;
}

}  // namespace rf
