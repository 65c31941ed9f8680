// Products with at most 16 rows (a decode step's R sequences) as bandwidth-bound GEMVs.
//
// The tile GEMMs give such a product one 128- or 256-column tile per CTA, so a 5120-wide projection streams its
// weights through 20 SMs and a 27B decode step reads its 54 GB of weights far below HBM bandwidth (21 ms of device
// time for one sequence against an 8 ms floor). Two kernels here stream the weights once through every SM instead.
//
// gemv_mma_kernel (the default, 1-16 rows): the roles of the operands are swapped so the tensor cores see a full
// 16-row A operand whatever the row count: a CTA owns 16 output columns (SwiGLU: 16 features, that is 16 gate and
// 16 up weight rows), their weight rows are the A operand of mma.m16n8k16 (bf16 in, fp32 accumulate) and the
// activation rows are the 8-column B operand (one n-tile for 1-8 rows, two for 9-16). The k order inside each
// 32-wide k block is permuted alike in A and B so that every lane reads whole 16-byte pieces: lane (g = lane / 4,
// t = lane % 4) loads k 8t .. 8t + 7 of weight rows g and g + 8 and of activation row g, and the two k16 steps of
// the block take words {0, 1} and {2, 3} of those pieces. The 8 warps of a CTA take the k blocks in turn (warp w:
// blocks w, w + 8, ...) and their partial sums are added in warp order through shared memory. A row's result
// therefore depends on nothing but its own activations and the weights: the same bits for 1 row or 16, whichever
// rows it is batched with (batch-invariant decode). The instruction is the warp-level mma: the kernel is bound by
// the weight stream (16 weight rows x 32 k per pair of MMAs), not by the tensor pipe.
//
// gemv_kernel (1-8 rows, the CUDA-core form kept as the A/B alternative): every warp owns 2 (1-2 rows) or 4 (3-8
// rows) output columns (for SwiGLU, output features and their gate and up rows): its lanes stream those weight rows
// once in 16-byte pieces against the activation rows, and the dot products are summed across the warp.
//
// Weights are read with non-allocating loads (read once), activations through L1 (shared by a CTA's columns).
// Epilogues as the tile GEMMs': kEpiStore (bf16, + bias[n], + residual[m, n]), kEpiSwiGLU (silu(gate) * up of the
// packed gate/up rows, blocks of `half` rows), kEpiF32 (fp32).
#include "gemm.h"
#include "kernels.h"

#include "mma.cuh"

#include <algorithm>
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

constexpr int kMmaWarps = 8;

__device__ __forceinline__ uint32_t word_of(const uint4& v, int i) {
  return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w;
}

// NF: activation n-tiles (1: rows 1-8, 2: rows 9-16; rows >= M read as zeros); EPI: epilogue; U: k blocks a warp
// loads before it multiplies (8 weight pieces of 16 bytes in flight per lane for both U = 4 with one weight tile
// and U = 2 with the two of SwiGLU).
template <int NF, int EPI, int U>
__global__ void __launch_bounds__(kMmaWarps * 32) gemv_mma_kernel(const __nv_bfloat16* __restrict__ A, long lda,
                                                                 const __nv_bfloat16* __restrict__ B, long ldb,
                                                                 GemmArgs args, int half) {
  constexpr int NA = EPI == kEpiSwiGLU ? 2 : 1;   // weight tiles of 16 rows (SwiGLU: gate, up)
  __shared__ float red[kMmaWarps][NA * NF * 4][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int g = lane >> 2, t = lane & 3;
  const int M = args.M, K = args.K;
  const int n_out = EPI == kEpiSwiGLU ? args.N / 2 : args.N;
  const int c0 = blockIdx.x * 16;
  // every address a lane forms lies inside the operands, skipped loads included: the lane's column offset is at
  // most K - 8 (a lane that ever loads has 8 t < K, so the offset is then 8 t) and a skipped block reads offset 0
  const int t8 = min(8 * t, K - 8);
  const __nv_bfloat16* wp[NA][2];
  bool wok[NA][2];
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const int c = c0 + g + 8 * h;
      const bool ok = c < n_out;
      int row = c;
      if constexpr (EPI == kEpiSwiGLU) row = (c / half) * 2 * half + c % half + a * half;
      wp[a][h] = B + (long)(ok ? row : 0) * ldb + t8;
      wok[a][h] = ok;
    }
  const __nv_bfloat16* xp[NF];
  bool xok[NF];
#pragma unroll
  for (int f = 0; f < NF; ++f) {
    const int m = g + 8 * f;
    xok[f] = m < M;
    xp[f] = A + (long)(xok[f] ? m : 0) * lda + t8;
  }
  float acc[NA][NF][4];
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int f = 0; f < NF; ++f)
#pragma unroll
      for (int r = 0; r < 4; ++r) acc[a][f][r] = 0.f;
  const uint4 zero = make_uint4(0, 0, 0, 0);
  const int nb = (K + 31) / 32;   // k blocks of 32
  for (int b0 = warp; b0 < nb; b0 += kMmaWarps * U) {
    uint4 wv[U][NA][2], xv[U][NF];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int b = b0 + u * kMmaWarps;
      const bool in = b < nb && b * 32 + 8 * t < K;   // K % 8 == 0: whole pieces
      const long off = in ? (long)b * 32 : 0;
#pragma unroll
      for (int a = 0; a < NA; ++a)
#pragma unroll
        for (int h = 0; h < 2; ++h) wv[u][a][h] = in && wok[a][h] ? ld_stream(wp[a][h] + off) : zero;
#pragma unroll
      for (int f = 0; f < NF; ++f)
        xv[u][f] = in && xok[f] ? __ldg(reinterpret_cast<const uint4*>(xp[f] + off)) : zero;
    }
#pragma unroll
    for (int u = 0; u < U; ++u)
#pragma unroll
      for (int s = 0; s < 2; ++s)
#pragma unroll
        for (int a = 0; a < NA; ++a) {
          const uint32_t ar[4] = {word_of(wv[u][a][0], 2 * s), word_of(wv[u][a][1], 2 * s),
                                  word_of(wv[u][a][0], 2 * s + 1), word_of(wv[u][a][1], 2 * s + 1)};
#pragma unroll
          for (int f = 0; f < NF; ++f) mma_bf16(acc[a][f], ar, word_of(xv[u][f], 2 * s), word_of(xv[u][f], 2 * s + 1));
        }
  }
#pragma unroll
  for (int a = 0; a < NA; ++a)
#pragma unroll
    for (int f = 0; f < NF; ++f)
#pragma unroll
      for (int r = 0; r < 4; ++r) red[warp][(a * NF + f) * 4 + r][lane] = acc[a][f][r];
  __syncthreads();
  // accumulator element r of lane l in n-tile f: weight row (output column) c0 + l / 4 + 8 (r / 2), activation row
  // 8 f + 2 (l % 4) + r % 2
  for (int i = threadIdx.x; i < NF * 4 * 32; i += kMmaWarps * 32) {
    const int l = i & 31, f = i >> 7, r = (i >> 5) & 3;
    const int c = c0 + (l >> 2) + 8 * (r >> 1);
    const int m = 8 * f + 2 * (l & 3) + (r & 1);
    if (m >= M || c >= n_out) continue;
    float v[NA];
#pragma unroll
    for (int a = 0; a < NA; ++a) {
      float sum = 0.f;
#pragma unroll
      for (int w = 0; w < kMmaWarps; ++w) sum += red[w][(a * NF + f) * 4 + r][l];
      v[a] = sum;
    }
    if constexpr (EPI == kEpiSwiGLU) {
      reinterpret_cast<__nv_bfloat16*>(args.out)[(long)m * args.ldo + c] = __float2bfloat16(silu_f(v[0]) * v[NA - 1]);
    } else if constexpr (EPI == kEpiF32) {
      reinterpret_cast<float*>(args.out)[(long)m * args.ldo + c] = v[0];
    } else {
      float o = v[0];
      if (args.bias != nullptr) o += __bfloat162float(args.bias[c]);
      if (args.residual != nullptr) o += __bfloat162float(args.residual[(long)m * args.ldr + c]);
      reinterpret_cast<__nv_bfloat16*>(args.out)[(long)m * args.ldo + c] = __float2bfloat16(o);
    }
  }
}

template <int NF>
void launch_gemv_mma(const GemmOperands& op, const GemmArgs& args, int epi, int half, cudaStream_t stream) {
  const int n_out = epi == kEpiSwiGLU ? args.N / 2 : args.N;
  const int blocks = (n_out + 15) / 16;
  const auto* A = reinterpret_cast<const __nv_bfloat16*>(op.A);
  const auto* B = reinterpret_cast<const __nv_bfloat16*>(op.B);
  if (epi == kEpiSwiGLU)
    gemv_mma_kernel<NF, kEpiSwiGLU, 2><<<blocks, kMmaWarps * 32, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  else if (epi == kEpiF32)
    gemv_mma_kernel<NF, kEpiF32, 4><<<blocks, kMmaWarps * 32, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  else
    gemv_mma_kernel<NF, kEpiStore, 4><<<blocks, kMmaWarps * 32, 0, stream>>>(A, op.lda, B, op.ldb, args, half);
  count_launch();
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
bool gemv_mma = true;

// Rows routed here by default: 1-16, all on the tensor-core kernel (one summation order for every row count).
// Measured on the 27B decode step with the CUDA-core kernel (one B200, device time per token): 1 row 14.7 ms here
// against 22.8 ms on the tile GEMMs; 3 rows 29.0 against 28.9; 8 rows 61.3 against 44.0 (the FMAs of 8 rows per
// weight piece and the activation conversions then cost more than the tile GEMMs' idle SMs), which is why that
// kernel takes at most 8 rows, and by default (set_gemv_mma(false)) 1-2.
int gemv_max_rows = 16;

bool gemm_bf16_gemv(const GemmOperands& op, const GemmArgs& args, int epi, int bn, cudaStream_t stream) {
  const int cap = std::min(gemv_max_rows, gemv_mma ? 16 : 8);
  if (!gemv_enabled || args.M < 1 || args.M > cap || op.a_mn || op.b_mn || args.k_splits != 1) return false;
  if (epi != kEpiStore && epi != kEpiSwiGLU && epi != kEpiF32) return false;
  if (args.K % 8 != 0 || op.lda % 8 != 0 || op.ldb % 8 != 0) return false;   // 16-byte pieces of every row
  if (reinterpret_cast<uintptr_t>(op.A) % 16 || reinterpret_cast<uintptr_t>(op.B) % 16) return false;
  const int half = bn / 2;
  if (epi == kEpiSwiGLU && (half <= 0 || args.N % (2 * half) != 0)) return false;
  if (gemv_mma) {
    if (epi == kEpiSwiGLU && half % 16 != 0) return false;   // a CTA's 16 features inside one gate / up block
    if (args.M <= 8) launch_gemv_mma<1>(op, args, epi, half, stream);
    else launch_gemv_mma<2>(op, args, epi, half, stream);
    return true;
  }
  if (args.M == 1) launch_gemv<1, 2>(op, args, epi, half, stream);
  else if (args.M == 2) launch_gemv<2, 2>(op, args, epi, half, stream);
  else if (args.M <= 4) launch_gemv<4, 4>(op, args, epi, half, stream);
  else launch_gemv<8, 4>(op, args, epi, half, stream);
  return true;
}

}  // namespace rf
