// Mixture-of-experts on sm_100a.
//
//  router_topk     one warp per token: softmax over the expert logits (fp32), top-k by repeated warp arg-max
//                  (ties to the lower index), weights renormalised to sum to one
//  moe_count       per (token, slot): atomic rank of the slot inside its expert's segment
//  moe_scan        one CTA: segment starts and cumulative 128-row tile counts per expert
//  moe_scatter     per (token, slot): position in the expert-sorted buffer, and the token's row copied there
//  grouped GEMM    persistent tcgen05 GEMM over every (expert, 128-row tile, N tile): A = the expert-sorted rows
//                  (2-D tensor map), B = all experts' weights through one 3-D tensor map [E][N][K]; tiles are
//                  decoded on the device from the cumulative tile counts (no host sync). Epilogues: SwiGLU
//                  (gate/up interleaved per 128-row block) or a plain bf16 store; rows past the expert's segment
//                  are masked
//  moe_combine     out[t] = h[t] + sum_k w[t, k] y[pos[t, k]] + sigmoid(g[t]) ys[t]   (fp32, one rounding)
// A row's product never depends on where its expert's segment lies, so results are identical run to run even
// though the atomic ranks (segment order) vary.
#include "gemm.h"
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace rf {

// ---------------------------------------------------------------------------------------- router
__global__ void router_topk_kernel(const float* __restrict__ logits, long ld, int n, int E, int k,
                                   int* __restrict__ idx, float* __restrict__ wts, int norm) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  if (warp >= n) return;
  const float* row = logits + (long)warp * ld;
  constexpr int MAXV = 32;   // E <= 1024
  float v[MAXV];
  const int per = (E + 31) / 32;
  float mx = -INFINITY;
  for (int j = 0; j < per; ++j) {
    const int e = lane + 32 * j;
    v[j] = e < E ? row[e] : -INFINITY;
    mx = fmaxf(mx, v[j]);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  float sum = 0.f;
  for (int j = 0; j < per; ++j) {
    v[j] = lane + 32 * j < E ? expf(v[j] - mx) : 0.f;
    sum += v[j];
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o);
  const float inv = 1.f / sum;
  float picked_sum = 0.f;
  float picked[16];
  int pidx[16];
  for (int s = 0; s < k; ++s) {
    float best = -1.f;
    int bi = 0x7fffffff;
    for (int j = 0; j < per; ++j) {
      const int e = lane + 32 * j;
      const float p = v[j] * inv;
      if (e < E && (p > best || (p == best && e < bi))) {
        best = p;
        bi = e;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ob = __shfl_xor_sync(0xffffffffu, best, o);
      const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (ob > best || (ob == best && oi < bi)) {
        best = ob;
        bi = oi;
      }
    }
    if (s < 16) {
      picked[s] = best;
      pidx[s] = bi;
    }
    picked_sum += best;
    if ((bi & 31) == lane) v[bi >> 5] = -1.f;   // owner lane removes the expert
  }
  if (lane == 0) {
    const float r = norm ? 1.f / picked_sum : 1.f;
    for (int s = 0; s < k && s < 16; ++s) {
      idx[(long)warp * k + s] = pidx[s];
      wts[(long)warp * k + s] = picked[s] * r;
    }
  }
}

void router_topk(const float* logits, long ld, int n, int E, int k, int* idx, float* wts, int norm,
                 cudaStream_t stream) {
  if (n <= 0) return;
  router_topk_kernel<<<(n * 32 + 255) / 256, 256, 0, stream>>>(logits, ld, n, E, k, idx, wts, norm);
  count_launch();
}

// ---------------------------------------------------------------------------------------- align
__global__ void moe_count_kernel(const int* __restrict__ idx, int nk, int e0, int E, int* __restrict__ counts,
                                 int* __restrict__ rank) {
  const int i = blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= nk) return;
  const int e = idx[i] - e0;
  rank[i] = (e >= 0 && e < E) ? atomicAdd(&counts[e], 1) : -1;
}

// one CTA of 1024 threads: exclusive scans of counts and of ceil(counts / 128)
__global__ void moe_scan_kernel(const int* __restrict__ counts, int E, int* __restrict__ seg_start,
                                int* __restrict__ tile_start) {
  __shared__ int sc[1024], st[1024];
  const int t = threadIdx.x;
  int c = 0, tc = 0;
  const int per = (E + 1023) / 1024;   // experts per thread (E <= 4096)
  for (int j = 0; j < per; ++j) {
    const int e = t * per + j;
    if (e < E) {
      c += counts[e];
      tc += (counts[e] + 127) / 128;
    }
  }
  sc[t] = c;
  st[t] = tc;
  __syncthreads();
  for (int o = 1; o < 1024; o <<= 1) {
    int a = t >= o ? sc[t - o] : 0, b = t >= o ? st[t - o] : 0;
    __syncthreads();
    sc[t] += a;
    st[t] += b;
    __syncthreads();
  }
  int run_c = sc[t] - c, run_t = st[t] - tc;
  for (int j = 0; j < per; ++j) {
    const int e = t * per + j;
    if (e < E) {
      seg_start[e] = run_c;
      tile_start[e] = run_t;
      run_c += counts[e];
      run_t += (counts[e] + 127) / 128;
    }
  }
  if (t == 1023) {
    seg_start[E] = sc[1023];
    tile_start[E] = st[1023];
  }
}

// grid: one CTA per (token, slot); copies the token's row to its expert-sorted position
__global__ void moe_scatter_kernel(const int* __restrict__ idx, const int* __restrict__ rank,
                                   const int* __restrict__ seg_start, int k, int e0, int* __restrict__ pos,
                                   const __nv_bfloat16* __restrict__ x, long ldx, __nv_bfloat16* __restrict__ xp,
                                   int d) {
  const int i = blockIdx.x;
  if (rank[i] < 0) {          // another rank's expert
    if (threadIdx.x == 0) pos[i] = -1;
    return;
  }
  const int p = seg_start[idx[i] - e0] + rank[i];
  if (threadIdx.x == 0) pos[i] = p;
  const uint4* src = reinterpret_cast<const uint4*>(x + (long)(i / k) * ldx);
  uint4* dst = reinterpret_cast<uint4*>(xp + (long)p * d);
  for (int v = threadIdx.x; v < d / 8; v += blockDim.x) dst[v] = src[v];
}

void moe_align(const int* idx, int n, int k, int e0, int E, int* counts, int* rank, int* seg_start, int* tile_start,
               int* pos, const __nv_bfloat16* x, long ldx, __nv_bfloat16* xp, int d, cudaStream_t stream) {
  const int nk = n * k;
  cudaMemsetAsync(counts, 0, sizeof(int) * E, stream);
  if (nk > 0) {
    moe_count_kernel<<<(nk + 255) / 256, 256, 0, stream>>>(idx, nk, e0, E, counts, rank);
    count_launch();
  }
  moe_scan_kernel<<<1, 1024, 0, stream>>>(counts, E, seg_start, tile_start);
  count_launch();
  if (nk > 0) {
    moe_scatter_kernel<<<nk, 128, 0, stream>>>(idx, rank, seg_start, k, e0, pos, x, ldx, xp, d);
    count_launch();
  }
}

// --------------------------------------------------------------------------------------- combine
// grid: one CTA per token; out = h + sum_k w y[pos] + sigmoid(gate) * ys  (gate = logits[t, E] when given)
__global__ void moe_combine_kernel(const __nv_bfloat16* __restrict__ h, long ldh, const __nv_bfloat16* __restrict__ y,
                                   const int* __restrict__ pos, const float* __restrict__ w, int k,
                                   const __nv_bfloat16* __restrict__ ys, const float* __restrict__ gate_logit,
                                   long ldg, __nv_bfloat16* __restrict__ out, int d) {
  const int t = blockIdx.x;
  float g = 0.f;
  if (ys != nullptr) {
    const float z = gate_logit != nullptr ? gate_logit[(long)t * ldg] : 0.f;
    g = gate_logit != nullptr ? 1.f / (1.f + expf(-z)) : 1.f;
  }
  for (int c = threadIdx.x * 8; c < d; c += blockDim.x * 8) {
    float acc[8];
    if (h != nullptr) {
      uint4 hv = *reinterpret_cast<const uint4*>(h + (long)t * ldh + c);
      const __nv_bfloat16* he = reinterpret_cast<const __nv_bfloat16*>(&hv);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(he[j]);
    } else {
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] = 0.f;
    }
    for (int s = 0; s < k; ++s) {
      const int p = pos[(long)t * k + s];
      if (p < 0) continue;    // expert on another rank
      const float ws = w[(long)t * k + s];
      uint4 yv = *reinterpret_cast<const uint4*>(y + (long)p * d + c);
      const __nv_bfloat16* ye = reinterpret_cast<const __nv_bfloat16*>(&yv);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += ws * __bfloat162float(ye[j]);
    }
    if (ys != nullptr) {
      uint4 sv = *reinterpret_cast<const uint4*>(ys + (long)t * d + c);
      const __nv_bfloat16* se = reinterpret_cast<const __nv_bfloat16*>(&sv);
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j] += g * __bfloat162float(se[j]);
    }
    uint4 o;
    o.x = pack_bf16x2(acc[0], acc[1]);
    o.y = pack_bf16x2(acc[2], acc[3]);
    o.z = pack_bf16x2(acc[4], acc[5]);
    o.w = pack_bf16x2(acc[6], acc[7]);
    *reinterpret_cast<uint4*>(out + (long)t * d + c) = o;
  }
}

void moe_combine(const __nv_bfloat16* h, long ldh, const __nv_bfloat16* y, const int* pos, const float* w, int n,
                 int k, const __nv_bfloat16* ys, const float* gate_logit, long ldg, __nv_bfloat16* out, int d,
                 cudaStream_t stream) {
  if (n <= 0) return;
  moe_combine_kernel<<<n, 256, 0, stream>>>(h, ldh, y, pos, w, k, ys, gate_logit, ldg, out, d);
  count_launch();
}

// ---------------------------------------------------------------------------------- grouped GEMM
constexpr int GBM = 128;
constexpr int GBK = 64;
constexpr int GBN = 256;
constexpr int GSTAGES = 4;
constexpr int G_A_BYTES = GBM * GBK * 2;
constexpr int G_B_BYTES = GBN * GBK * 2;
constexpr int G_STAGE = G_A_BYTES + G_B_BYTES;
constexpr int G_SMEM = 1024 + GSTAGES * G_STAGE + 8 * (2 * GSTAGES + 4) + 16;

struct GroupedArgs {
  int N, K, E;
  const int* seg_start;    // [E + 1]
  const int* tile_start;   // [E + 1] cumulative 128-row tiles
  void* out;               // bf16 [rows][ldo]
  long ldo;
  int swiglu;
  int* err;
};

__device__ __forceinline__ int find_expert(const int* tile_start, int E, int g) {
  int lo = 0, hi = E - 1;
  while (lo < hi) {   // largest e with tile_start[e] <= g (experts with no tiles are skipped)
    const int mid = (lo + hi + 1) >> 1;
    if (tile_start[mid] <= g) lo = mid;
    else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float silu_g(float x) { return x / (1.0f + __expf(-x)); }

__global__ void __launch_bounds__(192, 1)
    grouped_gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB,
                        GroupedArgs args) {
  constexpr uint32_t IDESC = idesc_bf16_f32(GBM, GBN, false, false);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + GSTAGES * G_STAGE);
  uint64_t* empty = full + GSTAGES;
  uint64_t* tfull = empty + GSTAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  const int warp = warp_id(), lane = lane_id();
  const int num_nb = (args.N + GBN - 1) / GBN;
  const int total_mt = args.tile_start[args.E];
  const int num_tiles = total_mt * num_nb;
  const int nkb = (args.K + GBK - 1) / GBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < GSTAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 2 * GBN);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  auto decode = [&](int t, int& e, int& row0, int& rows, int& nb) {
    // N tiles innermost: the num_nb CTAs of one row tile run together (A read from DRAM once, then L2), and an
    // expert's few row tiles sit num_nb apart (its weight tiles shared through L2 as well)
    const int g = t / num_nb;
    nb = t % num_nb;
    e = find_expert(args.tile_start, args.E, g);
    row0 = args.seg_start[e] + (g - args.tile_start[e]) * GBM;
    rows = min(GBM, args.seg_start[e + 1] - row0);
  };

  if (warp == 0) {
    if (lane == 0) {
      uint32_t stage = 0, phase = 0, issued = 0, last_par = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x) {
        int e, row0, rows, nb;
        decode(t, e, row0, rows, nb);
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrTimeoutProducer)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          mbar_expect_tx(&full[stage], G_STAGE);
          uint8_t* sA = smem + stage * G_STAGE;
          tma_load_2d(sA, &tmA, &full[stage], kb * GBK, row0);
          tma_load_3d(sA + G_A_BYTES, &tmB, &full[stage], kb * GBK, nb * GBN, e);
          if (++stage == GSTAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok)
        for (int s = 0; s < GSTAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, args.err, kErrTimeoutDrain);
    }
  } else if (warp == 1) {
    uint32_t stage = 0, phase = 0;
    int it = 0;
    bool ok = true;
    for (int t = blockIdx.x; t < num_tiles && ok; t += gridDim.x, ++it) {
      const uint32_t buf = it & 1, aphase = (it >> 1) & 1;
      if (*abort_flag || !mbar_wait(&tempty[buf], aphase ^ 1u, args.err, kErrTimeoutMma)) {
        ok = false;
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * GBN;
      for (int kb = 0; kb < nkb; ++kb) {
        if (*abort_flag || !mbar_wait(&full[stage], phase, args.err, kErrTimeoutMma)) {
          ok = false;
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * G_STAGE);
          const uint32_t b_addr = a_addr + G_A_BYTES;
#pragma unroll
          for (int k = 0; k < GBK / 16; ++k)
            umma_f16(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024), sdesc_sw128(b_addr + k * 32, 16, 1024), IDESC,
                     (kb > 0 || k > 0) ? 1u : 0u);
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == GSTAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull[buf]);
      __syncwarp();
    }
  } else {
    const int q = warp & 3;
    int it = 0;
    for (int t = blockIdx.x; t < num_tiles; t += gridDim.x, ++it) {
      int e, row0, rows, nb;
      decode(t, e, row0, rows, nb);
      const uint32_t buf = it & 1, aphase = (it >> 1) & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], aphase, args.err, kErrTimeoutEpilogue)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int r = q * 32 + lane;
      const bool row_ok = r < rows;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * GBN;
      __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)(row0 + r) * args.ldo;
      if (args.swiglu) {
#pragma unroll 1
        for (int c = 0; c < GBN / 2; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + GBN / 2 + c, u);
          tmem_wait_ld();
          const int col0 = nb * (GBN / 2) + c;
          if (row_ok && col0 < args.N / 2) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 v;
              v.x = pack_bf16x2(silu_g(__uint_as_float(g[j])) * __uint_as_float(u[j]),
                                silu_g(__uint_as_float(g[j + 1])) * __uint_as_float(u[j + 1]));
              v.y = pack_bf16x2(silu_g(__uint_as_float(g[j + 2])) * __uint_as_float(u[j + 2]),
                                silu_g(__uint_as_float(g[j + 3])) * __uint_as_float(u[j + 3]));
              v.z = pack_bf16x2(silu_g(__uint_as_float(g[j + 4])) * __uint_as_float(u[j + 4]),
                                silu_g(__uint_as_float(g[j + 5])) * __uint_as_float(u[j + 5]));
              v.w = pack_bf16x2(silu_g(__uint_as_float(g[j + 6])) * __uint_as_float(u[j + 6]),
                                silu_g(__uint_as_float(g[j + 7])) * __uint_as_float(u[j + 7]));
              *reinterpret_cast<uint4*>(out + col0 + j) = v;
            }
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < GBN; c += 32) {
          uint32_t v[32];
          tmem_ld32(tbase + c, v);
          tmem_wait_ld();
          const int col0 = nb * GBN + c;
          if (row_ok && col0 < args.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 8)
              *reinterpret_cast<uint4*>(out + col0 + j) =
                  make_uint4(pack_bf16x2(__uint_as_float(v[j]), __uint_as_float(v[j + 1])),
                             pack_bf16x2(__uint_as_float(v[j + 2]), __uint_as_float(v[j + 3])),
                             pack_bf16x2(__uint_as_float(v[j + 4]), __uint_as_float(v[j + 5])),
                             pack_bf16x2(__uint_as_float(v[j + 6]), __uint_as_float(v[j + 7])));
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, 2 * GBN);
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode3() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// xp [rows_cap, K] expert-sorted rows; w [E, N, K] stacked weights; out [rows_cap, N or N/2].
void grouped_gemm(const __nv_bfloat16* xp, long rows_cap, const __nv_bfloat16* w, int E, int N, int K,
                  const int* seg_start, const int* tile_start, __nv_bfloat16* out, long ldo, int swiglu, int* err,
                  cudaStream_t stream) {
  if (rows_cap <= 0) return;
  if (K % 8 != 0 || (swiglu && N % GBN != 0) || (!swiglu && N % 32 != 0))
    throw std::runtime_error("grouped_gemm: K % 8, N % 256 (SwiGLU) or N % 32");
  CUtensorMap ta = make_tmap_bf16_2d(xp, K, rows_cap, K, GBK, GBM);
  CUtensorMap tb;
  cuuint64_t dims[3] = {(cuuint64_t)K, (cuuint64_t)N, (cuuint64_t)E};
  cuuint64_t strides[2] = {(cuuint64_t)K * 2, (cuuint64_t)N * K * 2};
  cuuint32_t box[3] = {GBK, GBN, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode3()(&tb, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<__nv_bfloat16*>(w), dims, strides, box,
                         estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("grouped_gemm: tensor map encode failed " + std::to_string((int)r));
  static PerDeviceOnce once;
  once([] { cudaFuncSetAttribute(grouped_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, G_SMEM); });
  GroupedArgs a{N, K, E, seg_start, tile_start, out, ldo, swiglu, err};
  int dev = 0;
  cudaGetDevice(&dev);
  grouped_gemm_kernel<<<num_sms(dev), 192, G_SMEM, stream>>>(ta, tb, a);
  count_launch();
}

}  // namespace rf
