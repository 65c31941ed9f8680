// Persistent tcgen05 GEMM for sm_100a: C = A x B^T (+ epilogue), bf16 operands, fp32 TMEM accumulators.
//
// Roles per CTA (192 threads, one CTA per SM):
//   warp 0      TMA producer: A/B tiles into a STAGES-deep shared-memory ring (128-byte swizzle)
//   warp 1      TMEM owner + UMMA issuer: one elected lane issues tcgen05.mma (M=128, N=BN, K=16)
//   warps 2..5  epilogue: tcgen05.ld the accumulator (warp w reads TMEM lanes 32*(w%4)..+31), apply
//               the epilogue and write global memory
// Two TMEM accumulator buffers (2 x BN columns) let the epilogue of tile t overlap the MMAs of t+1.
//
// Operand majors: A is K-major ([M, K] row-major) or MN-major ([K, M] row-major); same for B
// ([N, K] or [K, N]). The MN-major forms serve the ridge Gram X^T Y, which reads row-major
// activations without a transpose.
//
// Epilogues: kEpiStore (bf16 out, optional bias[n] and residual[m, n]), kEpiSwiGLU (columns
// [0, BN/2) of each tile are gate rows, [BN/2, BN) the matching up rows: out = silu(g) * u),
// kEpiF32 (fp32 out), kEpiF64Acc (fp64 out += acc, split-K chunks added with atomics: the
// fp32-per-block, fp64-across-blocks accumulation of the ridge sufficient statistics), kEpiPeer (tiles
// stored into other GPUs' buffers) and kEpiNvlsAR: the tensor-parallel row-parallel product fused with its
// all-reduce. The CTA then has 10 warps: the comm warps reduce the row blocks this rank owns through the
// NVSwitch (multimem.ld_reduce / multimem.st) as soon as every rank's epilogues have finished them, while the
// other warps keep computing later tiles (the grouped tile order finishes row blocks 16 at a time; a row-major
// order measured slower). Warps 6-9 are the comm warps.
#include "gemm.h"
#include "kernels.h"
#include "ptx.cuh"
#include "comm.cuh"

#include <cudaTypedefs.h>
#include <algorithm>
#include <cstdio>
#include <mutex>
#include <stdexcept>
#include <string>

namespace rf {

constexpr int BM = 128;
constexpr int BK = 64;
constexpr int kGemmThreads = 192;

constexpr int kCommWarps = 4;     // kEpiNvlsAR: warps 6..9 move the reduced rows
constexpr int kCommUnroll = 8;    // 16-byte multimem loads in flight per comm thread (16 measured no faster)
constexpr int kCommBatch = 8;     // owned row blocks reduced in one pass when they are already complete

template <int EPI>
struct GemmThreads {
  static constexpr int value = EPI == kEpiNvlsAR ? kGemmThreads + 32 * kCommWarps : kGemmThreads;
};
constexpr int kGroupM = 16;   // rasterisation: consecutive tiles walk 16 M-blocks per N-block

template <int BN>
struct GemmCfg {
  static constexpr int A_BYTES = BM * BK * 2;
  static constexpr int B_BYTES = BN * BK * 2;
  static constexpr int STAGE_BYTES = A_BYTES + B_BYTES;
  static constexpr int STAGES = BN == 256 ? 4 : 6;
  static constexpr int TMEM_COLS = 2 * BN;
  static constexpr int BAR_BYTES = 8 * (2 * STAGES + 4) + 16;
  static constexpr int SMEM_BYTES = 1024 + STAGES * STAGE_BYTES + BAR_BYTES;
  // kEpiNvlsAG: per epilogue warp a 32-row x 64-column bf16 staging tile, so the multicast stores go out as
  // 128-byte row segments instead of one 16-byte piece per row
  static constexpr int STAGE_OFF = (STAGES * STAGE_BYTES + BAR_BYTES + 127) / 128 * 128;
  static constexpr int AG_STAGING = 4 * 32 * 128;
  static constexpr int SMEM_BYTES_AG = 1024 + STAGE_OFF + AG_STAGING;
};

template <int BN, int EPI>
constexpr int gemm_smem_bytes() {
  return EPI == kEpiNvlsAG ? GemmCfg<BN>::SMEM_BYTES_AG : GemmCfg<BN>::SMEM_BYTES;
}

struct TileCoord {
  int mb, nb, ks;
};

__device__ __forceinline__ TileCoord tile_coord(int t, int num_mb, int num_nb, int k_splits) {
  TileCoord c;
  c.ks = t % k_splits;
  int t2 = t / k_splits;
  int per_group = kGroupM * num_nb;
  int group = t2 / per_group;
  int first = group * kGroupM;
  int gsize = min(num_mb - first, kGroupM);
  int r = t2 % per_group;
  c.mb = first + r % gsize;
  c.nb = r / gsize;
  return c;
}

__device__ __forceinline__ float silu_f(float x) { return x / (1.0f + __expf(-x)); }

template <int BN, int EPI, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(GemmThreads<EPI>::value, 1)
    gemm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args) {
  using Cfg = GemmCfg<BN>;
  constexpr int STAGES = Cfg::STAGES;
  constexpr uint32_t IDESC = idesc_bf16_f32(BM, BN, A_MN, B_MN);

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + STAGES * Cfg::STAGE_BYTES);
  uint64_t* empty = full + STAGES;
  uint64_t* tfull = empty + STAGES;
  uint64_t* tempty = tfull + 2;
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(tempty + 2);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  __shared__ int s_tile_warps[2];   // kEpiNvlsAR: epilogue warps done with the tile in accumulator buffer b
  __shared__ int s_comm_ok;

  const int warp = warp_id();
  const int lane = lane_id();
  const int num_mb = (args.M + BM - 1) / BM;
  const int num_nb = (args.N + BN - 1) / BN;
  const int num_tiles = num_mb * num_nb * args.k_splits;
  // kEpiNvlsAR with comm_ctas > 0: the last comm_ctas CTAs only move reduced rows (no tiles), the others only
  // compute tiles, so the reduction traffic does not share SM ports with the GEMM's TMA loads
  int tile_ctas = gridDim.x, comm_first = 0;
  if constexpr (EPI == kEpiNvlsAR) {
    if (args.nvls.comm_ctas > 0 && args.nvls.comm_ctas < (int)gridDim.x) {
      tile_ctas = gridDim.x - args.nvls.comm_ctas;
      comm_first = tile_ctas;
    }
  }
  const int tile_begin = (int)blockIdx.x < tile_ctas ? (int)blockIdx.x : num_tiles;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 128);
    }
    *abort_flag = 0;
    s_tile_warps[0] = s_tile_warps[1] = 0;
    fence_barrier_init();
    tma_prefetch_desc(&tmA);
    tma_prefetch_desc(&tmB);
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, Cfg::TMEM_COLS);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      uint32_t stage = 0, phase = 0;
      uint32_t issued = 0, last_par = 0;   // per stage: a load was issued / parity of its phase
      bool ok = true;
      for (int t = tile_begin; t < num_tiles && ok; t += tile_ctas) {
        TileCoord tc = tile_coord(t, num_mb, num_nb, args.k_splits);
        const int k0 = tc.ks * args.k_chunk;
        const int k1 = min(args.K, k0 + args.k_chunk);
        const int nkb = (k1 - k0 + BK - 1) / BK;
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag || !mbar_wait(&empty[stage], phase ^ 1u, args.err, kErrTimeoutProducer)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          mbar_expect_tx(&full[stage], Cfg::STAGE_BYTES);
          uint8_t* sA = smem + stage * Cfg::STAGE_BYTES;
          uint8_t* sB = sA + Cfg::A_BYTES;
          const int kc = k0 + kb * BK;
          if (!A_MN) {
            tma_load_2d(sA, &tmA, &full[stage], kc, tc.mb * BM);
          } else {
#pragma unroll
            for (int h = 0; h < BM / 64; ++h) tma_load_2d(sA + h * 8192, &tmA, &full[stage], tc.mb * BM + h * 64, kc);
          }
          if (!B_MN) {
            tma_load_2d(sB, &tmB, &full[stage], kc, tc.nb * BN);
          } else {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h) tma_load_2d(sB + h * 8192, &tmB, &full[stage], tc.nb * BN + h * 64, kc);
          }
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok) {
        // Drain: the last load issued into every stage must land before the CTA may exit.
        for (int s = 0; s < STAGES; ++s)
          if (issued & (1u << s)) mbar_wait(&full[s], (last_par >> s) & 1u, args.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ UMMA issuer
    uint32_t stage = 0, phase = 0;
    int it = 0;
    bool ok = true;
    for (int t = tile_begin; t < num_tiles && ok; t += tile_ctas, ++it) {
      TileCoord tc = tile_coord(t, num_mb, num_nb, args.k_splits);
      const int k0 = tc.ks * args.k_chunk;
      const int k1 = min(args.K, k0 + args.k_chunk);
      const int nkb = (k1 - k0 + BK - 1) / BK;
      const uint32_t buf = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (*abort_flag || !mbar_wait(&tempty[buf], aphase ^ 1u, args.err, kErrTimeoutMma)) {
        ok = false;
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const uint32_t d_tmem = tmem_base + buf * BN;
      for (int kb = 0; kb < nkb; ++kb) {
        if (*abort_flag || !mbar_wait(&full[stage], phase, args.err, kErrTimeoutMma)) {
          ok = false;
          *abort_flag = 1;
          break;
        }
        tc_fence_after();
        if (lane == 0) {
          const uint32_t a_addr = smem_u32(smem + stage * Cfg::STAGE_BYTES);
          const uint32_t b_addr = a_addr + Cfg::A_BYTES;
#pragma unroll
          for (int k = 0; k < BK / 16; ++k) {
            const uint64_t ad = A_MN ? sdesc_sw128(a_addr + k * 2048, 8192, 1024) : sdesc_sw128(a_addr + k * 32, 16, 1024);
            const uint64_t bd = B_MN ? sdesc_sw128(b_addr + k * 2048, 8192, 1024) : sdesc_sw128(b_addr + k * 32, 16, 1024);
            umma_f16(d_tmem, ad, bd, IDESC, (kb > 0 || k > 0) ? 1u : 0u);
          }
          umma_commit(&empty[stage]);
        }
        __syncwarp();
        if (++stage == STAGES) {
          stage = 0;
          phase ^= 1u;
        }
      }
      if (!ok) break;
      if (lane == 0) umma_commit(&tfull[buf]);
      __syncwarp();
    }
    if (!ok) {
      // Wait (bounded) for MMAs already issued before TMEM is released.
      if (lane == 0) umma_commit(&tfull[0]);
      __syncwarp();
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------------ epilogue (warps 2..5)
    const int q = warp & 3;                 // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int it = 0;
    for (int t = tile_begin; t < num_tiles; t += tile_ctas, ++it) {
      TileCoord tc = tile_coord(t, num_mb, num_nb, args.k_splits);
      const uint32_t buf = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (*abort_flag || !mbar_wait(&tfull[buf], aphase, args.err, kErrTimeoutEpilogue)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = tc.mb * BM + row_in_tile;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * BN;

      if constexpr (EPI == kEpiSwiGLU) {
        constexpr int HALF = BN / 2;
        const int ncols_out = args.N / 2;
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
#pragma unroll 1
        for (int c = 0; c < HALF; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + HALF + c, u);
          tmem_wait_ld();
          const int col0 = tc.nb * HALF + c;
          if (row_ok) {
            __nv_bfloat16* dst = out + (size_t)row * args.ldo + col0;
            if (col0 + 32 <= ncols_out && args.vec_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 v;
                v.x = pack_bf16x2(silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]),
                                  silu_f(__uint_as_float(g[j + 1])) * __uint_as_float(u[j + 1]));
                v.y = pack_bf16x2(silu_f(__uint_as_float(g[j + 2])) * __uint_as_float(u[j + 2]),
                                  silu_f(__uint_as_float(g[j + 3])) * __uint_as_float(u[j + 3]));
                v.z = pack_bf16x2(silu_f(__uint_as_float(g[j + 4])) * __uint_as_float(u[j + 4]),
                                  silu_f(__uint_as_float(g[j + 5])) * __uint_as_float(u[j + 5]));
                v.w = pack_bf16x2(silu_f(__uint_as_float(g[j + 6])) * __uint_as_float(u[j + 6]),
                                  silu_f(__uint_as_float(g[j + 7])) * __uint_as_float(u[j + 7]));
                *reinterpret_cast<uint4*>(dst + j) = v;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < ncols_out)
                  dst[j] = __float2bfloat16(silu_f(__uint_as_float(g[j])) * __uint_as_float(u[j]));
            }
          }
        }
      } else if constexpr (EPI == kEpiNvlsAG) {
        // 64 columns at a time: bias, bf16, staged row-major (16-byte units XOR-swizzled by row), then each
        // instruction multicasts 4 rows x 128 contiguous bytes
        uint4* stg = reinterpret_cast<uint4*>(smem + Cfg::STAGE_OFF) + (size_t)q * 32 * 8;
        const int row0 = tc.mb * BM + q * 32;
        __nv_bfloat16* out = reinterpret_cast<__nv_bfloat16*>(args.out);
#pragma unroll 1
        for (int c = 0; c < BN; c += 64) {
          uint32_t ra[32], rb[32];
          tmem_ld32(tbase + c, ra);
          tmem_ld32(tbase + c + 32, rb);
          tmem_wait_ld();
          const int col0 = tc.nb * BN + c;
          if (col0 >= args.N) continue;
          float v[64];
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            v[j] = __uint_as_float(ra[j]);
            v[32 + j] = __uint_as_float(rb[j]);
          }
          if (args.bias != nullptr) {
#pragma unroll
            for (int j = 0; j < 64; ++j) v[j] += __bfloat162float(args.bias[col0 + j]);
          }
#pragma unroll
          for (int u = 0; u < 8; ++u) {
            uint4 w;
            w.x = pack_bf16x2(v[8 * u], v[8 * u + 1]);
            w.y = pack_bf16x2(v[8 * u + 2], v[8 * u + 3]);
            w.z = pack_bf16x2(v[8 * u + 4], v[8 * u + 5]);
            w.w = pack_bf16x2(v[8 * u + 6], v[8 * u + 7]);
            stg[lane * 8 + (u ^ (lane & 7))] = w;
          }
          __syncwarp();
#pragma unroll
          for (int k = 0; k < 8; ++k) {
            const int rr = k * 4 + (lane >> 3), u = lane & 7;
            const uint4 w = stg[rr * 8 + (u ^ (rr & 7))];
            if (row0 + rr < args.M) multimem_st_16(out + (size_t)(row0 + rr) * args.ldo + col0 + u * 8, w);
          }
          __syncwarp();
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < BN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_wait_ld();
          const int col0 = tc.nb * BN + c;
          if (!row_ok || col0 >= args.N) continue;
          const bool full_chunk = (col0 + 32 <= args.N);
          if constexpr (EPI == kEpiStore || EPI == kEpiNvlsAR) {
            __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(args.out) + (size_t)row * args.ldo + col0;
            float v[32];
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(r[j]);
            if (args.bias != nullptr) {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.N) v[j] += __bfloat162float(args.bias[col0 + j]);
            }
            if (args.residual != nullptr) {
              const __nv_bfloat16* res = args.residual + (size_t)row * args.ldr + col0;
              if (full_chunk && args.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 8) {
                  uint4 w = *reinterpret_cast<const uint4*>(res + j);
                  v[j] += bf16_lo(w.x); v[j + 1] += bf16_hi(w.x);
                  v[j + 2] += bf16_lo(w.y); v[j + 3] += bf16_hi(w.y);
                  v[j + 4] += bf16_lo(w.z); v[j + 5] += bf16_hi(w.z);
                  v[j + 6] += bf16_lo(w.w); v[j + 7] += bf16_hi(w.w);
                }
              } else {
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < args.N) v[j] += __bfloat162float(res[j]);
              }
            }
            if (full_chunk && args.vec_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 8) {
                uint4 w;
                w.x = pack_bf16x2(v[j], v[j + 1]);
                w.y = pack_bf16x2(v[j + 2], v[j + 3]);
                w.z = pack_bf16x2(v[j + 4], v[j + 5]);
                w.w = pack_bf16x2(v[j + 6], v[j + 7]);
                *reinterpret_cast<uint4*>(dst + j) = w;
              }
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.N) dst[j] = __float2bfloat16(v[j]);
            }
          } else if constexpr (EPI == kEpiPeer) {
            const PeerArgs& pa = args.peer;
            if (pa.mode == 0) {
              const int q = row / pa.row_chunk;
              __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(pa.peer[q]) + (size_t)pa.slot * pa.slot_stride +
                                   (size_t)(row - q * pa.row_chunk) * pa.ld + col0;
              if (full_chunk && args.vec_ok) {
#pragma unroll
                for (int j = 0; j < 32; j += 8)
                  *reinterpret_cast<uint4*>(dst + j) =
                      make_uint4(pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])),
                                 pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                                 pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5])),
                                 pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7])));
              } else {
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < args.N) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
              }
            } else {
              if (args.bias != nullptr) {
                for (int j = 0; j < 32; ++j)
                  if (col0 + j < args.N)
                    r[j] = __float_as_uint(__uint_as_float(r[j]) + __bfloat162float(args.bias[col0 + j]));
              }
              uint4 packed[4];
#pragma unroll
              for (int j = 0; j < 32; j += 8)
                packed[j / 8] = make_uint4(pack_bf16x2(__uint_as_float(r[j]), __uint_as_float(r[j + 1])),
                                           pack_bf16x2(__uint_as_float(r[j + 2]), __uint_as_float(r[j + 3])),
                                           pack_bf16x2(__uint_as_float(r[j + 4]), __uint_as_float(r[j + 5])),
                                           pack_bf16x2(__uint_as_float(r[j + 6]), __uint_as_float(r[j + 7])));
              for (int q = 0; q < pa.n_peers; ++q) {
                __nv_bfloat16* dst =
                    reinterpret_cast<__nv_bfloat16*>(pa.peer[q]) + (size_t)row * pa.ld + pa.col_off + col0;
                if (full_chunk && args.vec_ok) {
#pragma unroll
                  for (int j = 0; j < 4; ++j) *reinterpret_cast<uint4*>(dst + 8 * j) = packed[j];
                } else {
                  for (int j = 0; j < 32; ++j)
                    if (col0 + j < args.N) dst[j] = __float2bfloat16(__uint_as_float(r[j]));
                }
              }
            }
          } else if constexpr (EPI == kEpiF32) {
            float* dst = reinterpret_cast<float*>(args.out) + (size_t)row * args.ldo + col0;
            if (full_chunk && args.vec_ok) {
#pragma unroll
              for (int j = 0; j < 32; j += 4)
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(r[j], r[j + 1], r[j + 2], r[j + 3]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.N) dst[j] = __uint_as_float(r[j]);
            }
          } else {  // kEpiF64Acc
            double* dst = reinterpret_cast<double*>(args.out) + (size_t)row * args.ldo + col0;
            if (args.k_splits == 1) {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.N) dst[j] += (double)__uint_as_float(r[j]);
            } else {
              for (int j = 0; j < 32; ++j)
                if (col0 + j < args.N) atomicAdd(dst + j, (double)__uint_as_float(r[j]));
            }
          }
        }
      }
      if constexpr (EPI == kEpiNvlsAR) {
        // the fourth epilogue warp to finish this tile counts it for its row block; the block's last tile
        // announces the block to every rank
        __syncwarp();
        if (lane == 0) {
          __threadfence();
          if (atomicAdd(&s_tile_warps[buf], 1) == 3) {
            atomicExch(&s_tile_warps[buf], 0);
            const NvlsGemmArgs& nv = args.nvls;
            if (atomicAdd(nv.rb_count + tc.mb, 1) == num_nb - 1) {
              nv.rb_count[tc.mb] = 0;
              __threadfence_system();
              for (int q = 0; q < nv.world; ++q) st_release_sys(nv.peer_flags[q] + tc.mb * kMaxPeers + nv.rank, nv.epoch);
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(&tempty[buf]);
    }
    if constexpr (EPI == kEpiNvlsAG) {
      // every epilogue warp of every CTA is done storing: the last CTA announces this rank; one thread per CTA
      // waits (bounded) for every rank, so the gathered tensor is complete when the kernel ends
      named_bar_sync(2, 128);
      if (warp == 2 && lane == 0) {
        const NvlsGemmArgs& nv = args.nvls;
        const int done_off = nv.max_mb * kMaxPeers;
        __threadfence_system();
        if (atomicAdd(nv.done_count, 1) == (int)gridDim.x - 1) {
          *nv.done_count = 0;
          for (int q = 0; q < nv.world; ++q) st_release_sys(nv.peer_flags[q] + done_off + nv.rank, nv.epoch);
        }
        bool good = true;
        for (int q = 0; q < nv.world && good; ++q) good = wait_value(nv.flags + done_off + q, nv.epoch, args.err);
      }
    }
  } else if constexpr (EPI == kEpiNvlsAR) {
    // ------------------------------------------------------------------ comm warps (6..9)
    // Owned row blocks (mb % world == rank) in ascending order; each pass waits for the next one and takes up to
    // kCommBatch following owned blocks that are already complete on every rank. Every CTA moves its own
    // 1/gridDim slice of each block, so the whole grid shares every block.
    constexpr int CT = 32 * kCommWarps;
    const NvlsGemmArgs& nv = args.nvls;
    const int ct = threadIdx.x - 6 * 32;
    const int units_row = args.N / 8;
    const int comm_ctas = (int)gridDim.x - comm_first;            // CTAs sharing every row block
    const int comm_idx = (int)blockIdx.x - comm_first;            // < 0: this CTA computes tiles only
    const long slice = ((long)BM * units_row + comm_ctas - 1) / comm_ctas;
    const char* in = reinterpret_cast<const char*>(nv.mc_part);
    char* outp = reinterpret_cast<char*>(nv.mc_out);
    __shared__ int s_batch;
    bool ok = true;
    int mb = nv.rank;
    while (mb < num_mb && ok) {
      if (ct == 0) {
        bool good = true;
        for (int q = 0; q < nv.world && good; ++q) good = wait_value(nv.flags + mb * kMaxPeers + q, nv.epoch, args.err);
        int nb = 1;
        while (good && nb < kCommBatch && mb + nb * nv.world < num_mb) {
          const int nxt = mb + nb * nv.world;
          bool ready = true;
          for (int q = 0; q < nv.world && ready; ++q) ready = ld_acquire_sys(nv.flags + nxt * kMaxPeers + q) == nv.epoch;
          if (!ready) break;
          ++nb;
        }
        s_comm_ok = good ? 1 : 0;
        s_batch = nb;
      }
      named_bar_sync(1, CT);
      ok = s_comm_ok != 0;
      const int nbatch = s_batch;
      named_bar_sync(1, CT);
      if (!ok) break;
      const long total = (nv.comm_off || comm_idx < 0) ? 0 : (long)nbatch * slice;
      for (long j0 = ct; j0 < total; j0 += (long)CT * kCommUnroll) {
        uint4 v[kCommUnroll];
        long off[kCommUnroll];
#pragma unroll
        for (int k = 0; k < kCommUnroll; ++k) {
          const long j = j0 + (long)k * CT;
          off[k] = -1;
          if (j < total) {
            const int b = (int)(j / slice);
            const long u = (long)comm_idx * slice + (j - (long)b * slice);
            const int blk = mb + b * nv.world;
            const int r0 = blk * BM;
            const long nu = (long)(min(args.M, r0 + BM) - r0) * units_row;
            if (u < nu) {
              off[k] = ((long)(r0 + u / units_row) * args.ldo + (u % units_row) * 8) * 2;
              multimem_ld_reduce_bf16x8(in + off[k], v[k]);
            }
          }
        }
#pragma unroll
        for (int k = 0; k < kCommUnroll; ++k)
          if (off[k] >= 0) multimem_st_16(outp + off[k], v[k]);
      }
      mb += nbatch * nv.world;
    }
    // every CTA's sums are out: the last CTA announces this rank done; every CTA waits for all ranks
    named_bar_sync(1, CT);
    if (ct == 0) {
      __threadfence_system();
      const int done_off = nv.max_mb * kMaxPeers;
      if (atomicAdd(nv.done_count, 1) == (int)gridDim.x - 1) {
        *nv.done_count = 0;
        for (int q = 0; q < nv.world; ++q) st_release_sys(nv.peer_flags[q] + done_off + nv.rank, nv.epoch);
      }
      bool good = true;
      for (int q = 0; q < nv.world && good; ++q) good = wait_value(nv.flags + done_off + q, nv.epoch, args.err);
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, Cfg::TMEM_COLS);
  }
}

// ============================================================================== host side

static PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
    if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D bf16 tensor map over a row-major matrix [outer, inner] with row pitch `pitch_elems`.
CUtensorMap make_tmap_bf16_2d(const void* base, uint64_t inner, uint64_t outer, uint64_t pitch_elems,
                              uint32_t box_inner, uint32_t box_outer) {
  CUtensorMap tm;
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_fn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

int num_sms(int device) {
  static int cached[64] = {0};
  if (device < 0 || device >= 64) return 148;
  if (cached[device] == 0) {
    int v = 0;
    cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, device);
    cached[device] = v > 0 ? v : 148;
  }
  return cached[device];
}

template <int BN, int EPI, bool A_MN, bool B_MN>
static void launch_gemm(const GemmOperands& op, GemmArgs args, int max_ctas, cudaStream_t stream) {
  using Cfg = GemmCfg<BN>;
  auto kernel = gemm_kernel<BN, EPI, A_MN, B_MN>;
  static PerDeviceOnce once;
  once([kernel] { cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, gemm_smem_bytes<BN, EPI>()); });
  int dev = 0;
  cudaGetDevice(&dev);
  CUtensorMap ta = A_MN ? make_tmap_bf16_2d(op.A, args.M, args.K, op.lda, 64, 64)
                        : make_tmap_bf16_2d(op.A, args.K, args.M, op.lda, 64, BM);
  CUtensorMap tb = B_MN ? make_tmap_bf16_2d(op.B, args.N, args.K, op.ldb, 64, 64)
                        : make_tmap_bf16_2d(op.B, args.K, args.N, op.ldb, 64, BN);
  const int num_tiles = ((args.M + BM - 1) / BM) * ((args.N + BN - 1) / BN) * args.k_splits;
  int ctas = num_sms(dev);
  if (max_ctas > 0 && max_ctas < ctas) ctas = max_ctas;
  if (num_tiles < ctas) ctas = num_tiles;
  if (ctas <= 0) return;
  if (EPI == kEpiNvlsAR && ctas != num_sms(dev) && num_tiles < num_sms(dev)) {
    // every CTA takes part in the reduction: keep one CTA per SM even when there are fewer tiles
    ctas = max_ctas > 0 ? std::min(max_ctas, num_sms(dev)) : num_sms(dev);
  }
  kernel<<<ctas, GemmThreads<EPI>::value, gemm_smem_bytes<BN, EPI>(), stream>>>(ta, tb, args);
  count_launch();
}

void gemm_bf16(const GemmOperands& op, GemmArgs args, int epi, int bn, int max_ctas, cudaStream_t stream) {
  if (args.M <= 0 || args.N <= 0 || args.K <= 0) return;
  if (args.k_splits <= 0) args.k_splits = 1;
  if (args.k_chunk <= 0 || args.k_splits == 1) args.k_chunk = args.K;
  if (args.k_splits > 1 && args.k_chunk % BK != 0) throw std::runtime_error("split-K chunk must be a multiple of 64");
  if (epi == kEpiSwiGLU && (args.N % bn != 0)) throw std::runtime_error("SwiGLU GEMM needs N % BN == 0");
  if (epi != kEpiF64Acc && args.k_splits != 1) throw std::runtime_error("split-K only with the fp64 epilogue");
  if (args.M <= 16 && gemm_bf16_gemv(op, args, epi, bn, stream)) return;
  if (bn == 256 && max_ctas != 1 && gemm_bf16_2sm(op, args, epi, max_ctas, stream)) return;
#define RF_GEMM_CASE(BN_, EPI_, AM_, BMJ_)                                               \
  if (bn == BN_ && epi == EPI_ && op.a_mn == AM_ && op.b_mn == BMJ_) {                   \
    launch_gemm<BN_, EPI_, AM_, BMJ_>(op, args, max_ctas, stream);                       \
    return;                                                                              \
  }
  RF_GEMM_CASE(256, kEpiStore, false, false)
  RF_GEMM_CASE(128, kEpiStore, false, false)
  RF_GEMM_CASE(256, kEpiSwiGLU, false, false)
  RF_GEMM_CASE(128, kEpiSwiGLU, false, false)
  RF_GEMM_CASE(256, kEpiF32, false, false)
  RF_GEMM_CASE(128, kEpiF32, false, false)
  RF_GEMM_CASE(256, kEpiF64Acc, true, true)
  RF_GEMM_CASE(128, kEpiF64Acc, true, true)
  RF_GEMM_CASE(256, kEpiF64Acc, false, false)
  RF_GEMM_CASE(256, kEpiStore, true, true)
  RF_GEMM_CASE(256, kEpiPeer, false, false)
  RF_GEMM_CASE(128, kEpiPeer, false, false)
  RF_GEMM_CASE(256, kEpiNvlsAR, false, false)
  RF_GEMM_CASE(128, kEpiNvlsAR, false, false)
  RF_GEMM_CASE(256, kEpiNvlsAG, false, false)
  RF_GEMM_CASE(128, kEpiNvlsAG, false, false)
#undef RF_GEMM_CASE
  throw std::runtime_error("gemm_bf16: unsupported (bn, epilogue, majors) combination");
}

}  // namespace rf
