// Two-SM tcgen05 GEMM for sm_100a (cta_group::2): C = A x B^T with the store (bias / residual) or SwiGLU epilogue.
//
// A cluster of two CTAs on one TPC computes a 256 x 256 output tile with one tcgen05.mma.cta_group::2 stream:
//   CTA r (r = %cluster_ctarank) loads rows [256 mb + 128 r, +128) of A and rows [256 nb + 128 r, +128) of B into its
//   own shared memory (per-CTA TMA loads, no multicast; the .cta_group::2 form lets both CTAs' loads complete on the
//   leader's full barrier); the leader (r = 0) issues the MMAs, which read both CTAs' halves at the same shared
//   offsets; CTA r's TMEM receives output rows [256 mb + 128 r, +128) x all 256 columns.
// Per SM this halves the B tile each k-step moves from L2 into shared memory and reads into the tensor core
// (a 128 x 256 tile on one SM reads 128 + 256 operand rows per k; here each SM reads 128 + 128), which is what limits
// the one-SM kernel (gemm.cu) at ~75 % tensor-pipe activity.
//
// Roles per CTA (192 threads): warp 0 TMA producer (both CTAs), warp 1 TMEM allocator (both, collectively) and MMA
// issuer (leader only), warps 2..5 epilogue (both: each reads its own TMEM lanes). Barriers:
//   full[s]   leader only: expect_tx of both CTAs' bytes; both CTAs' loads complete on it
//   empty[s]  per CTA: the leader's tcgen05.commit arrives on both CTAs' copies (multicast commit)
//   tfull[b]  per CTA: accumulator b holds a finished tile (multicast commit)
//   tempty[b] leader only: 256 arrivals (both CTAs' epilogue threads, remote arrives) free accumulator b
// Every wait is bounded (2 s); a timeout records an error code, the CTA drains and both CTAs meet at the final
// cluster barrier before the TMEM is released.
#include "gemm.h"
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace rf {
namespace {

constexpr int kTileM = 256;                    // per CTA pair
constexpr int kTileN = 256;
constexpr int kBK = 64;
constexpr int kStages = 6;
constexpr int kHalfBytes = 128 * kBK * 2;       // one CTA's A half or B half per stage
constexpr int kStageBytes = 2 * kHalfBytes;     // A half + B half
constexpr int kThreads = 192;
constexpr int kBarOff = kStages * kStageBytes;
constexpr int kSmemBytes = 1024 + kBarOff + 8 * (2 * kStages + 5) + 16;
constexpr int kGroupM2 = 8;                     // rasterisation: 8 pair-rows of tiles per column sweep

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_count() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
  return r;
}
// the shared::cluster address of this CTA's variable at `saddr` in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_barrier() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void arrive_remote(uint32_t cl_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_addr) : "memory");
}
__device__ __forceinline__ bool test_cluster(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}
// bounded wait (cluster-scope acquire: the barrier is signalled from the peer CTA or by the pair's MMAs)
__device__ __forceinline__ bool wait_cluster(uint64_t* bar, uint32_t parity, int* err, int code) {
  if (test_cluster(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns();
  uint32_t spins = 0;
  while (true) {
    if (test_cluster(bar, parity)) return true;
    if ((++spins & 255u) == 0u && global_timer_ns() - t0 > kWaitNs) {
      record_error(err, code);
      return false;
    }
  }
}
__device__ __forceinline__ void tma_load_pair(uint32_t dst, const CUtensorMap* tm, uint32_t bar_cl, int c0, int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(dst),
      "l"(tm), "r"(bar_cl), "r"(c0), "r"(c1)
      : "memory");
}
__device__ __forceinline__ void mma_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// arrive (once) on the barrier at this offset in both CTAs of the pair when the pair's MMAs issued so far complete
__device__ __forceinline__ void commit_pair(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
                   smem_u32(bar)),
               "h"((uint16_t)3)
               : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* holder, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(holder)), "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

__device__ __forceinline__ float silu2(float x) { return x / (1.0f + __expf(-x)); }

__device__ __forceinline__ void tile_of(int t, int num_mb, int num_nb, int& mb, int& nb) {
  const int per_group = kGroupM2 * num_nb;
  const int group = t / per_group;
  const int first = group * kGroupM2;
  const int gsize = min(num_mb - first, kGroupM2);
  const int r = t % per_group;
  mb = first + r % gsize;
  nb = r / gsize;
}

template <int EPI>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    gemm2sm_kernel(const __grid_constant__ CUtensorMap tmA, const __grid_constant__ CUtensorMap tmB, GemmArgs args) {
  constexpr uint32_t IDESC = idesc_bf16_f32(kTileM, kTileN, false, false);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kBarOff);
  uint64_t* empty = full + kStages;
  uint64_t* tfull = empty + kStages;
  uint64_t* tempty = tfull + 2;
  uint64_t* drain = tempty + 2;        // abort path only: every MMA issued so far has completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(drain + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int warp = warp_id(), lane = lane_id();
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int num_mb = (args.M + kTileM - 1) / kTileM;
  const int num_nb = (args.N + kTileN - 1) / kTileN;
  const int num_tiles = num_mb * num_nb;
  const int first_tile = (int)cluster_index();
  const int tile_step = (int)cluster_count();

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull[b], 1);
      mbar_init(&tempty[b], 2 * 128);
    }
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {                     // both CTAs' warp 1, collectively: 512 columns in each CTA's TMEM
    tmem_alloc_pair(tmem_holder, 2 * kTileN);
    tmem_relinquish_pair();
  }
  tc_fence_before();
  __syncthreads();
  cluster_barrier();                   // the peer's barriers exist before any remote arrive or load completes
  tc_fence_after();
  const uint32_t tmem_base = *tmem_holder;

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer (both CTAs)
    if (lane == 0) {
      uint32_t full_cl[kStages];
      for (int s = 0; s < kStages; ++s) full_cl[s] = map_shared(smem_u32(&full[s]), 0);
      uint32_t stage = 0, phase = 0;
      uint32_t issued = 0, last_par = 0;
      bool ok = true;
      const int nkb = (args.K + kBK - 1) / kBK;
      for (int t = first_tile; t < num_tiles && ok; t += tile_step) {
        int mb, nb;
        tile_of(t, num_mb, num_nb, mb, nb);
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag || !wait_cluster(&empty[stage], phase ^ 1u, args.err, kErrTimeoutProducer)) {
            ok = false;
            *abort_flag = 1;
            break;
          }
          issued |= 1u << stage;
          last_par = (last_par & ~(1u << stage)) | (phase << stage);
          if (leader) mbar_expect_tx(&full[stage], 2 * kStageBytes);
          const uint32_t sA = smem_u32(smem + stage * kStageBytes);
          tma_load_pair(sA, &tmA, full_cl[stage], kb * kBK, mb * kTileM + (int)rank * 128);
          tma_load_pair(sA + kHalfBytes, &tmB, full_cl[stage], kb * kBK, nb * kTileN + (int)rank * 128);
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
      }
      if (!ok && leader) {             // every load of both CTAs completes on the leader's full barriers
        for (int s = 0; s < kStages; ++s)
          if (issued & (1u << s)) wait_cluster(&full[s], (last_par >> s) & 1u, args.err, kErrTimeoutDrain);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer (leader)
    if (leader) {
      uint32_t stage = 0, phase = 0;
      int it = 0;
      bool ok = true;
      const int nkb = (args.K + kBK - 1) / kBK;
      for (int t = first_tile; t < num_tiles && ok; t += tile_step, ++it) {
        const uint32_t buf = it & 1;
        const uint32_t aphase = (it >> 1) & 1;
        if (*abort_flag || !wait_cluster(&tempty[buf], aphase ^ 1u, args.err, kErrTimeoutMma)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kTileN;
        for (int kb = 0; kb < nkb; ++kb) {
          if (*abort_flag || !wait_cluster(&full[stage], phase, args.err, kErrTimeoutMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          if (lane == 0) {
            const uint32_t a_addr = smem_u32(smem + stage * kStageBytes);
            const uint32_t b_addr = a_addr + kHalfBytes;
#pragma unroll
            for (int k = 0; k < kBK / 16; ++k)
              mma_pair(d_tmem, sdesc_sw128(a_addr + k * 32, 16, 1024), sdesc_sw128(b_addr + k * 32, 16, 1024), IDESC,
                       (kb > 0 || k > 0) ? 1u : 0u);
            commit_pair(&empty[stage]);
          }
          __syncwarp();
          if (++stage == kStages) {
            stage = 0;
            phase ^= 1u;
          }
        }
        if (!ok) break;
        if (lane == 0) commit_pair(&tfull[buf]);
        __syncwarp();
      }
      if (!ok) {
        *abort_flag = 1;
        if (lane == 0) commit_pair(drain);       // arrives once every MMA issued so far has finished
        __syncwarp();
        wait_cluster(drain, 0, args.err, kErrTimeoutDrain);
      }
    }
  } else {
    // ------------------------------------------------------------------ epilogue (warps 2..5, both CTAs)
    const int q = warp & 3;
    const uint32_t tempty_cl[2] = {map_shared(smem_u32(&tempty[0]), 0), map_shared(smem_u32(&tempty[1]), 0)};
    int it = 0;
    for (int t = first_tile; t < num_tiles; t += tile_step, ++it) {
      int mb, nb;
      tile_of(t, num_mb, num_nb, mb, nb);
      const uint32_t buf = it & 1;
      const uint32_t aphase = (it >> 1) & 1;
      if (*abort_flag || !wait_cluster(&tfull[buf], aphase, args.err, kErrTimeoutEpilogue)) {
        *abort_flag = 1;
        break;
      }
      tc_fence_after();
      const int row = mb * kTileM + (int)rank * 128 + q * 32 + lane;
      const bool row_ok = row < args.M;
      const uint32_t tbase = tmem_base + ((uint32_t)(q * 32) << 16) + buf * kTileN;
      __nv_bfloat16* outp = reinterpret_cast<__nv_bfloat16*>(args.out);
      if constexpr (EPI == kEpiSwiGLU) {
        constexpr int HALF = kTileN / 2;
        const int ncols_out = args.N / 2;
#pragma unroll 1
        for (int c = 0; c < HALF; c += 32) {
          uint32_t g[32], u[32];
          tmem_ld32(tbase + c, g);
          tmem_ld32(tbase + HALF + c, u);
          tmem_wait_ld();
          const int col0 = nb * HALF + c;
          if (!row_ok) continue;
          __nv_bfloat16* dst = outp + (size_t)row * args.ldo + col0;
          if (col0 + 32 <= ncols_out && args.vec_ok) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) {
              uint4 v;
              v.x = pack_bf16x2(silu2(__uint_as_float(g[j])) * __uint_as_float(u[j]),
                                silu2(__uint_as_float(g[j + 1])) * __uint_as_float(u[j + 1]));
              v.y = pack_bf16x2(silu2(__uint_as_float(g[j + 2])) * __uint_as_float(u[j + 2]),
                                silu2(__uint_as_float(g[j + 3])) * __uint_as_float(u[j + 3]));
              v.z = pack_bf16x2(silu2(__uint_as_float(g[j + 4])) * __uint_as_float(u[j + 4]),
                                silu2(__uint_as_float(g[j + 5])) * __uint_as_float(u[j + 5]));
              v.w = pack_bf16x2(silu2(__uint_as_float(g[j + 6])) * __uint_as_float(u[j + 6]),
                                silu2(__uint_as_float(g[j + 7])) * __uint_as_float(u[j + 7]));
              *reinterpret_cast<uint4*>(dst + j) = v;
            }
          } else {
            for (int j = 0; j < 32; ++j)
              if (col0 + j < ncols_out)
                dst[j] = __float2bfloat16(silu2(__uint_as_float(g[j])) * __uint_as_float(u[j]));
          }
        }
      } else {
#pragma unroll 1
        for (int c = 0; c < kTileN; c += 32) {
          uint32_t r[32];
          tmem_ld32(tbase + c, r);
          tmem_wait_ld();
          const int col0 = nb * kTileN + c;
          if (!row_ok || col0 >= args.N) continue;
          const bool full_chunk = col0 + 32 <= args.N;
          __nv_bfloat16* dst = outp + (size_t)row * args.ldo + col0;
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
                const uint4 w = *reinterpret_cast<const uint4*>(res + j);
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
        }
      }
      tc_fence_before();
      arrive_remote(tempty_cl[buf]);
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_barrier();                   // neither CTA leaves while the pair's MMAs or loads may touch its memory
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, 2 * kTileN);
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode2() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

CUtensorMap tmap_rows128(const void* base, uint64_t k, uint64_t rows, uint64_t pitch_elems) {
  if (reinterpret_cast<uintptr_t>(base) % 16 != 0) throw std::runtime_error("TMA base must be 16-byte aligned");
  if ((pitch_elems * 2) % 16 != 0) throw std::runtime_error("TMA row pitch must be a multiple of 16 bytes");
  CUtensorMap tm;
  cuuint64_t dims[2] = {k, rows};
  cuuint64_t strides[1] = {pitch_elems * 2};
  cuuint32_t box[2] = {kBK, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode2()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("cuTensorMapEncodeTiled failed: " + std::to_string((int)r));
  return tm;
}

template <int EPI>
void launch2sm(const GemmOperands& op, const GemmArgs& args, int max_ctas, cudaStream_t stream) {
  auto kernel = gemm2sm_kernel<EPI>;
  static PerDeviceOnce once;
  static int max_clusters[PerDeviceOnce::kMaxDevices] = {0};
  int dev = 0;
  cudaGetDevice(&dev);
  once([kernel, dev] {
    cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemBytes);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(2 * 148, 1, 1);
    cfg.blockDim = dim3(kThreads, 1, 1);
    cfg.dynamicSmemBytes = kSmemBytes;
    cudaLaunchAttribute attr;
    attr.id = cudaLaunchAttributeClusterDimension;
    attr.val.clusterDim.x = 2;
    attr.val.clusterDim.y = 1;
    attr.val.clusterDim.z = 1;
    cfg.attrs = &attr;
    cfg.numAttrs = 1;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kernel, &cfg) != cudaSuccess || n <= 0) {
      cudaGetLastError();
      n = num_sms(dev) / 2;
    }
    if (dev >= 0 && dev < PerDeviceOnce::kMaxDevices) max_clusters[dev] = n;
  });
  int clusters = (dev >= 0 && dev < PerDeviceOnce::kMaxDevices && max_clusters[dev] > 0) ? max_clusters[dev]
                                                                                          : num_sms(dev) / 2;
  const int tiles = ((args.M + kTileM - 1) / kTileM) * ((args.N + kTileN - 1) / kTileN);
  if (tiles < clusters) clusters = tiles;
  if (max_ctas >= 2 && max_ctas / 2 < clusters) clusters = max_ctas / 2;   // leave SMs to a concurrent kernel
  const CUtensorMap ta = tmap_rows128(op.A, args.K, args.M, op.lda);
  const CUtensorMap tb = tmap_rows128(op.B, args.K, args.N, op.ldb);
  kernel<<<2 * clusters, kThreads, kSmemBytes, stream>>>(ta, tb, args);
  count_launch();
}

}  // namespace

bool gemm_2sm_enabled = true;

bool gemm_bf16_2sm(const GemmOperands& op, const GemmArgs& args, int epi, int max_ctas, cudaStream_t stream) {
  if (!gemm_2sm_enabled || op.a_mn || op.b_mn || args.k_splits != 1) return false;
  if (epi != kEpiStore && epi != kEpiSwiGLU) return false;
  if (epi == kEpiSwiGLU && args.N % kTileN != 0) return false;
  if (args.M < kTileM || args.K % 8 != 0) return false;   // small M: the one-SM tiles waste less
  if (max_ctas == 1) return false;
  if (epi == kEpiStore) launch2sm<kEpiStore>(op, args, max_ctas, stream);
  else launch2sm<kEpiSwiGLU>(op, args, max_ctas, stream);
  return true;
}

}  // namespace rf
