// Collectives through NVSwitch multicast (NVLS): multimem loads that reduce in the switch and multimem stores
// that the switch replicates to every GPU. The buffers are symmetric allocations bound to one multicast object:
// an offset in the multicast range addresses that offset in every rank's buffer at once.
//
//  nvls_allreduce     one-shot all-reduce of bf16 rows. Each rank owns rows [row0, row1): it reads them reduced
//                     over all ranks (multimem.ld_reduce, fp32 accumulation in the switch) and writes the sums to
//                     every rank's output buffer (multimem.st). Per GPU that moves ~S out and ~S in (S = the
//                     tensor's bytes) against 2 (N - 1) / N S each way for a ring. A cross-rank barrier before (every
//                     rank's partial written) and after (every rank's sums landed), then every CTA copies the
//                     gathered rows into the caller's fresh output tensor.
//  nvls_allreduce_f64 one-shot all-reduce of an fp64 vector (the ridge fit's sufficient statistics): rank r reads
//                     elements [r n / N, (r + 1) n / N) summed in the switch (multimem.ld_reduce .f64, exact
//                     fp64 adds) and multicasts the sums; barriers as above.
//  nvls_allgather     each rank's column slice [rows, cols] of a [rows, d] tensor written into every rank's copy at
//                     column offset rank * cols by one multimem.st per 16 bytes, then a cross-rank barrier.
// Barriers are epoch-stamped flag words in a symmetric int32 array, written with st.release.sys to every peer's
// copy and polled locally with ld.acquire.sys; every wait is bounded (kCommWaitNs) and a timeout records
// kErrTimeoutPeer and skips the data movement. The grid never exceeds one CTA per SM, so all CTAs are resident
// while they wait.
#include "gemm.h"
#include "kernels.h"
#include "comm.cuh"

#include <algorithm>

namespace rf {

constexpr int kNvlsThreads = 512;
constexpr int kNvlsUnroll = 4;

template <bool ACC32>
__device__ __forceinline__ void mm_ld_reduce_bf16x8(const void* mc, uint4& v) {
  if constexpr (ACC32)
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.acc::f32.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(mc)
                 : "memory");
  else
    asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.bf16x2 {%0, %1, %2, %3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(mc)
                 : "memory");
}
__device__ __forceinline__ void mm_st_16(void* mc, const uint4& v) {
  asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(mc), "r"(v.x), "r"(v.y),
               "r"(v.z), "r"(v.w)
               : "memory");
}

// CTA 0 / thread 0 announces `epoch` in slot `slot` of every rank's flag array.
__device__ __forceinline__ void arrive(const NvlsFlags& f, int slot, int epoch) {
  __threadfence_system();
  for (int q = 0; q < f.world; ++q) st_release_sys(f.peer[q] + slot * kMaxRanksNvls + f.rank, epoch);
}

// thread 0 of the calling CTA waits for every rank's `epoch` in slot `slot` of the local flags; returns false on
// timeout. The result is broadcast through shared memory.
__device__ bool wait_all(const NvlsFlags& f, int slot, int epoch, int* err, int* s_ok) {
  if (threadIdx.x == 0) {
    bool ok = true;
    for (int q = 0; q < f.world && ok; ++q) ok = wait_value(f.local + slot * kMaxRanksNvls + q, epoch, err);
    *s_ok = ok ? 1 : 0;
    __threadfence();
  }
  __syncthreads();
  return *s_ok != 0;
}

// The last CTA to get here announces `epoch` in `slot` to every rank (all CTAs' stores fenced first).
__device__ void last_cta_arrive(const NvlsFlags& f, int slot, int epoch, int* counter) {
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence_system();
    if (atomicAdd(counter, 1) == (int)gridDim.x - 1) {
      *counter = 0;
      arrive(f, slot, epoch);
    }
  }
}

template <bool ACC32>
__global__ void __launch_bounds__(kNvlsThreads) nvls_allreduce_kernel(NvlsAllReduceArgs a) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x == 0) arrive(a.f, a.slot_in, a.epoch);
  const bool ok = wait_all(a.f, a.slot_in, a.epoch, a.err, &s_ok);
  const int units_row = a.d / 8;
  if (ok) {
    const long n_units = (long)(a.row1 - a.row0) * units_row;
    const long base = (long)a.row0 * units_row;
    const long stride = (long)gridDim.x * blockDim.x;
    const char* in = reinterpret_cast<const char*>(a.mc_in);
    char* out = reinterpret_cast<char*>(a.mc_out);
    for (long u0 = (long)blockIdx.x * blockDim.x + threadIdx.x; u0 < n_units; u0 += stride * kNvlsUnroll) {
      uint4 v[kNvlsUnroll];
#pragma unroll
      for (int k = 0; k < kNvlsUnroll; ++k) {
        const long u = u0 + k * stride;
        if (u < n_units) mm_ld_reduce_bf16x8<ACC32>(in + (base + u) * 16, v[k]);
      }
#pragma unroll
      for (int k = 0; k < kNvlsUnroll; ++k) {
        const long u = u0 + k * stride;
        if (u < n_units) mm_st_16(out + (base + u) * 16, v[k]);
      }
    }
  }
  last_cta_arrive(a.f, a.slot_out, a.epoch, a.counter);
  const bool done = ok && wait_all(a.f, a.slot_out, a.epoch, a.err, &s_ok);
  if (!done || a.dst == nullptr) return;
  // every rank's sums are in the local output buffer: copy all rows into the caller's tensor
  const long n16 = (long)a.rows * units_row;
  const uint4* src = reinterpret_cast<const uint4*>(a.out_local);
  uint4* dst = reinterpret_cast<uint4*>(a.dst);
  for (long u = (long)blockIdx.x * blockDim.x + threadIdx.x; u < n16; u += (long)gridDim.x * blockDim.x) dst[u] = src[u];
}

__global__ void __launch_bounds__(kNvlsThreads) nvls_allgather_kernel(NvlsAllGatherArgs a) {
  __shared__ int s_ok;
  const int units_row = a.cols / 8;
  const long n_units = (long)a.rows * units_row;
  const long stride = (long)gridDim.x * blockDim.x;
  char* out = reinterpret_cast<char*>(a.mc_out);
  for (long u = (long)blockIdx.x * blockDim.x + threadIdx.x; u < n_units; u += stride) {
    const long r = u / units_row, c = (u % units_row) * 8;
    const uint4 v = *reinterpret_cast<const uint4*>(a.src + r * a.ld_src + c);
    mm_st_16(out + ((r * a.d) + a.col_off + c) * 2, v);
  }
  last_cta_arrive(a.f, a.slot, a.epoch, a.counter);
  if (blockIdx.x == 0) wait_all(a.f, a.slot, a.epoch, a.err, &s_ok);
}

__global__ void __launch_bounds__(kNvlsThreads) nvls_allreduce_f64_kernel(NvlsAllReduceF64Args a) {
  __shared__ int s_ok;
  if (blockIdx.x == 0 && threadIdx.x == 0) arrive(a.f, a.slot_in, a.epoch);
  const bool ok = wait_all(a.f, a.slot_in, a.epoch, a.err, &s_ok);
  if (ok) {
    const long per = (a.n + a.f.world - 1) / a.f.world;
    const long i0 = (long)a.f.rank * per, i1 = min(a.n, i0 + per);
    const long stride = (long)gridDim.x * blockDim.x;
    const double* in = reinterpret_cast<const double*>(a.mc_in);
    double* out = reinterpret_cast<double*>(a.mc_out);
    for (long u0 = i0 + (long)blockIdx.x * blockDim.x + threadIdx.x; u0 < i1; u0 += stride * kNvlsUnroll) {
      double v[kNvlsUnroll];
#pragma unroll
      for (int k = 0; k < kNvlsUnroll; ++k) {
        const long u = u0 + k * stride;
        if (u < i1)
          asm volatile("multimem.ld_reduce.relaxed.sys.global.add.f64 %0, [%1];" : "=d"(v[k]) : "l"(in + u) : "memory");
      }
#pragma unroll
      for (int k = 0; k < kNvlsUnroll; ++k) {
        const long u = u0 + k * stride;
        if (u < i1) asm volatile("multimem.st.relaxed.sys.global.f64 [%0], %1;" ::"l"(out + u), "d"(v[k]) : "memory");
      }
    }
  }
  last_cta_arrive(a.f, a.slot_out, a.epoch, a.counter);
  if (ok) wait_all(a.f, a.slot_out, a.epoch, a.err, &s_ok);
}

__global__ void nvls_barrier_kernel(NvlsFlags f, int slot, int epoch, int* err) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) arrive(f, slot, epoch);
  wait_all(f, slot, epoch, err, &s_ok);
}

static int grid_for(long units, int device) {
  const long want = (units + kNvlsThreads - 1) / kNvlsThreads;
  return (int)std::max(1L, std::min<long>(want, num_sms(device)));
}

void nvls_allreduce(const NvlsAllReduceArgs& a, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long units = std::max((long)(a.row1 - a.row0) * (a.d / 8), (long)a.rows * (a.d / 8) / kNvlsUnroll);
  int grid = grid_for(units / kNvlsUnroll + 1, dev);
  if (a.max_ctas > 0) grid = std::min(grid, a.max_ctas);
  if (a.acc32)
    nvls_allreduce_kernel<true><<<grid, kNvlsThreads, 0, stream>>>(a);
  else
    nvls_allreduce_kernel<false><<<grid, kNvlsThreads, 0, stream>>>(a);
  count_launch();
}

void nvls_allreduce_f64(const NvlsAllReduceF64Args& a, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  const long mine = (a.n + a.f.world - 1) / a.f.world;
  nvls_allreduce_f64_kernel<<<grid_for(mine / kNvlsUnroll + 1, dev), kNvlsThreads, 0, stream>>>(a);
  count_launch();
}

void nvls_allgather(const NvlsAllGatherArgs& a, cudaStream_t stream) {
  int dev = 0;
  cudaGetDevice(&dev);
  nvls_allgather_kernel<<<grid_for((long)a.rows * (a.cols / 8), dev), kNvlsThreads, 0, stream>>>(a);
  count_launch();
}

void nvls_barrier(const NvlsFlags& f, int slot, int epoch, int* err, cudaStream_t stream) {
  nvls_barrier_kernel<<<1, 32, 0, stream>>>(f, slot, epoch, err);
  count_launch();
}

}  // namespace rf
