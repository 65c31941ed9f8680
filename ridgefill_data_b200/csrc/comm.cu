// Peer-memory collectives over NVLink for tensor parallelism (one rank per GPU, CUDA IPC mappings).
//
//  signal         one thread: system fence, then a release store of `value` into slot `slot` of every peer's
//                 flag array (the producer's data stores to those peers happened before: same stream)
//  reduce_rows    the owner of a row block waits (bounded) until every rank has signalled its partial, sums the
//                 n_peers bf16 partial slots in fp32 plus the optional residual, writes the reduced rows to its
//                 own buffer, and the last CTA signals "reduced" to every peer
//  gather_rows    every rank waits (bounded) for each owner's "reduced" flag and pulls that owner's rows over
//                 NVLink into its own output tensor
//  wait_flags     a one-CTA bounded wait until slots [first, first + n) all hold `value`
// Every wait is bounded by kCommWaitNs of wall time; a timeout records kErrTimeoutPeer in the error word and the
// kernel returns without touching the data, so the host can raise instead of hanging the GPU.
#include "kernels.h"
#include "ptx.cuh"
#include "comm.cuh"

#include <cstring>
#include <stdexcept>
#include <string>

namespace rf {

__global__ void signal_kernel(PeerFlags f, int slot, int value) {
  if (threadIdx.x == 0 && blockIdx.x == 0) {
    __threadfence_system();
    for (int q = 0; q < f.n; ++q) st_release_sys(f.ptr[q] + slot, value);
  }
}

void comm_signal(const PeerFlags& f, int slot, int value, cudaStream_t stream) {
  signal_kernel<<<1, 32, 0, stream>>>(f, slot, value);
  count_launch();
}

__global__ void wait_flags_kernel(const int* flags, int first, int n, int value, int* err, uint64_t limit_ns) {
  if (threadIdx.x < n) wait_value(flags + first + threadIdx.x, value, err, limit_ns);
  __syncthreads();
}

void comm_wait(const int* flags, int first, int n, int value, int* err, cudaStream_t stream, uint64_t limit_ns) {
  if (n > 32) throw std::runtime_error("comm_wait: at most 32 flags per call");
  wait_flags_kernel<<<1, 32, 0, stream>>>(flags, first, n, value, err, limit_ns ? limit_ns : kCommWaitNs);
  count_launch();
}

// grid: (ceil(rows / 8) CTAs of 256 threads; each warp reduces one row of d elements.
__global__ void __launch_bounds__(256) reduce_rows_kernel(ReduceRowsArgs a) {
  __shared__ int ok;
  if (threadIdx.x == 0) {
    bool good = true;
    for (int s = 0; s < a.n_peers && good; ++s) good = wait_value(a.flags + a.arrive_slot + s, a.value, a.err);
    ok = good ? 1 : 0;
  }
  __syncthreads();
  if (ok) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row = blockIdx.x * 8 + warp;
    if (row < a.rows) {
      for (int c = lane * 8; c < a.d; c += 256) {
        float acc[8];
        if (a.residual != nullptr) {
          uint4 rv = *reinterpret_cast<const uint4*>(a.residual + (size_t)row * a.ld_res + c);
          const __nv_bfloat16* re = reinterpret_cast<const __nv_bfloat16*>(&rv);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = __bfloat162float(re[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] = 0.f;
        }
        for (int s = 0; s < a.n_peers; ++s) {
          uint4 pv = *reinterpret_cast<const uint4*>(a.recv + (size_t)s * a.slot_stride + (size_t)row * a.d + c);
          const __nv_bfloat16* pe = reinterpret_cast<const __nv_bfloat16*>(&pv);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += __bfloat162float(pe[j]);
        }
        uint4 o;
        o.x = pack_bf16x2(acc[0], acc[1]);
        o.y = pack_bf16x2(acc[2], acc[3]);
        o.z = pack_bf16x2(acc[4], acc[5]);
        o.w = pack_bf16x2(acc[6], acc[7]);
        *reinterpret_cast<uint4*>(a.red + (size_t)row * a.d + c) = o;
      }
    }
  }
  // the last CTA to finish announces the reduced rows to every rank
  __syncthreads();
  if (threadIdx.x == 0) {
    __threadfence();
    const int done = atomicAdd(a.counter, 1);
    if (done == (int)gridDim.x - 1) {
      *a.counter = 0;
      if (!ok) return;
      __threadfence_system();
      for (int q = 0; q < a.n_peers; ++q) st_release_sys(a.peer_flags.ptr[q] + a.reduced_slot + a.my_rank, a.value);
    }
  }
}

void comm_reduce_rows(const ReduceRowsArgs& a, cudaStream_t stream) {
  const int blocks = a.rows > 0 ? (a.rows + 7) / 8 : 1;
  reduce_rows_kernel<<<blocks, 256, 0, stream>>>(a);
  count_launch();
}

// grid: (row blocks of 8 rows, n_peers owners); block 256: each warp copies one row from the owner's buffer.
__global__ void __launch_bounds__(256) gather_rows_kernel(GatherRowsArgs a) {
  const int q = blockIdx.y;
  __shared__ int ok;
  if (threadIdx.x == 0) ok = wait_value(a.flags + a.reduced_slot + q, a.value, a.err) ? 1 : 0;
  __syncthreads();
  if (!ok) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int r = blockIdx.x * 8 + warp;
  if (r >= a.row_chunk) return;
  const int row = q * a.row_chunk + r;
  if (row >= a.total_rows) return;
  const __nv_bfloat16* src = a.peer_red[q] + (size_t)r * a.d;
  __nv_bfloat16* dst = a.out + (size_t)row * a.ld_out;
  for (int c = lane * 8; c < a.d; c += 256)
    *reinterpret_cast<uint4*>(dst + c) = *reinterpret_cast<const uint4*>(src + c);
}

void comm_gather_rows(const GatherRowsArgs& a, cudaStream_t stream) {
  dim3 grid((a.row_chunk + 7) / 8, a.n_peers);
  if (a.row_chunk <= 0) grid.x = 1;
  gather_rows_kernel<<<grid, 256, 0, stream>>>(a);
  count_launch();
}

// ---------------------------------------------------------------------------- CUDA IPC plumbing
void* ipc_malloc(size_t bytes) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) throw std::runtime_error(std::string("ipc_malloc: ") + cudaGetErrorString(e));
  cudaMemset(p, 0, bytes);
  return p;
}

void ipc_free(void* p) { cudaFree(p); }

std::string ipc_handle(void* p) {
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcGetMemHandle: ") + cudaGetErrorString(e));
  return std::string(reinterpret_cast<const char*>(&h), sizeof(h));
}

void* ipc_open(const std::string& handle) {
  if (handle.size() != sizeof(cudaIpcMemHandle_t)) throw std::runtime_error("ipc_open: bad handle size");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle.data(), sizeof(h));
  void* p = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) throw std::runtime_error(std::string("cudaIpcOpenMemHandle: ") + cudaGetErrorString(e));
  return p;
}

void ipc_close(void* p) { cudaIpcCloseMemHandle(p); }

}  // namespace rf
