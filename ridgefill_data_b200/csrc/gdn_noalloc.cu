// rf_gdn_chunk_scan_noalloc: the chunked gated delta rule (the kernels of gdn.cu) with every piece of
// scratch memory taken from a fixed, file-scope device array instead of the caller's allocator.
//
// This entry point has no counterpart in the reference; it is an addition of this library.
//
// Who needs it: a caller that must not allocate device memory while it runs. Examples are an inference
// server that hands each request a fixed slice of a pre-reserved memory pool and forbids any growth, a
// host runtime with its own allocator that cannot see or free memory taken behind its back, and
// latency-critical loops where cudaMalloc / cudaFree would synchronise the device or fragment the heap.
// Such a caller passes only its inputs, outputs and the recurrent state; nothing is allocated here.
//
// The scratch array (kScratchBytes = 16 MiB, 256-byte aligned) is part of the library image: every GPU
// that loads the library holds it until the process exits. It bounds the problem size: the call needs
//   nv * (n_pad * (dk + dv) + n_chunks * dv * dk + n_pad * dv) * 2 bytes   (output mode)
//   nv * n_pad * (dk + dv) * 2 bytes                                         (fill mode, q == NULL)
// with n_pad = n rounded up to 64 and n_chunks = n_pad / 64; larger calls are rejected with
// RF_NOALLOC_TOO_LARGE before anything is launched.
//
// Host code sees the array's name only as a host-side stand-in, never as a device address: the first
// call on each device (with that device current) resolves the address with cudaGetSymbolAddress and
// caches it. Make that first call before any stream capture begins on the device.
//
// All calls share the one array and it keeps the previous call's contents. Every scratch element the
// kernels read is written earlier in the same call, and the error word is cleared at the start of each
// call; rf_gdn_noalloc_last_error reads it back after the call (gdn_noalloc.h declares the interface).
// Calls that overlap on the GPU (concurrent streams, or several host threads) race on the array: issue
// them one after another.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "gdn_noalloc.h"
#include "kernels.h"

namespace {

constexpr size_t kScratchBytes = size_t(16) << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_gdn_scratch[kScratchBytes];
static __device__ int g_gdn_noalloc_err;

struct DeviceSlot {
  void* scratch = nullptr;
  int* err = nullptr;
};

DeviceSlot g_slots[kMaxDevices];
std::mutex g_slots_mu;

size_t align256(size_t b) { return (b + 255) / 256 * 256; }

}  // namespace

extern "C" {

// Bytes of scratch a call of this shape needs (0 for a shape the kernels do not support).
size_t rf_gdn_noalloc_scratch_bytes(int n, int nk, int nv, int dk, int dv, int output_mode) {
  if (n <= 0 || nk <= 0 || nv <= 0 || dk != 128 || (dv != 64 && dv != 128) || nv % nk != 0) return 0;
  const size_t n_pad = (size_t(n) + 63) / 64 * 64;
  const size_t n_chunks = n_pad / 64;
  size_t bytes = align256(size_t(nv) * n_pad * dk * 2) + align256(size_t(nv) * n_pad * dv * 2);
  if (output_mode) bytes += align256(size_t(nv) * n_chunks * dv * dk * 2) + align256(size_t(nv) * n_pad * dv * 2);
  return bytes;
}

size_t rf_gdn_noalloc_capacity(void) { return kScratchBytes; }

const char* rf_gdn_noalloc_strerror(int status) {
  switch (status) {
    case RF_NOALLOC_OK: return "ok";
    case RF_NOALLOC_BAD_ARGS:
      return "unsupported shape or null pointer (needs dk == 128, dv in {64, 128}, nv a multiple of nk, "
             "k/v/beta/g/state non-null, and q and out both given or both null)";
    case RF_NOALLOC_TOO_LARGE:
      return "the call needs more scratch than the fixed 16 MiB device array holds (see "
             "rf_gdn_noalloc_scratch_bytes); split the sequence into shorter calls";
    case RF_NOALLOC_CUDA_ERROR: return "a CUDA runtime call failed (cudaGetLastError has the cause)";
    case RF_NOALLOC_KERNEL_ERROR:
      return "a kernel of the last call recorded an error code (a timed-out bounded wait, a bad shape or index)";
    default: return "unknown status";
  }
}

// q, k: [nk, n, dk] bf16 (q NULL: fill mode, state only); v: [nv, n, dv] bf16; beta, g: [nv, n] fp32;
// state: [nv, dk, dv] fp32, read and updated in place; out: [n, nv * dv] bf16 with row pitch out_row
// elements (NULL in fill mode). All pointers are device pointers; the work is queued on `stream`.
int rf_gdn_chunk_scan_noalloc(const void* q, const void* k, const void* v, const float* beta, const float* g,
                              float* state, void* out, long out_row, int n, int nk, int nv, int dk, int dv,
                              cudaStream_t stream) {
  const bool output_mode = q != nullptr;
  if (k == nullptr || v == nullptr || beta == nullptr || g == nullptr || state == nullptr ||
      output_mode != (out != nullptr))
    return RF_NOALLOC_BAD_ARGS;
  const size_t need = rf_gdn_noalloc_scratch_bytes(n, nk, nv, dk, dv, output_mode ? 1 : 0);
  if (need == 0) return RF_NOALLOC_BAD_ARGS;
  if (need > kScratchBytes) return RF_NOALLOC_TOO_LARGE;

  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RF_NOALLOC_CUDA_ERROR;
  DeviceSlot slot;
  {
    std::lock_guard<std::mutex> lock(g_slots_mu);
    if (g_slots[dev].scratch == nullptr) {
      void* p = nullptr;
      void* e = nullptr;
      if (cudaGetSymbolAddress(&p, g_gdn_scratch) != cudaSuccess || p == nullptr) return RF_NOALLOC_CUDA_ERROR;
      if (cudaGetSymbolAddress(&e, g_gdn_noalloc_err) != cudaSuccess || e == nullptr) return RF_NOALLOC_CUDA_ERROR;
      g_slots[dev].scratch = p;
      g_slots[dev].err = static_cast<int*>(e);
    }
    slot = g_slots[dev];
  }
  if (cudaMemsetAsync(slot.err, 0, sizeof(int), stream) != cudaSuccess) return RF_NOALLOC_CUDA_ERROR;

  const size_t n_pad = (size_t(n) + 63) / 64 * 64;
  const size_t n_chunks = n_pad / 64;
  unsigned char* base = static_cast<unsigned char*>(slot.scratch);
  size_t off = 0;
  auto take = [&](size_t bytes) {
    void* p = base + off;
    off += align256(bytes);
    return static_cast<__nv_bfloat16*>(p);
  };
  rf::GdnScanArgs a{};
  a.q = static_cast<const __nv_bfloat16*>(q);
  a.k = static_cast<const __nv_bfloat16*>(k);
  a.v = static_cast<const __nv_bfloat16*>(v);
  a.beta = beta;
  a.g = g;
  a.state = state;
  a.out = static_cast<__nv_bfloat16*>(out);
  a.out_row = out_row;
  a.w_buf = take(size_t(nv) * n_pad * dk * 2);
  a.u_buf = take(size_t(nv) * n_pad * dv * 2);
  if (output_mode) {
    a.s_buf = take(size_t(nv) * n_chunks * dv * dk * 2);
    a.vt_buf = take(size_t(nv) * n_pad * dv * 2);
  }
  a.n = n;
  a.nk = nk;
  a.nv = nv;
  a.dk = dk;
  a.dv = dv;
  a.err = slot.err;
  rf::gdn_chunk_scan(a, stream);
  return cudaPeekAtLastError() == cudaSuccess ? RF_NOALLOC_OK : RF_NOALLOC_CUDA_ERROR;
}

int rf_gdn_noalloc_last_error(int* code, cudaStream_t stream) {
  if (code == nullptr) return RF_NOALLOC_BAD_ARGS;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return RF_NOALLOC_CUDA_ERROR;
  int* err = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_slots_mu);
    err = g_slots[dev].err;
  }
  if (err == nullptr) return RF_NOALLOC_BAD_ARGS;
  // a pageable host destination: the copy is staged by the driver, nothing is allocated here
  if (cudaMemcpyAsync(code, err, sizeof(int), cudaMemcpyDeviceToHost, stream) != cudaSuccess ||
      cudaStreamSynchronize(stream) != cudaSuccess)
    return RF_NOALLOC_CUDA_ERROR;
  return *code == 0 ? RF_NOALLOC_OK : RF_NOALLOC_KERNEL_ERROR;
}

}  // extern "C"
