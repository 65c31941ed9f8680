// C interface of the allocation-free Gated DeltaNet chunk scan (gdn_noalloc.cu).
//
// This interface has no counterpart in the reference; it is an addition of this library. It serves callers
// that may not allocate device memory while they run; gdn_noalloc.cu says who they are and how the fixed
// scratch array behaves (its size limit, its per-device set-up on the first call, and why overlapping calls race).
#pragma once
#include <cstddef>
#include <cuda_runtime.h>

#ifdef __cplusplus
extern "C" {
#endif

enum RfNoAllocStatus {
  RF_NOALLOC_OK = 0,
  RF_NOALLOC_BAD_ARGS = 1,      // unsupported shape or a missing pointer; nothing was queued
  RF_NOALLOC_TOO_LARGE = 2,     // the shape needs more scratch than the fixed array holds; nothing was queued
  RF_NOALLOC_CUDA_ERROR = 3,    // a CUDA runtime call failed (cudaGetLastError has the cause)
  RF_NOALLOC_KERNEL_ERROR = 4,  // rf_gdn_noalloc_last_error: a kernel of the last call recorded an error code
};

// Bytes of scratch one call of this shape needs (0 for a shape the kernels do not support).
size_t rf_gdn_noalloc_scratch_bytes(int n, int nk, int nv, int dk, int dv, int output_mode);

// Size of the fixed scratch array (the largest value rf_gdn_noalloc_scratch_bytes may return for a call to run).
size_t rf_gdn_noalloc_capacity(void);

// A short English description of a status code.
const char* rf_gdn_noalloc_strerror(int status);

// The chunked gated delta rule over n tokens. q, k: [nk, n, dk] bf16 (q NULL: fill mode, state only);
// v: [nv, n, dv] bf16; beta, g: [nv, n] fp32; state: [nv, dk, dv] fp32, read and updated in place;
// out: [n, nv * dv] bf16 with row pitch out_row elements (NULL in fill mode). Device pointers; the work is
// queued on `stream` and the call returns without waiting for it.
int rf_gdn_chunk_scan_noalloc(const void* q, const void* k, const void* v, const float* beta, const float* g,
                              float* state, void* out, long out_row, int n, int nk, int nv, int dk, int dv,
                              cudaStream_t stream);

// Waits for `stream`, then stores in *code the error code the kernels of the last call on the current device
// recorded (0: none; 1-7: a timed-out bounded wait, an unsupported shape, a bad index). Returns RF_NOALLOC_OK
// when *code is 0, RF_NOALLOC_KERNEL_ERROR when it is not, RF_NOALLOC_CUDA_ERROR when the read failed, and
// RF_NOALLOC_BAD_ARGS when code is NULL or no call has run on this device yet.
int rf_gdn_noalloc_last_error(int* code, cudaStream_t stream);

#ifdef __cplusplus
}
#endif
