// Warp-level bf16 MMA helpers (m16n8k16, fp32 accumulate) and ldmatrix fragment loaders for the
// small per-warp tiles of the flash-attention and Gated DeltaNet kernels.
//
// Fragment layout of mma.m16n8k16 (g = lane / 4, t = lane % 4):
//   A (16x16): a0 (g, 2t..2t+1)  a1 (g+8, 2t..)  a2 (g, 2t+8..)  a3 (g+8, 2t+8..)
//   B (16x8):  b0 (k 2t..2t+1, n g)  b1 (k 2t+8.., n g)
//   C (16x8):  c0,c1 (g, 2t..2t+1)  c2,c3 (g+8, 2t..2t+1)
// Shared-memory tiles are row-major with a pitch in elements (pad rows by 8 to avoid bank conflicts).
#pragma once
#include <cuda_bf16.h>
#include <cstdint>

namespace rf {

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void mma_bf16(float (&c)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// A fragment of rows [r0, r0+16) x cols [k0, k0+16) of a row-major [M][K] bf16 tile.
__device__ __forceinline__ void lda_row(uint32_t (&a)[4], const __nv_bfloat16* base, int pitch, int r0, int k0,
                                        int lane) {
  const __nv_bfloat16* p = base + (size_t)(r0 + (lane & 15)) * pitch + k0 + (lane >> 4) * 8;
  ldsm_x4(static_cast<uint32_t>(__cvta_generic_to_shared(p)), a[0], a[1], a[2], a[3]);
}

// A fragment (m [m0, m0+16) x k [k0, k0+16)) of A = X^T where X is a row-major [K][M] tile.
__device__ __forceinline__ void lda_trans(uint32_t (&a)[4], const __nv_bfloat16* base, int pitch, int m0, int k0,
                                          int lane) {
  const int k = k0 + (lane & 7) + (lane >> 4) * 8;
  const int m = m0 + ((lane >> 3) & 1) * 8;
  const __nv_bfloat16* p = base + (size_t)k * pitch + m;
  ldsm_x4_t(static_cast<uint32_t>(__cvta_generic_to_shared(p)), a[0], a[1], a[2], a[3]);
}

// B fragments of two adjacent n-tiles (n [n0, n0+16)) x k [k0, k0+16) where B[k][n] = X[n][k] and X is
// row-major [N][K] (e.g. K-rows of attention keys). b[0..1]: n-tile n0, b[2..3]: n-tile n0+8.
__device__ __forceinline__ void ldb_nk(uint32_t (&b)[4], const __nv_bfloat16* base, int pitch, int n0, int k0,
                                       int lane) {
  const int n = n0 + (lane & 7) + (lane >> 4) * 8;
  const int k = k0 + ((lane >> 3) & 1) * 8;
  const __nv_bfloat16* p = base + (size_t)n * pitch + k;
  ldsm_x4(static_cast<uint32_t>(__cvta_generic_to_shared(p)), b[0], b[1], b[2], b[3]);
}

// B fragments of two adjacent n-tiles where B is a row-major [K][N] tile (e.g. V rows, the state).
__device__ __forceinline__ void ldb_kn(uint32_t (&b)[4], const __nv_bfloat16* base, int pitch, int n0, int k0,
                                       int lane) {
  const int k = k0 + (lane & 7) + ((lane >> 3) & 1) * 8;
  const int n = n0 + (lane >> 4) * 8;
  const __nv_bfloat16* p = base + (size_t)k * pitch + n;
  ldsm_x4_t(static_cast<uint32_t>(__cvta_generic_to_shared(p)), b[0], b[1], b[2], b[3]);
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&v);
}

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int sz = pred ? 16 : 0;
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

}  // namespace rf
