// Row-wise kernels of the prefill path (memory-bound; one pass each):
//   rmsnorm           y = RMSNorm(x) with the plain (HF order: normalise fp32, round, times w) or
//                     zero-centred ((1 + w) in fp32, one rounding) weight
//   head_norm_rope    per (row, head): optional head RMSNorm, rotate-half RoPE on the first `rot` dims from a
//                     bf16 cos/sin table, written head-major (queries, or straight into the K/V cache)
//   gated_rmsnorm     Gated DeltaNet output: per-head RMSNorm, times w, times silu(z)
//   embed_gather      rows of the embedding table
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>

namespace rf {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

// per (4 or 8) consecutive bf16 of a lane as one 8- or 16-byte access when the address allows it, else one by one.
// per is a compile-time constant at every call, so the loops unroll and the arrays stay in registers.
__device__ __forceinline__ void load_bf16(const __nv_bfloat16* p, int per, float (&v)[8]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (per == 8 && (a & 15) == 0) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else if (per == 4 && (a & 7) == 0) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    for (int j = 0; j < per; ++j) v[j] = __bfloat162float(p[j]);
  }
}

__device__ __forceinline__ void store_bf16(__nv_bfloat16* p, int per, const float (&v)[8]) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  if (per == 8 && (a & 15) == 0) {
    uint4 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint4*>(p) = u;
  } else if (per == 4 && (a & 7) == 0) {
    uint2 u;
    __nv_bfloat162* h = reinterpret_cast<__nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) h[i] = __floats2bfloat162_rn(v[2 * i], v[2 * i + 1]);
    *reinterpret_cast<uint2*>(p) = u;
  } else {
    for (int j = 0; j < per; ++j) p[j] = __float2bfloat16(v[j]);
  }
}

// ------------------------------------------------------------------------------------- rmsnorm
// One CTA (256 threads) per row; the row (d <= 8192) is held in registers between the two passes.
template <int MODE>
__global__ void __launch_bounds__(256) rmsnorm_kernel(const __nv_bfloat16* __restrict__ x, long ldx,
                                                      const __nv_bfloat16* __restrict__ w, __nv_bfloat16* __restrict__ y,
                                                      long ldy, int d, float eps) {
  constexpr int MAXV = 4;  // up to 4 x 8 elements per thread: d <= 8192
  const long row = blockIdx.x;
  const __nv_bfloat16* xr = x + row * ldx;
  __nv_bfloat16* yr = y + row * ldy;
  const int nvec = d / 8;
  uint4 buf[MAXV];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = threadIdx.x + j * 256;
    if (v < nvec) {
      buf[j] = *reinterpret_cast<const uint4*>(xr + v * 8);
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&buf[j]);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float f = __bfloat162float(e[q]);
        ss += f * f;
      }
    }
  }
  __shared__ float red[8];
  ss = warp_sum(ss);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < 8 ? red[threadIdx.x] : 0.f;
    v = warp_sum(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)d + eps);
#pragma unroll
  for (int j = 0; j < MAXV; ++j) {
    const int v = threadIdx.x + j * 256;
    if (v < nvec) {
      const __nv_bfloat16* e = reinterpret_cast<const __nv_bfloat16*>(&buf[j]);
      uint4 wv = *reinterpret_cast<const uint4*>(w + v * 8);
      const __nv_bfloat16* we = reinterpret_cast<const __nv_bfloat16*>(&wv);
      uint4 out;
      __nv_bfloat16* oe = reinterpret_cast<__nv_bfloat16*>(&out);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const float f = __bfloat162float(e[q]) * inv;
        if (MODE == 0)
          oe[q] = __float2bfloat16(bfr(f) * __bfloat162float(we[q]));
        else
          oe[q] = __float2bfloat16(f * (1.0f + __bfloat162float(we[q])));
      }
      *reinterpret_cast<uint4*>(yr + v * 8) = out;
    }
  }
}

void rmsnorm(const __nv_bfloat16* x, long ldx, const __nv_bfloat16* w, __nv_bfloat16* y, long ldy, int rows, int d,
             float eps, int zero_centred, cudaStream_t stream) {
  if (rows <= 0) return;
  if (zero_centred)
    rmsnorm_kernel<1><<<rows, 256, 0, stream>>>(x, ldx, w, y, ldy, d, eps);
  else
    rmsnorm_kernel<0><<<rows, 256, 0, stream>>>(x, ldx, w, y, ldy, d, eps);
  count_launch();
}

// ----------------------------------------------------------------------------- head_norm_rope
// One warp per (row, head); head_dim <= 256 (PER = head_dim / 32 elements per lane, a template parameter so that the
// lane's elements live in registers).
template <int PER>
__global__ void __launch_bounds__(256) head_norm_rope_kernel(HeadNormRopeArgs a) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int row = warp / a.n_heads;
  const int head = warp % a.n_heads;
  if (row >= a.n_rows) return;
  const int hd = a.head_dim;
  constexpr int per = PER;  // elements per lane (hd multiple of 32)
  const __nv_bfloat16* src = a.src + (long)row * a.src_row_stride + (long)head * a.src_head_stride;
  // every independent load first (the row, the norm weights, the position and this lane's cos / sin entries), so
  // one memory latency covers them all
  float v[8], wv[8], cv[8], sv[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = wv[j] = cv[j] = sv[j] = 0.f;
  // lane owns elements lane*per .. lane*per+per-1
  load_bf16(src + lane * per, per, v);
  if (a.norm_mode >= 0) load_bf16(a.norm_w + lane * per, per, wv);
  const int h = a.rot / 2;
  if (a.rot > 0 && lane * per < a.rot) {
    const int p = a.pos != nullptr ? __ldg(a.pos + row) : row + a.pos_offset;
    const __nv_bfloat16* cs = a.cos + (long)p * h;
    const __nv_bfloat16* sn = a.sin + (long)p * h;
    // rotate-half pairs i and i +- h share the angle of min(i, i - h); a lane's per elements lie on one side of h
    // (per divides h), so its angles are per consecutive table entries: one vector load each for cos and sin
    const int i0 = lane * per;
    const int t0 = i0 < h ? i0 : i0 - h;
    if (i0 + per <= a.rot) {
      load_bf16(cs + t0, per, cv);
      load_bf16(sn + t0, per, sv);
    } else {
      for (int j = 0; j < per; ++j) {
        if (i0 + j < a.rot) {
          cv[j] = __bfloat162float(cs[t0 + j]);
          sv[j] = __bfloat162float(sn[t0 + j]);
        }
      }
    }
  }
  if (a.norm_mode >= 0) {
    float ss = 0.f;
    for (int j = 0; j < per; ++j) ss += v[j] * v[j];
    ss = warp_sum(ss);
    const float inv = rsqrtf(ss / (float)hd + a.eps);
    for (int j = 0; j < per; ++j) {
      const float f = v[j] * inv;
      v[j] = (a.norm_mode == 0) ? bfr(bfr(f) * wv[j]) : bfr(f * (1.0f + wv[j]));
    }
  }
  if (a.rot > 0) {
    // rotate-half over [0, rot): out[i] = x[i] cos[i] - x[i + h] sin[i] (i < h), out[i] = x[i] cos[i - h] + x[i - h] sin
    float out[8];
    for (int j = 0; j < per; ++j) out[j] = v[j];
    // partner exchange: element i pairs with i +- h; h is a multiple of per when rot % (2*per) == 0
    const int loff = h / per;
    for (int j = 0; j < per; ++j) {
      const int i = lane * per + j;
      const float up = __shfl_down_sync(0xffffffffu, v[j], loff);  // value at i + h
      const float dn = __shfl_up_sync(0xffffffffu, v[j], loff);    // value at i - h
      if (i < a.rot) out[j] = i < h ? bfr(bfr(v[j] * cv[j]) + bfr(-up * sv[j])) : bfr(bfr(v[j] * cv[j]) + bfr(dn * sv[j]));
    }
    for (int j = 0; j < per; ++j) v[j] = out[j];
  }
  __nv_bfloat16* dst;
  if (a.dst_row_from_pos) {
    const int r = a.pos[row];
    if (r < 0 || r >= a.dst_rows) return;   // outside the cache's capacity: nothing written
    dst = a.dst_pages != nullptr
              ? a.dst + (long)a.dst_pages[r / a.page_size] * a.dst_page_stride + (long)head * a.dst_head_stride +
                    (long)(r % a.page_size) * a.dst_row_stride
              : a.dst + (long)head * a.dst_head_stride + (long)r * a.dst_row_stride;
  } else if (a.dst_pages != nullptr) {
    const int r = a.dst_row0 + row;
    dst = a.dst + (long)a.dst_pages[r / a.page_size] * a.dst_page_stride + (long)head * a.dst_head_stride +
          (long)(r % a.page_size) * a.dst_row_stride;
  } else {
    dst = a.dst + (long)head * a.dst_head_stride + (long)row * a.dst_row_stride;
  }
  store_bf16(dst + lane * per, per, v);
}

void head_norm_rope(const HeadNormRopeArgs& a, cudaStream_t stream) {
  if (a.n_rows <= 0 || a.n_heads <= 0) return;
  const long warps = (long)a.n_rows * a.n_heads;
  const int blocks = (int)((warps * 32 + 255) / 256);
  switch (a.head_dim / 32) {
    case 1: head_norm_rope_kernel<1><<<blocks, 256, 0, stream>>>(a); break;
    case 2: head_norm_rope_kernel<2><<<blocks, 256, 0, stream>>>(a); break;
    case 3: head_norm_rope_kernel<3><<<blocks, 256, 0, stream>>>(a); break;
    case 4: head_norm_rope_kernel<4><<<blocks, 256, 0, stream>>>(a); break;
    case 5: head_norm_rope_kernel<5><<<blocks, 256, 0, stream>>>(a); break;
    case 6: head_norm_rope_kernel<6><<<blocks, 256, 0, stream>>>(a); break;
    case 7: head_norm_rope_kernel<7><<<blocks, 256, 0, stream>>>(a); break;
    default: head_norm_rope_kernel<8><<<blocks, 256, 0, stream>>>(a); break;
  }
  count_launch();
}

// ------------------------------------------------------------------------------ gated_rmsnorm
// y[row, head, :] = bf16( bf16(w * bf16(norm(o))) * silu(z) ); one warp per (row, head), dv <= 256. silu(z) on the
// special-function exponential and a fast divide (relative error near 1e-6, far below the bf16 rounding of y).
template <int PER>
__global__ void __launch_bounds__(256) gated_rmsnorm_kernel(const __nv_bfloat16* __restrict__ o, long ldo,
                                                            const __nv_bfloat16* __restrict__ z, long ldz,
                                                            const __nv_bfloat16* __restrict__ w,
                                                            __nv_bfloat16* __restrict__ y, long ldy, int rows,
                                                            int heads, int dv, float eps) {
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int row = warp / heads;
  const int head = warp % heads;
  if (row >= rows) return;
  constexpr int per = PER;
  const __nv_bfloat16* orow = o + (long)row * ldo + head * dv;
  const __nv_bfloat16* zrow = z + (long)row * ldz + head * dv;
  float v[8], zv[8], wv[8];
  load_bf16(orow + lane * per, per, v);
  load_bf16(zrow + lane * per, per, zv);
  load_bf16(w + lane * per, per, wv);
  float ss = 0.f;
  for (int j = 0; j < per; ++j) ss += v[j] * v[j];
  ss = warp_sum(ss);
  const float inv = rsqrtf(ss / (float)dv + eps);
  __nv_bfloat16* yrow = y + (long)row * ldy + head * dv;
  float out[8];
  for (int j = 0; j < per; ++j) {
    const float t = bfr(wv[j] * bfr(v[j] * inv));
    const float zz = zv[j];
    out[j] = t * __fdividef(zz, 1.0f + __expf(-zz));   // silu on the fast exponential, as the GEMM epilogues'
  }
  store_bf16(yrow + lane * per, per, out);
}

void gated_rmsnorm(const __nv_bfloat16* o, long ldo, const __nv_bfloat16* z, long ldz, const __nv_bfloat16* w,
                   __nv_bfloat16* y, long ldy, int rows, int heads, int dv, float eps, cudaStream_t stream) {
  if (rows <= 0) return;
  const long warps = (long)rows * heads;
  switch (dv / 32) {
#define RF_GATED_CASE(P)                                                                                         \
    case P:                                                                                                      \
      gated_rmsnorm_kernel<P><<<(int)((warps * 32 + 255) / 256), 256, 0, stream>>>(o, ldo, z, ldz, w, y, ldy, rows, \
                                                                                  heads, dv, eps);               \
      break;
    RF_GATED_CASE(1)
    RF_GATED_CASE(2)
    RF_GATED_CASE(3)
    RF_GATED_CASE(4)
    RF_GATED_CASE(5)
    RF_GATED_CASE(6)
    RF_GATED_CASE(7)
    default:
      RF_GATED_CASE(8)
#undef RF_GATED_CASE
  }
  count_launch();
}

// ------------------------------------------------------------------------------- embed_gather
// An id outside [0, vocab) records kErrBadIndex and writes a zero row (the host raises on check_errors).
__global__ void embed_gather_kernel(const __nv_bfloat16* __restrict__ table, const int64_t* __restrict__ ids,
                                    __nv_bfloat16* __restrict__ out, int d, long vocab, int* err) {
  const long row = blockIdx.x;
  const long id = ids[row];
  uint4* dst = reinterpret_cast<uint4*>(out + row * (long)d);
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && err != nullptr) atomicMax(err, (int)kErrBadIndex);
    for (int v = threadIdx.x; v < d / 8; v += blockDim.x) dst[v] = make_uint4(0, 0, 0, 0);
    return;
  }
  const uint4* src = reinterpret_cast<const uint4*>(table + id * (long)d);
  for (int v = threadIdx.x; v < d / 8; v += blockDim.x) dst[v] = src[v];
}

void embed_gather(const __nv_bfloat16* table, const int64_t* ids, __nv_bfloat16* out, int rows, int d, long vocab,
                  cudaStream_t stream, int* err) {
  if (rows <= 0) return;
  embed_gather_kernel<<<rows, 128, 0, stream>>>(table, ids, out, d, vocab, err);
  count_launch();
}

// ------------------------------------------------------------------------------------ host-side error records
__global__ void record_error_kernel(int* err, int code) { record_error(err, code); }

void record_error_async(int* err, int code, cudaStream_t stream) {
  if (err == nullptr) return;
  record_error_kernel<<<1, 1, 0, stream>>>(err, code);
  count_launch();
}

}  // namespace rf
