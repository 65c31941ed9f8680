// One decode row of an attention layer for R sequences in two launches: the K/V append, the q and k head norm +
// RoPE and the attention over each sequence's cache, in place of four launches per sequence (two K/V writes, the
// query's norm + RoPE, and a 128-row tcgen05 flash tile that holds one live query row).
//
// decode_attn_kernel     grid (key split, KV head, sequence), 4 warps. The CTA owns the G = hq / hkv query heads of
//                        its KV head and keys [s L, min((s + 1) L, p + 1)) of the sequence, p being the sequence's
//                        position (read on the device: a CUDA graph of the step replays for every step) and
//                        L = 64 ceil((p + 1) / 4096) keys per split, so at most kDecSplits = 64 splits hold keys and the
//                        split of the keys depends on p alone (not on the cache's capacity, its pages or the batch:
//                        contiguous and paged caches, alone or batched, give the same bits). Its warps
//                        first compute the query heads' norm + RoPE from the projected row; the CTA whose split holds
//                        row p also computes the new key (norm + RoPE) and value, writes them into the cache at row p
//                        (contiguous buffers or the pages of a pool) and uses them from shared memory, so no CTA reads
//                        a row another one writes. Then each warp takes every 4th key: a lane holds hd / 32
//                        consecutive elements of the key, the value and each query, the G dot products are summed
//                        across the warp, and the warp keeps an online softmax (running max, sum and weighted values)
//                        per head. The 4 warps' states merge in warp order into the split's partial (max, sum,
//                        unnormalised output) in fp32.
// decode_combine_kernel  grid (query head, sequence), hd threads: the splits' partials merged in split order, divided
//                        by the sum, times sigmoid(gate) for gated attention, rounded to bf16.
//
// The norm + RoPE arithmetic is head_norm_rope's (norm.cu): the same per-lane layout, warp sum and roundings, so a
// row the decode step writes has the bits the prefill's K writer would give it. No spin waits and no tensor-core
// state: a decode row is bound by reading the cache, one pass over K and V per KV head.
#include "kernels.h"
#include "ptx.cuh"

#include <cuda_bf16.h>
#include <stdexcept>

namespace rf {

namespace {

constexpr int kDecWarps = 4;

__device__ __forceinline__ int split_keys(int p) { return 64 * max(1, (p + 1 + 4095) / 4096); }

__device__ __forceinline__ float dec_warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float dec_bfr(float x) { return __bfloat162float(__float2bfloat16(x)); }

template <int PER>
__device__ __forceinline__ void load_row(const __nv_bfloat16* p, float (&v)[PER]) {
  if constexpr (PER == 8) {
    const uint4 u = *reinterpret_cast<const uint4*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else if constexpr (PER == 4) {
    const uint2 u = *reinterpret_cast<const uint2*>(p);
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int i = 0; i < 2; ++i) {
      const float2 f = __bfloat1622float2(h[i]);
      v[2 * i] = f.x;
      v[2 * i + 1] = f.y;
    }
  } else {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(p));
    v[0] = f.x;
    v[1] = f.y;
  }
}

// Head norm (mode -1 none, 0 plain, 1 zero-centred) + rotate-half RoPE over [0, rot) at position p of one head
// row, lane owning elements lane * PER .. + PER - 1 (the layout and arithmetic of head_norm_rope_kernel).
template <int PER>
__device__ __forceinline__ void norm_rope_lane(const __nv_bfloat16* src, const __nv_bfloat16* w, int mode, float eps,
                                               const __nv_bfloat16* cos, const __nv_bfloat16* sin, int rot, int p,
                                               int lane, float (&v)[PER]) {
  constexpr int HD = 32 * PER;
  float wv[PER], cv[PER], sv[PER];
#pragma unroll
  for (int j = 0; j < PER; ++j) wv[j] = cv[j] = sv[j] = 0.f;
  load_row<PER>(src + lane * PER, v);
  if (mode >= 0) load_row<PER>(w + lane * PER, wv);
  const int h = rot / 2;
  const int i0 = lane * PER;
  if (rot > 0 && i0 < rot) {
    const int t0 = i0 < h ? i0 : i0 - h;
#pragma unroll
    for (int j = 0; j < PER; ++j)
      if (i0 + j < rot) {
        cv[j] = __bfloat162float(cos[(long)p * h + t0 + j]);
        sv[j] = __bfloat162float(sin[(long)p * h + t0 + j]);
      }
  }
  if (mode >= 0) {
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) ss += v[j] * v[j];
    ss = dec_warp_sum(ss);
    const float inv = rsqrtf(ss / (float)HD + eps);
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const float f = v[j] * inv;
      v[j] = mode == 0 ? dec_bfr(dec_bfr(f) * wv[j]) : dec_bfr(f * (1.0f + wv[j]));
    }
  }
  if (rot > 0) {
    const int loff = h / PER;
    float out[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int i = i0 + j;
      const float up = __shfl_down_sync(0xffffffffu, v[j], loff);
      const float dn = __shfl_up_sync(0xffffffffu, v[j], loff);
      out[j] = v[j];
      if (i < rot)
        out[j] = i < h ? dec_bfr(dec_bfr(v[j] * cv[j]) + dec_bfr(-up * sv[j]))
                       : dec_bfr(dec_bfr(v[j] * cv[j]) + dec_bfr(dn * sv[j]));
    }
#pragma unroll
    for (int j = 0; j < PER; ++j) v[j] = out[j];
  }
}

// element offset of cache row j of KV head g for sequence slot sq
__device__ __forceinline__ long cache_row(const DecodeAttnArgs& a, int sq, int g, int j, int hd) {
  if (a.pages[sq] != nullptr)
    return (long)a.pages[sq][j / a.page_size] * a.page_stride + (long)g * a.head_stride[sq] +
           (long)(j % a.page_size) * hd;
  return (long)g * a.head_stride[sq] + (long)j * hd;
}

template <int PER, int G>
__global__ void __launch_bounds__(kDecWarps * 32) decode_attn_kernel(DecodeAttnArgs a, int r0) {
  constexpr int HD = 32 * PER;
  __shared__ float qs[G][HD];
  __shared__ float kn[HD], vn[HD];
  __shared__ float accs[kDecWarps][G][HD];
  __shared__ float ms[kDecWarps][G], ls[kDecWarps][G];
  const int s = blockIdx.x, g = blockIdx.y, sq = blockIdx.z, r = r0 + sq;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int p = a.pos[r];
  if (p < 0 || p >= a.rows[sq]) {   // no room for the row: nothing written (the combine writes zeros)
    if (s == 0 && g == 0 && threadIdx.x == 0) record_error(a.err, kErrBadIndex);
    return;
  }
  const int L = split_keys(p);
  const int start = s * L;
  if (start > p) return;
  const int end = min(start + L, p + 1);
  const bool own = p < start + L;
  const __nv_bfloat16* row = a.qkv + (long)r * a.qkv_row;
  const int qstride = a.gated ? 2 * HD : HD;
  const int qw = a.hq * qstride;
  for (int hh = warp; hh < G; hh += kDecWarps) {
    float v[PER];
    norm_rope_lane<PER>(row + (long)(g * G + hh) * qstride, a.q_norm, a.norm_mode, a.eps, a.cos, a.sin, a.rot, p,
                        lane, v);
#pragma unroll
    for (int j = 0; j < PER; ++j) qs[hh][lane * PER + j] = v[j];
  }
  if (own && warp < 2) {
    float v[PER];
    if (warp == 0)
      norm_rope_lane<PER>(row + qw + (long)g * HD, a.k_norm, a.norm_mode, a.eps, a.cos, a.sin, a.rot, p, lane, v);
    else
      norm_rope_lane<PER>(row + qw + (long)(a.hkv + g) * HD, nullptr, -1, 0.f, nullptr, nullptr, 0, p, lane, v);
    __nv_bfloat16* dst = (warp == 0 ? a.k[sq] : a.v[sq]) + cache_row(a, sq, g, p, HD) + lane * PER;
    float* sh = warp == 0 ? kn : vn;
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      dst[j] = __float2bfloat16(v[j]);
      sh[lane * PER + j] = v[j];
    }
  }
  __syncthreads();
  float q[G][PER];
#pragma unroll
  for (int hh = 0; hh < G; ++hh)
#pragma unroll
    for (int j = 0; j < PER; ++j) q[hh][j] = qs[hh][lane * PER + j];
  float m[G], l[G], acc[G][PER];
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    m[hh] = -INFINITY;
    l[hh] = 0.f;
#pragma unroll
    for (int j = 0; j < PER; ++j) acc[hh][j] = 0.f;
  }
  const __nv_bfloat16* kb = a.k[sq];
  const __nv_bfloat16* vb = a.v[sq];
  // keys j0 and j0 + 4 per step: both rows' loads issued before either is used
  for (int j0 = start + warp; j0 < end; j0 += 2 * kDecWarps) {
    float kf[2][PER], vf[2][PER];
    bool live[2];
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u * kDecWarps;
      live[u] = j < end;
      if (!live[u] || j == p) continue;
      const long off = cache_row(a, sq, g, j, HD) + lane * PER;
      load_row<PER>(kb + off, kf[u]);
      load_row<PER>(vb + off, vf[u]);
    }
#pragma unroll
    for (int u = 0; u < 2; ++u) {
      const int j = j0 + u * kDecWarps;
      if (!live[u]) break;
      if (j == p) {
#pragma unroll
        for (int e = 0; e < PER; ++e) {
          kf[u][e] = kn[lane * PER + e];
          vf[u][e] = vn[lane * PER + e];
        }
      }
#pragma unroll
      for (int hh = 0; hh < G; ++hh) {
        float d = 0.f;
#pragma unroll
        for (int e = 0; e < PER; ++e) d = fmaf(q[hh][e], kf[u][e], d);
        const float sc = dec_warp_sum(d) * a.scale_log2;
        const float mn = fmaxf(m[hh], sc);
        const float corr = exp2f(m[hh] - mn);
        const float pj = exp2f(sc - mn);
        l[hh] = fmaf(l[hh], corr, pj);
#pragma unroll
        for (int e = 0; e < PER; ++e) acc[hh][e] = fmaf(pj, vf[u][e], acc[hh][e] * corr);
        m[hh] = mn;
      }
    }
  }
#pragma unroll
  for (int hh = 0; hh < G; ++hh) {
    if (lane == 0) {
      ms[warp][hh] = m[hh];
      ls[warp][hh] = l[hh];
    }
#pragma unroll
    for (int e = 0; e < PER; ++e) accs[warp][hh][lane * PER + e] = acc[hh][e];
  }
  __syncthreads();
  const long base = (((long)r * a.hkv + g) * kDecSplits + s) * G;
  for (int t = threadIdx.x; t < G * HD; t += kDecWarps * 32) {
    const int hh = t / HD, e = t % HD;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) M = fmaxf(M, ms[w][hh]);
    float L = 0.f, O = 0.f;
#pragma unroll
    for (int w = 0; w < kDecWarps; ++w) {
      const float f = exp2f(ms[w][hh] - M);   // 0 for a warp without keys (max -inf)
      L = fmaf(ls[w][hh], f, L);
      O = fmaf(accs[w][hh][e], f, O);
    }
    a.part_o[(base + hh) * HD + e] = O;
    if (e == 0) {
      a.part_ml[(base + hh) * 2] = M;
      a.part_ml[(base + hh) * 2 + 1] = L;
    }
  }
}

template <int G>
__global__ void decode_combine_kernel(DecodeAttnArgs a, int r0) {
  const int HD = blockDim.x;
  const int h = blockIdx.x, sq = blockIdx.y, r = r0 + sq, e = threadIdx.x;
  const int g = h / G, hh = h % G;
  __nv_bfloat16* out = a.out + (long)r * a.out_row + (long)h * HD + e;
  const int p = a.pos[r];
  if (p < 0 || p >= a.rows[sq]) {
    *out = __float2bfloat16(0.f);
    return;
  }
  const int ns = p / split_keys(p) + 1;
  const long base = ((long)r * a.hkv + g) * kDecSplits;
  float M = -INFINITY;
  for (int s = 0; s < ns; ++s) M = fmaxf(M, a.part_ml[((base + s) * G + hh) * 2]);
  float L = 0.f, O = 0.f;
  for (int s = 0; s < ns; ++s) {
    const long i = (base + s) * G + hh;
    const float f = exp2f(a.part_ml[i * 2] - M);
    L = fmaf(a.part_ml[i * 2 + 1], f, L);
    O = fmaf(a.part_o[i * HD + e], f, O);
  }
  float o = O / L;
  if (a.gated) {
    const float z = __bfloat162float(a.qkv[(long)r * a.qkv_row + (long)h * 2 * HD + HD + e]);
    o *= 1.f / (1.f + __expf(-z));
  }
  *out = __float2bfloat16(o);
}

template <int PER, int G>
void launch_decode(const DecodeAttnArgs& a, int r0, int rows, cudaStream_t stream) {
  decode_attn_kernel<PER, G><<<dim3(kDecSplits, a.hkv, rows), kDecWarps * 32, 0, stream>>>(a, r0);
  count_launch();
  decode_combine_kernel<G><<<dim3(a.hq, rows), 32 * PER, 0, stream>>>(a, r0);
  count_launch();
}

template <int PER>
void launch_decode_g(const DecodeAttnArgs& a, int G, int r0, int rows, cudaStream_t stream) {
  switch (G) {
    case 1: launch_decode<PER, 1>(a, r0, rows, stream); break;
    case 2: launch_decode<PER, 2>(a, r0, rows, stream); break;
    case 4: launch_decode<PER, 4>(a, r0, rows, stream); break;
    case 6: launch_decode<PER, 6>(a, r0, rows, stream); break;
    default: launch_decode<PER, 8>(a, r0, rows, stream); break;
  }
}

}  // namespace

bool decode_attention_supported(int hd, int hq, int hkv, int rot) {
  if (hd != 64 && hd != 128 && hd != 256) return false;
  if (hkv <= 0 || hq % hkv != 0) return false;
  const int G = hq / hkv;
  if (G != 1 && G != 2 && G != 4 && G != 6 && G != 8) return false;
  const int per = hd / 32;
  return rot == 0 || (rot <= hd && rot % (2 * per) == 0);
}

void decode_attention(const DecodeAttnArgs& a, int r0, int rows, cudaStream_t stream) {
  if (rows <= 0) return;
  if (rows > kDecodeSeqs || !decode_attention_supported(a.hd, a.hq, a.hkv, a.rot))
    throw std::runtime_error("decode_attention: unsupported shape");
  const int G = a.hq / a.hkv;
  switch (a.hd) {
    case 64: launch_decode_g<2>(a, G, r0, rows, stream); break;
    case 128: launch_decode_g<4>(a, G, r0, rows, stream); break;
    default: launch_decode_g<8>(a, G, r0, rows, stream); break;
  }
}

}  // namespace rf
