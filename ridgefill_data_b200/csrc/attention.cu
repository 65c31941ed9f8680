// Flash prefill attention: causal GQA over a K/V cache, queries at contiguous or arbitrary sorted
// positions (query at position p sees keys j <= p), online softmax in fp32 (exp2 with the scale folded
// in), probabilities rounded to bf16 for the P.V product, optional sigmoid output gate.
//
// CTA = 4 warps x 16 query rows of one query head; key tiles of 64 rows double-buffered with cp.async;
// S = Q K^T and O += P V on mma.sync m16n8k16 bf16 tensor cores. The key range of a CTA stops at its last
// query's position, so causal work is skipped tile-wise; diagonal tiles are masked element-wise.
#include "kernels.h"
#include "mma.cuh"

// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero): one instruction, ex2(-inf) = 0.
__device__ __forceinline__ float ex2_sfu(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

#include <cfloat>
#include <stdexcept>

namespace rf {

constexpr int FA_BM = 64;
constexpr int FA_BN = 64;
constexpr int FA_THREADS = 128;

template <int HD>
struct FaSmem {
  static constexpr int PITCH = HD + 8;
  static constexpr int TILE = FA_BN * PITCH;  // elements
  static constexpr int BYTES = (FA_BM * PITCH + 4 * TILE) * 2;
};

template <int HD>
__device__ __forceinline__ void fa_load_tile(__nv_bfloat16* dst, const __nv_bfloat16* src, int rows_valid, int tid) {
  constexpr int PITCH = FaSmem<HD>::PITCH;
  constexpr int VEC_PER_ROW = HD / 8;
  for (int v = tid; v < FA_BN * VEC_PER_ROW; v += FA_THREADS) {
    const int r = v / VEC_PER_ROW;
    const int c = (v % VEC_PER_ROW) * 8;
    const bool ok = r < rows_valid;
    cp_async16(dst + r * PITCH + c, ok ? (src + (long)r * HD + c) : src, ok);
  }
}

template <int HD>
__global__ void __launch_bounds__(FA_THREADS) flash_attn_kernel(AttnArgs a) {
  constexpr int PITCH = FaSmem<HD>::PITCH;
  constexpr int TILE = FaSmem<HD>::TILE;
  constexpr int NT_O = HD / 8;     // output n-tiles per warp
  extern __shared__ __align__(16) uint8_t fa_smem[];
  __nv_bfloat16* sQ = reinterpret_cast<__nv_bfloat16*>(fa_smem);
  __nv_bfloat16* sK = sQ + FA_BM * PITCH;
  __nv_bfloat16* sV = sK + 2 * TILE;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int g = lane >> 2;
  const int t = lane & 3;
  const int qt = gridDim.x - 1 - blockIdx.x;  // heavy (late) query tiles first
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int row0 = qt * FA_BM;
  const int rows_valid = min(FA_BM, a.nq - row0);
  if (rows_valid <= 0) return;

  auto qpos_of = [&](int r) -> int {
    const int rr = min(r, a.nq - 1);
    return a.qpos != nullptr ? a.qpos[rr] : a.q_start + rr;
  };
  const int p_first = qpos_of(row0);
  const int p_last = qpos_of(row0 + rows_valid - 1);
  const int n_keys = min(a.nk, p_last + 1);
  const int n_tiles = (n_keys + FA_BN - 1) / FA_BN;

  const __nv_bfloat16* qbase = a.q + (long)head * a.q_head_stride + (long)row0 * HD;
  const __nv_bfloat16* kbase = a.k + (long)kvh * a.kv_head_stride;
  const __nv_bfloat16* vbase = a.v + (long)kvh * a.kv_head_stride;

  // Q tile
  for (int v = tid; v < FA_BM * (HD / 8); v += FA_THREADS) {
    const int r = v / (HD / 8);
    const int c = (v % (HD / 8)) * 8;
    const bool ok = r < rows_valid;
    cp_async16(sQ + r * PITCH + c, ok ? (qbase + (long)r * HD + c) : qbase, ok);
  }
  if (n_tiles > 0) {
    fa_load_tile<HD>(sK, kbase, min(FA_BN, n_keys), tid);
    fa_load_tile<HD>(sV, vbase, min(FA_BN, n_keys), tid);
  }
  cp_async_commit();

  const int r_lo = warp * 16 + g;       // this thread's two rows within the tile
  const int r_hi = r_lo + 8;
  const int pos_lo = qpos_of(row0 + r_lo);
  const int pos_hi = qpos_of(row0 + r_hi);
  const float sl2 = a.scale * 1.4426950408889634f;

  float o[NT_O][4];
#pragma unroll
  for (int j = 0; j < NT_O; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
  float m_lo = -FLT_MAX, m_hi = -FLT_MAX, l_lo = 0.f, l_hi = 0.f;

  for (int kt = 0; kt < n_tiles; ++kt) {
    const int buf = kt & 1;
    if (kt + 1 < n_tiles) {
      const int k0 = (kt + 1) * FA_BN;
      fa_load_tile<HD>(sK + (buf ^ 1) * TILE, kbase + (long)k0 * HD, min(FA_BN, n_keys - k0), tid);
      fa_load_tile<HD>(sV + (buf ^ 1) * TILE, vbase + (long)k0 * HD, min(FA_BN, n_keys - k0), tid);
    }
    cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();

    const __nv_bfloat16* cK = sK + buf * TILE;
    const __nv_bfloat16* cV = sV + buf * TILE;
    float s[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < HD / 16; ++ks) {
      uint32_t af[4];
      lda_row(af, sQ, PITCH, warp * 16, ks * 16, lane);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, cK, PITCH, j2 * 16, ks * 16, lane);
        mma_bf16(s[2 * j2], af, bf[0], bf[1]);
        mma_bf16(s[2 * j2 + 1], af, bf[2], bf[3]);
      }
    }
    // mask (causal + key range) where the tile can reach past a row's position
    const int key0 = kt * FA_BN;
    if (key0 + FA_BN - 1 > p_first || key0 + FA_BN > n_keys) {
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = key0 + j * 8 + 2 * t;
        if (c > pos_lo || c >= n_keys) s[j][0] = -INFINITY;
        if (c + 1 > pos_lo || c + 1 >= n_keys) s[j][1] = -INFINITY;
        if (c > pos_hi || c >= n_keys) s[j][2] = -INFINITY;
        if (c + 1 > pos_hi || c + 1 >= n_keys) s[j][3] = -INFINITY;
      }
    }
    float mx_lo = -INFINITY, mx_hi = -INFINITY;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      mx_lo = fmaxf(mx_lo, fmaxf(s[j][0], s[j][1]));
      mx_hi = fmaxf(mx_hi, fmaxf(s[j][2], s[j][3]));
    }
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 1));
    mx_lo = fmaxf(mx_lo, __shfl_xor_sync(0xffffffffu, mx_lo, 2));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 1));
    mx_hi = fmaxf(mx_hi, __shfl_xor_sync(0xffffffffu, mx_hi, 2));
    const float mn_lo = fmaxf(m_lo, mx_lo);
    const float mn_hi = fmaxf(m_hi, mx_hi);
    const float base_lo = (mn_lo == -INFINITY) ? 0.f : mn_lo * sl2;
    const float base_hi = (mn_hi == -INFINITY) ? 0.f : mn_hi * sl2;
    const float corr_lo = ex2_sfu(fmaf(m_lo, sl2, -base_lo));
    const float corr_hi = ex2_sfu(fmaf(m_hi, sl2, -base_hi));
    m_lo = mn_lo;
    m_hi = mn_hi;
    float rs_lo = 0.f, rs_hi = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      s[j][0] = ex2_sfu(fmaf(s[j][0], sl2, -base_lo));
      s[j][1] = ex2_sfu(fmaf(s[j][1], sl2, -base_lo));
      s[j][2] = ex2_sfu(fmaf(s[j][2], sl2, -base_hi));
      s[j][3] = ex2_sfu(fmaf(s[j][3], sl2, -base_hi));
      rs_lo += s[j][0] + s[j][1];
      rs_hi += s[j][2] + s[j][3];
    }
    l_lo = l_lo * corr_lo + rs_lo;
    l_hi = l_hi * corr_hi + rs_hi;
#pragma unroll
    for (int j = 0; j < NT_O; ++j) {
      o[j][0] *= corr_lo;
      o[j][1] *= corr_lo;
      o[j][2] *= corr_hi;
      o[j][3] *= corr_hi;
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
      uint32_t pf[4];
      pf[0] = pack2(s[2 * kk][0], s[2 * kk][1]);
      pf[1] = pack2(s[2 * kk][2], s[2 * kk][3]);
      pf[2] = pack2(s[2 * kk + 1][0], s[2 * kk + 1][1]);
      pf[3] = pack2(s[2 * kk + 1][2], s[2 * kk + 1][3]);
#pragma unroll
      for (int j2 = 0; j2 < NT_O / 2; ++j2) {
        uint32_t bf[4];
        ldb_kn(bf, cV, PITCH, j2 * 16, kk * 16, lane);
        mma_bf16(o[2 * j2], pf, bf[0], bf[1]);
        mma_bf16(o[2 * j2 + 1], pf, bf[2], bf[3]);
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();

  // row sums across the quad
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 1);
  l_lo += __shfl_xor_sync(0xffffffffu, l_lo, 2);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 1);
  l_hi += __shfl_xor_sync(0xffffffffu, l_hi, 2);
  const float inv_lo = l_lo > 0.f ? 1.f / l_lo : 0.f;
  const float inv_hi = l_hi > 0.f ? 1.f / l_hi : 0.f;
#pragma unroll
  for (int half = 0; half < 2; ++half) {
    const int r = half ? r_hi : r_lo;
    if (r >= rows_valid) continue;
    const float inv = half ? inv_hi : inv_lo;
    const long qrow = row0 + r;
    __nv_bfloat16* dst = a.out + qrow * a.out_row + (long)head * HD;
    const __nv_bfloat16* gt = a.gate != nullptr ? a.gate + qrow * a.gate_row + (long)head * a.gate_head : nullptr;
#pragma unroll
    for (int j = 0; j < NT_O; ++j) {
      const int c = j * 8 + 2 * t;
      float v0 = __bfloat162float(__float2bfloat16(o[j][half * 2] * inv));
      float v1 = __bfloat162float(__float2bfloat16(o[j][half * 2 + 1] * inv));
      if (gt != nullptr) {
        const float g0 = __bfloat162float(gt[c]), g1 = __bfloat162float(gt[c + 1]);
        v0 *= __bfloat162float(__float2bfloat16(1.f / (1.f + expf(-g0))));
        v1 *= __bfloat162float(__float2bfloat16(1.f / (1.f + expf(-g1))));
      }
      *reinterpret_cast<uint32_t*>(dst + c) = pack2(v0, v1);
    }
  }
}

template <int HD>
static void launch_fa(const AttnArgs& a, cudaStream_t stream) {
  constexpr int SMEM = FaSmem<HD>::BYTES;
  static PerDeviceOnce once;
  once([] { cudaFuncSetAttribute(flash_attn_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM); });
  dim3 grid((a.nq + FA_BM - 1) / FA_BM, a.hq);
  flash_attn_kernel<HD><<<grid, FA_THREADS, SMEM, stream>>>(a); count_launch();
}

void flash_attention(const AttnArgs& a, cudaStream_t stream) {
  if (a.nq <= 0) return;
  if (a.kv_pages != nullptr && a.impl == 1)
    throw std::runtime_error("flash_attention: paged K/V runs on the tcgen05 kernel only");
  if (a.impl != 1 && flash_attention_tc(a, stream)) return;
  if (a.kv_pages != nullptr) throw std::runtime_error("flash_attention: paged K/V not supported for this call");
  if (a.impl == 2) throw std::runtime_error("flash_attention: the tcgen05 path does not cover this call");
  switch (a.hd) {
    case 64: launch_fa<64>(a, stream); break;
    case 128: launch_fa<128>(a, stream); break;
    case 256: launch_fa<256>(a, stream); break;
    default: break;
  }
}

}  // namespace rf
