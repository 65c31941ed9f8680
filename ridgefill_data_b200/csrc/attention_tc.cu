// Flash prefill attention on the 5th-generation tensor cores (tcgen05 + TMEM), for queries at contiguous
// positions q_start .. q_start + nq - 1, or at the ascending positions qpos[0 .. nq) (the exact rows of a bypass
// arm), over keys 0 .. nk - 1 (query at position p sees keys j <= p).
//
// CTA = 128 query rows of one query head (GQA: K/V of head / (hq / hkv)); 96 + 128 * SWG threads:
//   warp 0      TMA: Q once, then K tiles of BN keys into a 2-stage ring (3-D tensor maps [heads][rows][hd], so
//               keys past nk read as zeros)
//   warp 2      TMA: V tiles into their own 2-stage ring (a K load never queues behind a V stage still in use)
//   warp 1      UMMA issuer: S_j = Q K_j^T into one of NS TMEM S buffers, issued NS - 1 tiles ahead of the
//               O += P_j V_j product into the TMEM O accumulator (P from shared memory, V as an MN-major B
//               operand). NS = 3 gives the tensor cores two S tiles of work while the softmax of a third runs
//               (head_dim 128, where it measured 1-2 % faster); head_dim 256 keeps NS = 2.
//   warps 3..   softmax, SWG warpgroups: thread = (query row, BN / SWG columns of every S tile); S part from TMEM,
//               causal mask (diagonal tiles only), one FMA + one ex2 (special-function unit) per score with the
//               scale folded in, partial row sum. With two warpgroups the two halves of a row swap their partial
//               row max once per tile through shared memory (two mbarriers: values written, values read; bounded
//               waits), so both halves use the same max; the partial row sums are added in the epilogue;
//               O is rescaled in TMEM only when the row max grows by more than 2^8 (otherwise the stale max stays
//               exact for both O and l); P rounded to bf16 into shared memory in the 128-byte-swizzled K-major
//               layout; finally O / l (times sigmoid(gate)) to global memory, each warpgroup its HD / SWG columns.
// The default is one softmax warpgroup (SWG = 1), two P buffers and exponentials on the special-function unit. The
// other template choices are measured A/B variants, none faster by more than 2 %: two softmax warpgroups (SWG = 2),
// one P buffer (PB = 1), part of the exponentials on the FMA pipe (POLY), Q read from TMEM by the S product as the
// A operand (QT = 1: the first warpgroup copies its Q rows from the swizzled tile into TMEM), and each CTA walking
// the key tiles from its own start (a.rotate).
// Every mbarrier wait is bounded (ptx.cuh); the kernel records an error code instead of hanging.
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace rf {

template <int HD, int BN, int PB, int SWG, int NS, int QT>
struct TcFaCfg {
  static constexpr int Q_BYTES = 128 * HD * 2;
  static constexpr int K_BYTES = BN * HD * 2;
  static constexpr int V_BYTES = BN * HD * 2;
  static constexpr int P_BYTES = 128 * BN * 2;
  static constexpr int BAR_BYTES = 8 * 26;
  static constexpr int RED_BYTES = SWG == 2 ? 2 * 128 * 4 : 0;   // partial row max of each warpgroup
  // PB P buffers (2: the softmax of block j + 1 writes its P while the tensor cores still read block j's)
  static constexpr int SMEM = 1024 + Q_BYTES + 2 * (K_BYTES + V_BYTES) + PB * P_BYTES + BAR_BYTES + RED_BYTES;
  static constexpr int O_COL = NS * BN;
  static constexpr int Q_COL = O_COL + HD;     // QT: Q rows as the A operand in TMEM (2 bf16 per column)
  static constexpr int THREADS = 96 + 128 * SWG;
  static_assert(O_COL + HD + (QT ? HD / 2 : 0) <= 512, "S buffers, O (and Q) in the 512 TMEM columns");
  static_assert(SMEM <= 232448, "shared memory of one CTA");
};

struct TcFaArgs {
  int hq, hkv, nq, nk, q_start;
  const int* qpos;   // ascending query positions, or nullptr: q_start + row
  const int* kv_pages;   // paged K/V: page of every page_size key rows (nullptr: contiguous [hkv][rows][hd])
  int page_size;
  int rotate;        // start every CTA's key loop at its own tile
  float scale_log2;
  const __nv_bfloat16* gate;
  long gate_row, gate_head;
  __nv_bfloat16* out;
  long out_row;
  int* err;
};

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 2^x on the special-function unit (PTX ex2.approx, flush-to-zero): one instruction per element, ex2(-inf) = 0.
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// 2^x for x <= 0 on the FMA and integer pipes instead of the special-function unit. Range reduction by the
// round-to-nearest of an fp32 add with 1.5 * 2^23: x = n + f, n integer, f in [-1/2, 1/2]; 2^f by a cubic whose
// coefficients come from a Lawson (iteratively reweighted least-squares) minimax fit of 2^f on [-1/2, 1/2] for
// relative error (7.5e-5 in exact arithmetic, 1.5e-4 evaluated in fp32: far below the bf16 rounding of P); 2^n
// by adding n to the exponent field. Inputs below -126 (masked scores included) give exactly 0.
__device__ __forceinline__ float exp2_fma(float x) {
  const float t = __fadd_rn(x, 12582912.f);
  const float f = __fsub_rn(x, __fsub_rn(t, 12582912.f));
  const float p = fmaf(fmaf(fmaf(0.05517144f, f, 0.24261071f), f, 0.69326097f), f, 0.99992812f);
  const int n = __float_as_int(t) - 0x4B400000;
  return x < -126.f ? 0.f : __int_as_float(__float_as_int(p) + (n << 23));
}

template <int HD, int BN, int PB, int POLY, int SWG, int NS, int QT>
__global__ void __launch_bounds__(96 + 128 * SWG, 1)
    tc_flash_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                    const __grid_constant__ CUtensorMap tmV, TcFaArgs a) {
  using Cfg = TcFaCfg<HD, BN, PB, SWG, NS, QT>;
  static_assert(NS == 2 || NS == 3, "two or three S buffers");
  static_assert(SWG == 1 || SWG == 2, "one or two softmax warpgroups");
  static_assert(BN % (32 * SWG) == 0, "every warpgroup's part of an S tile is whole 32-column TMEM loads");
  static_assert(POLY >= 0 && POLY <= 8, "POLY: columns of every 8 whose exponential runs on the FMA pipe");
  constexpr uint32_t IDESC_S = idesc_bf16_f32(128, BN, false, false);
  constexpr uint32_t IDESC_O = idesc_bf16_f32(128, HD, false, true);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint8_t* sQ = smem;
  uint8_t* sK = sQ + Cfg::Q_BYTES;
  uint8_t* sV = sK + 2 * Cfg::K_BYTES;
  uint8_t* sP = sV + 2 * Cfg::V_BYTES;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sP + PB * Cfg::P_BYTES);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2]
  uint64_t* v_full = bars + 3;    // [2]
  uint64_t* k_empty = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [NS]
  uint64_t* s_free = bars + 12;   // [NS]
  uint64_t* p_full = bars + 15;    // [2]
  uint64_t* p_free = bars + 17;    // [2]
  uint64_t* o_final = bars + 19;
  uint64_t* x_full = bars + 20;    // both warpgroups wrote their partial row max
  uint64_t* x_read = bars + 21;    // both warpgroups read the other's
  uint64_t* q_tmem = bars + 22;    // QT: the Q rows are in TMEM
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);
  float* red = reinterpret_cast<float*>(bars + 25);   // [SWG][128]

  const int warp = warp_id(), lane = lane_id();
  const int qt = gridDim.x - 1 - blockIdx.x;   // late (heavy) query tiles first
  const int head = blockIdx.y;
  const int kvh = head / (a.hq / a.hkv);
  const int q0 = qt * 128;
  const int rows_valid = min(128, a.nq - q0);
  // keys this tile reads: up to the last (largest) query position of the tile
  const int last_pos = a.qpos != nullptr ? a.qpos[q0 + rows_valid - 1] : a.q_start + q0 + rows_valid - 1;
  const int n_keys = max(0, min(a.nk, last_pos + 1));
  const int ntiles = (n_keys + BN - 1) / BN;
  // processing order of the key tiles: with a.rotate, each CTA starts at its own tile (the online softmax does not
  // depend on the order), so the CTAs of one K/V head do not all request the same tile from the same L2 slices
  const int rot = (a.rotate && ntiles > 0) ? (int)((blockIdx.x * 5u + blockIdx.y * 3u) % (unsigned)ntiles) : 0;
  auto kt = [&](int j) { const int t = j + rot; return t >= ntiles ? t - ntiles : t; };

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_empty[s], 1);
    }
    for (int s = 0; s < NS; ++s) {
      mbar_init(&s_full[s], 1);
      mbar_init(&s_free[s], 128 * SWG);
    }
    for (int s = 0; s < 2; ++s) {
      mbar_init(&p_full[s], 128 * SWG);
      mbar_init(&p_free[s], 1);
    }
    mbar_init(o_final, 1);
    mbar_init(x_full, 128 * SWG);
    mbar_init(x_read, 128 * SWG);
    mbar_init(q_tmem, 128);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 0) {
    if (lane == 0) {
      mbar_expect_tx(q_full, Cfg::Q_BYTES);
#pragma unroll
      for (int b = 0; b < HD / 64; ++b) tma_load_3d(sQ + b * 128 * 128, &tmQ, q_full, b * 64, q0, head);
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1u;
        if (*abort_flag || !mbar_wait(&k_empty[st], par, a.err, kErrTimeoutProducer)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&k_full[st], Cfg::K_BYTES);
        // paged K/V: the key tile lies inside one page (page_size is a multiple of BN)
        const int kr = kt(j) * BN;
        const int page = a.kv_pages != nullptr ? a.kv_pages[kr / a.page_size] : 0;
        const int prow = a.kv_pages != nullptr ? kr % a.page_size : kr;
#pragma unroll
        for (int b = 0; b < HD / 64; ++b) {
          if (a.kv_pages != nullptr)
            tma_load_4d(sK + st * Cfg::K_BYTES + b * BN * 128, &tmK, &k_full[st], b * 64, prow, kvh, page);
          else
            tma_load_3d(sK + st * Cfg::K_BYTES + b * BN * 128, &tmK, &k_full[st], b * 64, kr, kvh);
        }
      }
    }
  } else if (warp == 2) {
    if (lane == 0) {
      for (int j = 0; j < ntiles; ++j) {
        const int st = j & 1;
        const uint32_t par = ((j >> 1) & 1) ^ 1u;
        if (*abort_flag || !mbar_wait(&v_empty[st], par, a.err, kErrTimeoutProducer)) {
          *abort_flag = 1;
          break;
        }
        mbar_expect_tx(&v_full[st], Cfg::V_BYTES);
        const int kr = kt(j) * BN;
        const int page = a.kv_pages != nullptr ? a.kv_pages[kr / a.page_size] : 0;
        const int prow = a.kv_pages != nullptr ? kr % a.page_size : kr;
#pragma unroll
        for (int b = 0; b < HD / 64; ++b) {
          if (a.kv_pages != nullptr)
            tma_load_4d(sV + st * Cfg::V_BYTES + b * BN * 128, &tmV, &v_full[st], b * 64, prow, kvh, page);
          else
            tma_load_3d(sV + st * Cfg::V_BYTES + b * BN * 128, &tmV, &v_full[st], b * 64, kr, kvh);
        }
      }
    }
  } else if (warp == 1) {
    bool ok = mbar_wait(q_full, 0, a.err, kErrTimeoutMma);
    if constexpr (QT) ok = ok && mbar_wait(q_tmem, 0, a.err, kErrTimeoutMma);
    tc_fence_after();
    const uint32_t q_addr = smem_u32(sQ), p_addr = smem_u32(sP);
    auto issue_pv = [&](int jj) -> bool {
      const int st = jj & 1;       // K/V stage of block jj
      const int pq = jj % PB;      // its P buffer
      if (!mbar_wait(&p_full[pq], (jj / PB) & 1, a.err, kErrTimeoutMma)) return false;
      if (!mbar_wait(&v_full[st], (jj >> 1) & 1, a.err, kErrTimeoutMma)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t v_addr = smem_u32(sV + st * Cfg::V_BYTES);
#pragma unroll
        for (int kk = 0; kk < BN / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(p_addr + pq * Cfg::P_BYTES + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(v_addr + kk * 2048, BN * 128, 1024);
          umma_f16(tmem + Cfg::O_COL, ad, bd, IDESC_O, (jj > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&p_free[pq]);
        umma_commit(&v_empty[st]);
      }
      __syncwarp();
      return true;
    };
    // S_jj = Q K_jj^T into S buffer jj % NS (free once the softmax of tile jj - NS has read it)
    auto issue_s = [&](int jj) -> bool {
      const int st = jj & 1;
      const int sb = jj % NS;
      if (*abort_flag || !mbar_wait(&k_full[st], (jj >> 1) & 1, a.err, kErrTimeoutMma)) return false;
      if (jj >= NS && !mbar_wait(&s_free[sb], ((jj - NS) / NS) & 1, a.err, kErrTimeoutMma)) return false;
      tc_fence_after();
      if (lane == 0) {
        const uint32_t k_addr = smem_u32(sK + st * Cfg::K_BYTES);
#pragma unroll
        for (int kk = 0; kk < HD / 16; ++kk) {
          const uint64_t bd = sdesc_sw128(k_addr + (kk >> 2) * BN * 128 + (kk & 3) * 32, 16, 1024);
          if constexpr (QT) {   // A from TMEM: K step kk is columns 8 kk .. 8 kk + 7 of the Q rows
            umma_f16_ts(tmem + sb * BN, tmem + Cfg::Q_COL + 8 * kk, bd, IDESC_S, kk > 0 ? 1u : 0u);
          } else {
            const uint64_t ad = sdesc_sw128(q_addr + (kk >> 2) * 128 * 128 + (kk & 3) * 32, 16, 1024);
            umma_f16(tmem + sb * BN, ad, bd, IDESC_S, kk > 0 ? 1u : 0u);
          }
        }
        umma_commit(&s_full[sb]);
        umma_commit(&k_empty[st]);
      }
      __syncwarp();
      return true;
    };
    for (int jj = 0; jj < NS - 1 && jj < ntiles && ok; ++jj) ok = issue_s(jj);
    for (int jj = 0; jj < ntiles && ok; ++jj) {
      if (jj + NS - 1 < ntiles && !issue_s(jj + NS - 1)) {
        ok = false;
        break;
      }
      if (!issue_pv(jj)) {
        ok = false;
        break;
      }
    }
    if (lane == 0) umma_commit(o_final);   // also drains whatever was issued on the abort path
    __syncwarp();
    if (!ok) *abort_flag = 1;
  } else {
    // ---------------------------------------------------------------- softmax + epilogue
    constexpr int CW = BN / SWG;            // columns of every S tile this warpgroup handles
    constexpr int OW = HD / SWG;            // columns of O it rescales and stores
    const int wg = (warp - 3) >> 2;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;
    const int cb = wg * CW;
    // rows past nq see no key (their outputs are not stored)
    const int pos = a.qpos == nullptr ? a.q_start + q0 + r : (r < rows_valid ? a.qpos[q0 + r] : -1);
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    int xph = 0;
    if constexpr (QT) {
      // the first warpgroup copies its Q row from the swizzled shared tile into TMEM (the S product's A operand)
      if (wg == 0) {
        ok = mbar_wait(q_full, 0, a.err, kErrTimeoutEpilogue);
        if (ok) {
#pragma unroll 1
          for (int b = 0; b < HD / 64; ++b) {
            uint32_t w16a[16], w16b[16];
#pragma unroll
            for (int ch = 0; ch < 8; ++ch) {
              const uint4 v = *reinterpret_cast<const uint4*>(sQ + b * 128 * 128 + r * 128 + ((ch ^ (r & 7)) << 4));
              uint32_t* dst = ch < 4 ? w16a + 4 * ch : w16b + 4 * (ch - 4);
              dst[0] = v.x;
              dst[1] = v.y;
              dst[2] = v.z;
              dst[3] = v.w;
            }
            tmem_st16(tmem + lane_off + Cfg::Q_COL + b * 32, w16a);
            tmem_st16(tmem + lane_off + Cfg::Q_COL + b * 32 + 16, w16b);
          }
          tmem_wait_st();
        }
        tc_fence_before();
        mbar_arrive(q_tmem);
      }
    }
    // one value per row to the other warpgroup and back (SWG == 2); NaN marks a warpgroup that stopped, so both
    // stop at the same tile. The write of phase p waits until the other side has read phase p - 1.
    auto exchange = [&](float v, float& other) -> bool {
      if (xph > 0 && !mbar_wait(x_read, (xph - 1) & 1, a.err, kErrTimeoutEpilogue)) return false;
      red[wg * 128 + r] = v;
      mbar_arrive(x_full);
      if (!mbar_wait(x_full, xph & 1, a.err, kErrTimeoutEpilogue)) return false;
      other = red[(wg ^ 1) * 128 + r];
      mbar_arrive(x_read);
      ++xph;
      return true;
    };
    for (int j = 0; j < ntiles; ++j) {
      const int st = j % NS;
      const bool got = !*abort_flag && mbar_wait(&s_full[st], (j / NS) & 1, a.err, kErrTimeoutEpilogue);
      // raw scores; the scale (log2 e / sqrt(d)) is applied inside the exponent's FMA
      float x[CW];
      float mt = -INFINITY;
      if (got) {
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < CW; c += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + st * BN + cb + c, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) x[c + e] = __uint_as_float(v[e]);
        }
        tc_fence_before();
        mbar_arrive(&s_free[st]);
        const int key0 = kt(j) * BN + cb;
        // only tiles that reach past this row's position (the diagonal) or past n_keys need the mask
        if (key0 + CW - 1 > pos || key0 + CW > n_keys) {
#pragma unroll
          for (int e = 0; e < CW; ++e) {
            const int key = key0 + e;
            if (key > pos || key >= n_keys) x[e] = -INFINITY;
          }
        }
        // row max as 8 independent chains
        float mp[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) mp[u] = x[u];
#pragma unroll
        for (int e = 8; e < CW; ++e) mp[e & 7] = fmaxf(mp[e & 7], x[e]);
        mt = fmaxf(fmaxf(fmaxf(mp[0], mp[1]), fmaxf(mp[2], mp[3])), fmaxf(fmaxf(mp[4], mp[5]), fmaxf(mp[6], mp[7])));
        if (mt != mt) mt = -INFINITY;   // NaN scores: keep NaN free for the stop mark
      }
      if constexpr (SWG == 2) {
        float mo = 0.f;
        if (!exchange(got ? mt : NAN, mo) || !got || mo != mo) {
          ok = false;
          break;
        }
        mt = fmaxf(mt, mo);
      } else if (!got) {
        ok = false;
        break;
      }
      const float m_new = fmaxf(m_used, mt * a.scale_log2);   // scale > 0: max commutes with it
      bool rescale = false;
      float factor = 1.f;
      if (m_used == -INFINITY) {
        m_used = m_new;
      } else if (m_new > m_used + 8.f) {
        rescale = true;
        factor = ex2(m_used - m_new);
        m_used = m_new;
      }
      const float base = m_used == -INFINITY ? 0.f : m_used;
      float sp[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll
      for (int e = 0; e < CW; ++e) {
        const float z = fmaf(x[e], a.scale_log2, -base);
        x[e] = (e & 7) < POLY ? exp2_fma(z) : ex2(z);   // POLY of every 8 columns off the SFU
        sp[e & 7] += x[e];
      }
      const float sum = ((sp[0] + sp[1]) + (sp[2] + sp[3])) + ((sp[4] + sp[5]) + (sp[6] + sp[7]));
      l = l * factor + sum;
      const int pb = j % PB;
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
        // O is rescaled in TMEM: every P V product so far (the last one is block j - 1's) must have landed
        if (!mbar_wait(&p_free[(j - 1) % PB], ((j - 1) / PB) & 1, a.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        {
#pragma unroll 1
          for (int c = wg * OW; c < (wg + 1) * OW; c += 32) {
            uint32_t v[32];
            tmem_ld32(tmem + lane_off + Cfg::O_COL + c, v);
            tmem_wait_ld();
            uint32_t w16a[16], w16b[16];
#pragma unroll
            for (int e = 0; e < 16; ++e) {
              w16a[e] = __float_as_uint(__uint_as_float(v[e]) * factor);
              w16b[e] = __float_as_uint(__uint_as_float(v[16 + e]) * factor);
            }
            tmem_st16(tmem + lane_off + Cfg::O_COL + c, w16a);
            tmem_st16(tmem + lane_off + Cfg::O_COL + c + 16, w16b);
          }
          tmem_wait_st();
        }
      }
      // P buffer pb was last read by block j - PB's P V product
      if (j >= PB && !mbar_wait(&p_free[pb], ((j - PB) / PB) & 1, a.err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      // P part -> shared memory, 128-byte swizzle, K-major (keys along K), 64-key column blocks
#pragma unroll
      for (int e = 0; e < CW; e += 8) {
        uint4 pk;
        pk.x = pack_bf16x2(x[e], x[e + 1]);
        pk.y = pack_bf16x2(x[e + 2], x[e + 3]);
        pk.z = pack_bf16x2(x[e + 4], x[e + 5]);
        pk.w = pack_bf16x2(x[e + 6], x[e + 7]);
        const int c = cb + e;
        const int blk = c >> 6, chunk = (c & 63) >> 3;
        uint8_t* dst = sP + pb * Cfg::P_BYTES + blk * 128 * 128 + r * 128 + ((chunk ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = pk;
      }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&p_full[pb]);
    }
    // the row sum: this warpgroup's part plus the other's
    float lt = l;
    if constexpr (SWG == 2) {
      float lo = 0.f;
      if (ok && (!exchange(l, lo) || lo != lo)) ok = false;
      lt = l + lo;
    }
    // epilogue
    if (ok && mbar_wait(o_final, 0, a.err, kErrTimeoutEpilogue)) {
      tc_fence_after();
      const float inv = lt > 0.f ? 1.f / lt : 0.f;
      const long qrow = q0 + r;
      const bool row_ok = r < rows_valid;
      __nv_bfloat16* dst = a.out + qrow * a.out_row + (long)head * HD;
      const __nv_bfloat16* gt = a.gate != nullptr ? a.gate + qrow * a.gate_row + (long)head * a.gate_head : nullptr;
#pragma unroll 1
      for (int c = wg * OW; c < (wg + 1) * OW; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + Cfg::O_COL + c, v);
        tmem_wait_ld();
        if (!row_ok) continue;
#pragma unroll
        for (int e = 0; e < 32; e += 8) {
          float o[8];
#pragma unroll
          for (int q = 0; q < 8; ++q) o[q] = __bfloat162float(__float2bfloat16(__uint_as_float(v[e + q]) * inv));
          if (gt != nullptr) {
            uint4 gv = *reinterpret_cast<const uint4*>(gt + c + e);
            const __nv_bfloat16* ge = reinterpret_cast<const __nv_bfloat16*>(&gv);
#pragma unroll
            for (int q = 0; q < 8; ++q) {
              const float z = __bfloat162float(ge[q]);
              o[q] *= __bfloat162float(__float2bfloat16(1.f / (1.f + expf(-z))));
            }
          }
          uint4 w;
          w.x = pack_bf16x2(o[0], o[1]);
          w.y = pack_bf16x2(o[2], o[3]);
          w.z = pack_bf16x2(o[4], o[5]);
          w.w = pack_bf16x2(o[6], o[7]);
          *reinterpret_cast<uint4*>(dst + c + e) = w;
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

static PFN_cuTensorMapEncodeTiled_v12000 encode_fa() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  if (fn == nullptr) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess || p == nullptr)
      throw std::runtime_error("cuTensorMapEncodeTiled entry point unavailable");
    fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }
  return fn;
}

// 3-D map over [heads][rows][hd] (row pitch hd, head pitch head_stride elements), box {64, box_rows, 1}
static CUtensorMap tmap3(const void* base, int hd, int rows, int heads, long head_stride, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[3] = {(cuuint64_t)hd, (cuuint64_t)rows, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)hd * 2, (cuuint64_t)head_stride * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_fa()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("tc_flash: tensor map encode failed " + std::to_string((int)r));
  return tm;
}

// 4-D map over a page pool [pages][heads][page_size][hd], box {64, box_rows, 1, 1}
static CUtensorMap tmap4_pages(const void* base, int hd, int page_size, int heads, int pages, int box_rows) {
  CUtensorMap tm;
  cuuint64_t dims[4] = {(cuuint64_t)hd, (cuuint64_t)page_size, (cuuint64_t)heads, (cuuint64_t)pages};
  cuuint64_t strides[3] = {(cuuint64_t)hd * 2, (cuuint64_t)page_size * hd * 2, (cuuint64_t)heads * page_size * hd * 2};
  cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = encode_fa()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("tc_flash: paged tensor map encode failed " + std::to_string((int)r));
  return tm;
}

template <int HD, int BN, int PB, int POLY, int SWG, int NS, int QT = 0>
static void launch_tc(const AttnArgs& x, cudaStream_t stream) {
  using Cfg = TcFaCfg<HD, BN, PB, SWG, NS, QT>;
  static PerDeviceOnce once;
  once([] {
    cudaFuncSetAttribute(tc_flash_kernel<HD, BN, PB, POLY, SWG, NS, QT>,
                         cudaFuncAttributeMaxDynamicSharedMemorySize, Cfg::SMEM);
  });
  CUtensorMap tq = tmap3(x.q, HD, x.nq, x.hq, x.q_head_stride, 128);
  CUtensorMap tk, tv;
  if (x.kv_pages != nullptr) {
    tk = tmap4_pages(x.k, HD, x.page_size, x.hkv, x.num_pages, BN);
    tv = tmap4_pages(x.v, HD, x.page_size, x.hkv, x.num_pages, BN);
  } else {
    tk = tmap3(x.k, HD, x.nk, x.hkv, x.kv_head_stride, BN);
    tv = tmap3(x.v, HD, x.nk, x.hkv, x.kv_head_stride, BN);
  }
  TcFaArgs a{x.hq, x.hkv, x.nq, x.nk, x.q_start, x.qpos, x.kv_pages, x.page_size, attn_rotate,
             x.scale * 1.4426950408889634f,
             x.gate, x.gate_row, x.gate_head, x.out, x.out_row, x.err};
  dim3 grid((x.nq + 127) / 128, x.hq);
  tc_flash_kernel<HD, BN, PB, POLY, SWG, NS, QT><<<grid, Cfg::THREADS, Cfg::SMEM, stream>>>(tq, tk, tv, a);
  count_launch();
}

int attn_p_buffers = 2;
int attn_poly = 0;
int attn_softmax_groups = 1;
int attn_s_buffers = 0;
int attn_rotate = 0;
int attn_q_tmem = 0;

// NS0: the S-buffer count measured faster for this head dim (head_dim 256: 2, 128: 3); attn_s_buffers overrides it
template <int HD, int BN, int NS0>
static void launch_variant(const AttnArgs& x, cudaStream_t stream) {
  constexpr int NS1 = NS0 == 2 ? 3 : 2;
  const bool other = attn_s_buffers != 0 && attn_s_buffers != NS0;
  if (attn_q_tmem) launch_tc<HD, BN, 2, 0, 1, 2, 1>(x, stream);   // Q in TMEM leaves room for two S buffers
  else if (other) launch_tc<HD, BN, 2, 0, 1, NS1>(x, stream);
  else if (attn_softmax_groups == 2) launch_tc<HD, BN, 2, 0, 2, NS0>(x, stream);
  else if (attn_p_buffers == 1) launch_tc<HD, BN, 1, 0, 1, NS0>(x, stream);
  else if (attn_poly == 2) launch_tc<HD, BN, 2, 2, 1, NS0>(x, stream);
  else if (attn_poly == 4) launch_tc<HD, BN, 2, 4, 1, NS0>(x, stream);
  else launch_tc<HD, BN, 2, 0, 1, NS0>(x, stream);
}

bool flash_attention_tc(const AttnArgs& x, cudaStream_t stream) {
  if (x.nq <= 0) return false;
  if (x.kv_pages != nullptr) {
    const int bn = x.hd == 256 ? 64 : 128;
    if ((x.hd != 128 && x.hd != 256) || x.page_size <= 0 || x.page_size % bn != 0 || x.num_pages <= 0)
      throw std::runtime_error("flash_attention: paged K/V needs head_dim 128 / 256 and a page size multiple of 128");
  }
  if (reinterpret_cast<uintptr_t>(x.q) % 16 || reinterpret_cast<uintptr_t>(x.k) % 16 ||
      reinterpret_cast<uintptr_t>(x.v) % 16)
    return false;
  if (x.gate != nullptr && (x.gate_row % 8 || x.gate_head % 8 || reinterpret_cast<uintptr_t>(x.gate) % 16))
    return false;
  if (x.out_row % 8) return false;
  switch (x.hd) {
    case 128: launch_variant<128, 128, 3>(x, stream); return true;
    case 256: launch_variant<256, 64, 2>(x, stream); return true;
    default: return false;
  }
}

}  // namespace rf
