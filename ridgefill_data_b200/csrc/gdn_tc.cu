// Gated DeltaNet state + output pass on the 5th-generation tensor cores (tcgen05 + TMEM).
//
// The sequential part of the chunked gated delta rule (chunk C = 64, dk = dv = 128), one CTA per value head (or per
// (value head, chunk group) for the two-level scan's output pass). The transposed state S^T [dv][dk] (fp32) lives
// in TMEM for the whole sequence: lane m = value dim m, column k = key dim k. Per chunk:
//   rows    S^T -> bf16 copy in shared memory (A operand), S^T *= e^(gl) in TMEM            (gl = the chunk's decay)
//   MMA     D1 = S^T W^T, D2 = S^T (q e^gam)^T, D3 = q k^T                             (W, q, k: TMA tiles)
//   rows    P = D3 * e^(gam_r - gam_c) (c <= r) -> bf16 shared (B operand of the output product)
//           V'^T = U^T - D1 -> bf16 shared twice: as is (output) and times e^(gl - gam_c) (state update)
//   MMA     S^T += (V'^T diag(e^(gl - gam))) k         (k as an MN-major B operand)
//           D2 += V'^T P^T                               (the chunk's output O^T, double-buffered in TMEM)
//   rows    O^T -> bf16 output rows (read one chunk later, off the recurrence's chain)
// The chain per chunk is two TMEM round trips and two tensor-core products; the output products run beside it.
//
// Opt-in (gdn_state_tc = 1); the default output pass is the mma.sync one in gdn.cu (see gdn_state_tc below).
//
// Roles (192 threads): warps 0-3 the 128 state rows; warp 4 allocates TMEM and one lane issues every tcgen05.mma;
// warp 5 loads each chunk's q, W, k, U^T tiles by TMA into a two-stage ring, computes the chunk's cumulative decays
// and writes q e^gam (bf16) for the D2 product. Every mbarrier wait is bounded; a wait that runs out records an
// error code and the CTA leaves its loop (the MMA lane drains what it issued before TMEM is freed).
//
// Same chunk arithmetic as the mma.sync passes in gdn.cu (reference: code/kva/ops.py:199-262); the products use
// bf16 operands with fp32 accumulation, the state stays fp32 in TMEM.
#include "kernels.h"
#include "ptx.cuh"

#include <cudaTypedefs.h>
#include <stdexcept>
#include <string>

namespace rf {

namespace {

constexpr int TC_C = 64;       // chunk rows
constexpr int TC_D = 128;      // dk = dv

struct GdnTcArgs {
  int n, nk, nv, n_chunks, groups;
  const float* g;              // [nv, n]
  float* state;                // [nv, dk, dv] (mode 0)
  const float* start_buf;      // [nv, groups, dv, dk] (mode 2)
  __nv_bfloat16* out;
  long out_row;
  int* err;
  unsigned long long* trace;
};

// shared memory (offsets from a 1024-byte aligned base)
constexpr int ST_QW = 0;                       // [2 blocks][128 rows][128 B]: rows 0-63 q, 64-127 W (dk blocks of 64)
constexpr int ST_K = ST_QW + 2 * 16384;        // [2 blocks][64 rows][128 B]
constexpr int ST_U = ST_K + 2 * 8192;          // [128 rows][128 B] U^T (value dims x chunk rows), 128-byte swizzle
constexpr int ST_GAM = ST_U + 16384;           // float gam[64]
constexpr int ST_BYTES = ST_GAM + 1024;
constexpr int SM_S = 2 * ST_BYTES;             // bf16 S^T [2 blocks][128 rows][128 B]
constexpr int SM_VA = SM_S + 32768;            // bf16 V'^T e^(gl - gam) [128 rows][128 B]
constexpr int SM_VU = SM_VA + 16384;           // bf16 V'^T [128 rows][128 B]
constexpr int SM_P = SM_VU + 16384;            // bf16 P [64 rows][128 B]
constexpr int SM_QS = SM_P + 8192;             // bf16 q e^gam [2 blocks][64 rows][128 B]
constexpr int SM_BAR = SM_QS + 16384;
constexpr int N_BARS = 20;
constexpr int SM_TOTAL = SM_BAR + N_BARS * 8 + 16;
constexpr int SMEM_BYTES = 1024 + SM_TOTAL;
static_assert(SMEM_BYTES <= 232448, "shared memory of one CTA");

// TMEM columns
constexpr uint32_t T_S = 0;        // S^T fp32, 128 columns
constexpr uint32_t T_D1 = 128;     // S^T W^T, 64
constexpr uint32_t T_D2 = 192;     // output, 2 x 64
constexpr uint32_t T_D3 = 320;     // q k^T, 64 (lanes 0-63 meaningful)

__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// 16-byte chunk j (0..7) of row r of a 128-byte-swizzled tile
__device__ __forceinline__ uint32_t sw128(int r, int j) { return (uint32_t)(r * 128 + ((j ^ (r & 7)) << 4)); }

template <int MODE>
__global__ void __launch_bounds__(192, 1)
    gdn_state_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                        const __grid_constant__ CUtensorMap tmW, const __grid_constant__ CUtensorMap tmU, GdnTcArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + SM_BAR);
  uint64_t* full = bars + 0;       // [2] TMA bytes of a stage
  uint64_t* ready = bars + 2;      // [2] stage's decays and q e^gam written
  uint64_t* empty = bars + 4;      // [2] stage free: 128 row arrivals + the MMA lane's commit
  uint64_t* ss_full = bars + 6;    // bf16 S^T written
  uint64_t* d1_full = bars + 7;    // D1, D2 (term 1) done
  uint64_t* d3_full = bars + 8;    // D3 done
  uint64_t* v_full = bars + 9;     // V' operands written
  uint64_t* s_done = bars + 10;    // state update done
  uint64_t* p_full = bars + 11;    // P written (64 arrivals)
  // [2] output of chunk i complete in TMEM (by chunk parity: chunk i + 1's can complete before chunk i's is read)
  uint64_t* o_full = bars + 12;
  uint64_t* d2_free = bars + 14;   // [2] output buffer read
  uint64_t* drain = bars + 16;     // everything the MMA lane issued has completed
  uint32_t* tmem_holder = reinterpret_cast<uint32_t*>(bars + N_BARS);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_holder + 1);

  const int h = blockIdx.x;
  const int kh = h / (a.nv / a.nk);
  const int warp = warp_id(), lane = lane_id();
  const int per_group = MODE == 0 ? a.n_chunks : (a.n_chunks + a.groups - 1) / a.groups;
  const int c_begin = MODE == 0 ? 0 : (int)blockIdx.z * per_group;
  const int c_end = MODE == 0 ? a.n_chunks : min(a.n_chunks, c_begin + per_group);
  const int nch = max(0, c_end - c_begin);
  // optional phase trace of the first CTA (a.trace [chunks][16] ns stamps; nullptr: off)
  auto tr = [&](int slot, int i) {
    if (a.trace != nullptr && blockIdx.x == 0 && blockIdx.z == 0 && i < 128 && (threadIdx.x & 31) == 0 &&
        (warp >= 4 || threadIdx.x == 0))
      a.trace[i * 16 + slot] = global_timer_ns();
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < 2; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&ready[s], 1);
      mbar_init(&empty[s], 129);
      mbar_init(&d2_free[s], 128);
      mbar_init(&o_full[s], 1);
    }
    mbar_init(ss_full, 128);
    mbar_init(d1_full, 1);
    mbar_init(d3_full, 1);
    mbar_init(v_full, 128);
    mbar_init(s_done, 1);
    mbar_init(p_full, 64);
    mbar_init(drain, 1);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 4) {
    tmem_alloc(tmem_holder, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_holder;

  if (warp == 5) {
    // ------------------------------------------------------------------ producer
    auto issue = [&](int i) -> bool {
      const int s = i & 1;
      if (*abort_flag || !mbar_wait(&empty[s], ((i >> 1) & 1) ^ 1u, a.err, kErrTimeoutProducer)) return false;
      if (lane == 0) {
        const int c = c_begin + i;
        uint8_t* st = smem + s * ST_BYTES;
        mbar_expect_tx(&full[s], 2 * 8192 + 2 * 8192 + 2 * 8192 + 16384);
        for (int b = 0; b < 2; ++b) {
          tma_load_3d(st + ST_QW + b * 16384, &tmQ, &full[s], b * 64, c * TC_C, kh);
          tma_load_3d(st + ST_QW + b * 16384 + 8192, &tmW, &full[s], b * 64, c * TC_C, h);
          tma_load_3d(st + ST_K + b * 8192, &tmK, &full[s], b * 64, c * TC_C, kh);
        }
        tma_load_2d(st + ST_U, &tmU, &full[s], 0, (h * a.n_chunks + c) * TC_D);
      }
      __syncwarp();
      return true;
    };
    bool ok = nch == 0 || issue(0);
    // log decays of a chunk's rows 2 lane, 2 lane + 1 (rows past n decay by nothing), fetched one chunk ahead
    auto load_g = [&](int c, float& x0, float& x1) {
      const int r = c * TC_C + 2 * lane;
      x0 = r < a.n ? a.g[(long)h * a.n + r] : 0.f;
      x1 = r + 1 < a.n ? a.g[(long)h * a.n + r + 1] : 0.f;
    };
    float gx0 = 0.f, gx1 = 0.f;
    if (nch > 0) load_g(c_begin, gx0, gx1);
    for (int i = 0; i < nch && ok; ++i) {
      const int s = i & 1;
      uint8_t* st = smem + s * ST_BYTES;
      float* gam = reinterpret_cast<float*>(st + ST_GAM);
      const float x0 = gx0, x1 = gx1;
      if (i + 1 < nch) load_g(c_begin + i + 1, gx0, gx1);
      // cumulative log decay of the chunk
      const float pair = x0 + x1;
      float incl = pair;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const float y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      gam[2 * lane] = incl - x1;
      gam[2 * lane + 1] = incl;
      if (!mbar_wait(&full[s], (i >> 1) & 1, a.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      tr(10, i);
      // q e^gam (bf16) for D2: the previous chunk's D2 product must have read the buffer
      if (i >= 1 && !mbar_wait(d1_full, (i - 1) & 1, a.err, kErrTimeoutProducer)) {
        ok = false;
        break;
      }
      __syncwarp();
      for (int v = lane; v < 2 * TC_C * 8; v += 32) {
        const int b = v / (TC_C * 8), r = (v / 8) % TC_C, j = v % 8;
        const float e = __expf(gam[r]);
        const uint32_t off = b * 16384 + sw128(r, j);
        const uint4 x = *reinterpret_cast<const uint4*>(st + ST_QW + off);
        const __nv_bfloat162* xv = reinterpret_cast<const __nv_bfloat162*>(&x);
        uint4 y;
        uint32_t* yv = reinterpret_cast<uint32_t*>(&y);
#pragma unroll
        for (int q = 0; q < 4; ++q) {
          const float2 f = __bfloat1622float2(xv[q]);
          yv[q] = pack_bf16x2(f.x * e, f.y * e);
        }
        *reinterpret_cast<uint4*>(smem + SM_QS + b * 8192 + sw128(r, j)) = y;
      }
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(&ready[s]);
      tr(0, i);
      if (i + 1 < nch && !issue(i + 1)) {
        ok = false;
        break;
      }
      tr(11, i);
    }
    if (!ok) *abort_flag = 1;
  } else if (warp == 4) {
    // ------------------------------------------------------------------ MMA issuer
    constexpr uint32_t ID_N64 = idesc_bf16_f32(128, 64, false, false);
    constexpr uint32_t ID_N128_BMN = idesc_bf16_f32(128, 128, false, true);
    const uint32_t s_addr = smem_u32(smem + SM_S), va_addr = smem_u32(smem + SM_VA), vu_addr = smem_u32(smem + SM_VU);
    const uint32_t p_addr = smem_u32(smem + SM_P), qs_addr = smem_u32(smem + SM_QS);
    bool ok = true;
    for (int i = 0; i < nch && ok; ++i) {
      const int s = i & 1;
      const uint32_t st = smem_u32(smem + s * ST_BYTES);
      const uint32_t d2 = T_D2 + 64 * (i & 1);
      if (*abort_flag || !mbar_wait(&ready[s], (i >> 1) & 1, a.err, kErrTimeoutMma) ||
          !mbar_wait(ss_full, i & 1, a.err, kErrTimeoutMma) ||
          (i >= 2 && !mbar_wait(&d2_free[i & 1], ((i - 2) >> 1) & 1, a.err, kErrTimeoutMma))) {
        ok = false;
        break;
      }
      tc_fence_after();
      tr(1, i);
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < TC_D / 16; ++kk) {
          const uint32_t kb = (kk >> 2) * 16384 + (kk & 3) * 32;
          const uint64_t ad = sdesc_sw128(s_addr + kb, 16, 1024);
          umma_f16(tmem + T_D1, ad, sdesc_sw128(st + ST_QW + kb + 8192, 16, 1024), ID_N64, kk > 0);
          umma_f16(tmem + d2, ad, sdesc_sw128(qs_addr + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024), ID_N64, kk > 0);
        }
        umma_commit(d1_full);
#pragma unroll
        for (int kk = 0; kk < TC_D / 16; ++kk) {
          const uint64_t ad = sdesc_sw128(st + ST_QW + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = sdesc_sw128(st + ST_K + (kk >> 2) * 8192 + (kk & 3) * 32, 16, 1024);
          umma_f16(tmem + T_D3, ad, bd, ID_N64, kk > 0);
        }
        umma_commit(d3_full);
      }
      __syncwarp();
      if (!mbar_wait(v_full, i & 1, a.err, kErrTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tr(2, i);
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < TC_C / 16; ++kk)
          umma_f16(tmem + T_S, sdesc_sw128(va_addr + kk * 32, 16, 1024),
                   sdesc_sw128(st + ST_K + kk * 2048, 8192, 1024), ID_N128_BMN, 1u);
        umma_commit(s_done);
      }
      __syncwarp();
      if (!mbar_wait(p_full, i & 1, a.err, kErrTimeoutMma)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tr(3, i);
      if (lane == 0) {
#pragma unroll
        for (int kk = 0; kk < TC_C / 16; ++kk)
          umma_f16(tmem + d2, sdesc_sw128(vu_addr + kk * 32, 16, 1024), sdesc_sw128(p_addr + kk * 32, 16, 1024),
                   ID_N64, 1u);
        umma_commit(&o_full[i & 1]);
        umma_commit(&empty[s]);
      }
      __syncwarp();
    }
    if (!ok) *abort_flag = 1;
    if (lane == 0) umma_commit(drain);   // completes once everything issued above has
    __syncwarp();
    mbar_wait(drain, 0, a.err, kErrTimeoutMma);
  } else {
    // ------------------------------------------------------------------ state rows (thread = value dim m)
    const int m = threadIdx.x;
    const uint32_t lane_off = (uint32_t)(warp * 32) << 16;
    float* state = a.state + (long)h * TC_D * TC_D;
    // initial S^T row m into TMEM columns 0..127
    {
      const float* sp = MODE == 0 ? nullptr : a.start_buf + ((long)h * a.groups + blockIdx.z) * TC_D * TC_D;
#pragma unroll 1
      for (int c = 0; c < TC_D; c += 16) {
        uint32_t w[16];
#pragma unroll
        for (int e = 0; e < 16; ++e)
          w[e] = __float_as_uint(MODE == 0 ? state[(long)(c + e) * TC_D + m] : sp[(long)m * TC_D + c + e]);
        tmem_st16(tmem + lane_off + T_S + c, w);
      }
      tmem_wait_st();
    }
    bool ok = true;
    int prev_rows = 0, prev_r0 = 0;
    auto read_output = [&](int j) -> bool {   // O^T of chunk j (index in this CTA's range) -> out rows
      if (!mbar_wait(&o_full[j & 1], (j >> 1) & 1, a.err, kErrTimeoutEpilogue)) return false;
      tc_fence_after();
      const uint32_t d2 = T_D2 + 64 * (j & 1);
      __nv_bfloat16* dst = a.out + (long)prev_r0 * a.out_row + (long)h * TC_D + m;
#pragma unroll
      for (int c = 0; c < TC_C; c += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + d2 + c, v);
        tmem_wait_ld();
#pragma unroll
        for (int e = 0; e < 32; ++e)
          if (c + e < prev_rows) dst[(long)(c + e) * a.out_row] = __float2bfloat16(__uint_as_float(v[e]));
      }
      tc_fence_before();
      mbar_arrive(&d2_free[j & 1]);
      return true;
    };
    for (int i = 0; i < nch; ++i) {
      const int s = i & 1;
      const int c = c_begin + i;
      const int r0 = c * TC_C;
      const int rows = min(TC_C, a.n - r0);
      const uint8_t* st = smem + s * ST_BYTES;
      const float* gam = reinterpret_cast<const float*>(st + ST_GAM);
      if (*abort_flag || !mbar_wait(&ready[s], (i >> 1) & 1, a.err, kErrTimeoutEpilogue) ||
          (i >= 1 && !mbar_wait(s_done, (i - 1) & 1, a.err, kErrTimeoutEpilogue))) {
        ok = false;
        break;
      }
      tc_fence_after();
      tr(4, i);
      const float gl = gam[TC_C - 1];
      const float cd = __expf(gl);
      // S^T row -> bf16 operand; S^T *= e^gl in TMEM
#pragma unroll 1
      for (int c0 = 0; c0 < TC_D; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + T_S + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 w;
          w.x = pack_bf16x2(__uint_as_float(v[8 * j + 0]), __uint_as_float(v[8 * j + 1]));
          w.y = pack_bf16x2(__uint_as_float(v[8 * j + 2]), __uint_as_float(v[8 * j + 3]));
          w.z = pack_bf16x2(__uint_as_float(v[8 * j + 4]), __uint_as_float(v[8 * j + 5]));
          w.w = pack_bf16x2(__uint_as_float(v[8 * j + 6]), __uint_as_float(v[8 * j + 7]));
          const int kc = c0 + 8 * j;   // key dim of the chunk's first element
          *reinterpret_cast<uint4*>(smem + SM_S + (kc >> 6) * 16384 + sw128(m, (kc & 63) >> 3)) = w;
        }
        uint32_t w16a[16], w16b[16];
#pragma unroll
        for (int e = 0; e < 16; ++e) {
          w16a[e] = __float_as_uint(__uint_as_float(v[e]) * cd);
          w16b[e] = __float_as_uint(__uint_as_float(v[16 + e]) * cd);
        }
        tmem_st16(tmem + lane_off + T_S + c0, w16a);
        tmem_st16(tmem + lane_off + T_S + c0 + 16, w16b);
      }
      tmem_wait_st();
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(ss_full);
      tr(5, i);
      // V'^T row = U^T row - D1 row; as is (output) and times e^(gl - gam_c) (state update)
      if (!mbar_wait(d1_full, i & 1, a.err, kErrTimeoutEpilogue)) {
        ok = false;
        break;
      }
      tc_fence_after();
      tr(6, i);
#pragma unroll
      for (int c0 = 0; c0 < TC_C; c0 += 32) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_off + T_D1 + c0, v);
        tmem_wait_ld();
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          const int ch = (c0 >> 3) + j;
          const uint4 uw = *reinterpret_cast<const uint4*>(st + ST_U + sw128(m, ch));
          const __nv_bfloat162* uv = reinterpret_cast<const __nv_bfloat162*>(&uw);
          float vp[8];
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const float2 u = __bfloat1622float2(uv[q]);
            vp[2 * q] = u.x - __uint_as_float(v[8 * j + 2 * q]);
            vp[2 * q + 1] = u.y - __uint_as_float(v[8 * j + 2 * q + 1]);
          }
          uint4 wu, wa;
          uint32_t* wuv = reinterpret_cast<uint32_t*>(&wu);
          uint32_t* wav = reinterpret_cast<uint32_t*>(&wa);
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int cc = 8 * ch + 2 * q;
            wuv[q] = pack_bf16x2(vp[2 * q], vp[2 * q + 1]);
            wav[q] = pack_bf16x2(vp[2 * q] * __expf(gl - gam[cc]), vp[2 * q + 1] * __expf(gl - gam[cc + 1]));
          }
          *reinterpret_cast<uint4*>(smem + SM_VU + sw128(m, ch)) = wu;
          *reinterpret_cast<uint4*>(smem + SM_VA + sw128(m, ch)) = wa;
        }
      }
      fence_async_smem();
      tc_fence_before();
      mbar_arrive(v_full);
      tr(7, i);
      // P rows (threads 0..63): D3 row m times e^(gam_m - gam_c) for c <= m
      if (m < TC_C) {
        if (!mbar_wait(d3_full, i & 1, a.err, kErrTimeoutEpilogue)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const float gm = gam[m];
#pragma unroll
        for (int c0 = 0; c0 < TC_C; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + T_D3 + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            float p[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int cc = c0 + 8 * j + e;
              p[e] = cc <= m ? __uint_as_float(v[8 * j + e]) * __expf(gm - gam[cc]) : 0.f;
            }
            uint4 w;
            w.x = pack_bf16x2(p[0], p[1]);
            w.y = pack_bf16x2(p[2], p[3]);
            w.z = pack_bf16x2(p[4], p[5]);
            w.w = pack_bf16x2(p[6], p[7]);
            *reinterpret_cast<uint4*>(smem + SM_P + sw128(m, (c0 >> 3) + j)) = w;
          }
        }
        fence_async_smem();
        tc_fence_before();
        mbar_arrive(p_full);
      }
      tr(8, i);
      mbar_arrive(&empty[s]);   // this stage's U^T and decays are no longer read
      // output of the previous chunk (its products finished while this chunk's ran)
      if (i >= 1 && !read_output(i - 1)) {
        ok = false;
        break;
      }
      tr(9, i);
      prev_rows = rows;
      prev_r0 = r0;
    }
    if (ok && nch > 0) ok = read_output(nch - 1);
    if (ok && MODE == 0 && nch > 0) {
      ok = mbar_wait(s_done, (nch - 1) & 1, a.err, kErrTimeoutEpilogue);
      if (ok) {
        tc_fence_after();
#pragma unroll 1
        for (int c0 = 0; c0 < TC_D; c0 += 32) {
          uint32_t v[32];
          tmem_ld32(tmem + lane_off + T_S + c0, v);
          tmem_wait_ld();
#pragma unroll
          for (int e = 0; e < 32; ++e) state[(long)(c0 + e) * TC_D + m] = __uint_as_float(v[e]);
        }
      }
    }
    if (!ok) *abort_flag = 1;
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 4) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
}

PFN_cuTensorMapEncodeTiled_v12000 encode_gdn() {
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

// [heads][rows][128] bf16, box {64, 64, 1}, 128-byte swizzle (rows past `rows` read as zeros)
CUtensorMap map_rows(const void* base, long rows, int heads) {
  CUtensorMap tm;
  cuuint64_t dims[3] = {(cuuint64_t)TC_D, (cuuint64_t)rows, (cuuint64_t)heads};
  cuuint64_t strides[2] = {(cuuint64_t)TC_D * 2, (cuuint64_t)rows * TC_D * 2};
  cuuint32_t box[3] = {64, (cuuint32_t)TC_C, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = encode_gdn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("gdn_state_tc: tensor map encode failed " + std::to_string((int)r));
  return tm;
}

// U^T scratch [nv * n_chunks * 128 rows][64] bf16, box {64, 128}, 128-byte swizzle
CUtensorMap map_u(const void* base, long rows) {
  CUtensorMap tm;
  cuuint64_t dims[2] = {(cuuint64_t)TC_C, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)TC_C * 2};
  cuuint32_t box[2] = {(cuuint32_t)TC_C, (cuuint32_t)TC_D};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = encode_gdn()(&tm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box,
                            estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) throw std::runtime_error("gdn_state_tc: tensor map encode failed " + std::to_string((int)r));
  return tm;
}

}  // namespace

// Off by default: measured 2x slower than the register-resident mma.sync pass at 48 heads x 16K (2.62 vs 1.34 ms
// for the whole scan). The phase trace shows why: 8.7 us per chunk, of which the S -> bf16 operand conversion, the
// V' step, P and the output readout (thread work between the tensor-core products, one warp per scheduler) take
// 0.5 / 1.0 / 2.6 / 2.6 us and every role-to-role handoff about 1.5 us; the recurrence is latency-bound, and two
// TMEM -> register -> shared-memory round trips per chunk cost more than the mma.sync pass's whole chunk (3.3 us).
int gdn_state_tc = 0;
unsigned long long* gdn_tc_trace = nullptr;

bool gdn_state_out_tc(const GdnScanArgs& a, int n_pad, int mode, cudaStream_t stream) {
  if (!gdn_state_tc || a.q == nullptr || a.out == nullptr || a.dk != TC_D || a.dv != TC_D) return false;
  if (mode != 0 && mode != 2) return false;
  if (mode == 2 && a.start_buf == nullptr) return false;
  for (const void* p : {(const void*)a.q, (const void*)a.k, (const void*)a.w_buf, (const void*)a.u_buf})
    if (reinterpret_cast<uintptr_t>(p) % 16) return false;
  const int n_chunks = n_pad / TC_C;
  static PerDeviceOnce once;
  once([] {
    cudaFuncSetAttribute(gdn_state_tc_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
    cudaFuncSetAttribute(gdn_state_tc_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, SMEM_BYTES);
  });
  const CUtensorMap tq = map_rows(a.q, a.n, a.nk);
  const CUtensorMap tk = map_rows(a.k, a.n, a.nk);
  const CUtensorMap tw = map_rows(a.w_buf, n_pad, a.nv);
  const CUtensorMap tu = map_u(a.u_buf, (long)a.nv * n_chunks * TC_D);
  GdnTcArgs x{a.n,   a.nk,  a.nv,      n_chunks,  mode == 2 ? a.groups : 1, a.g, a.state, a.start_buf,
              a.out, a.out_row, a.err, gdn_tc_trace};
  if (mode == 0)
    gdn_state_tc_kernel<0><<<dim3(a.nv), 192, SMEM_BYTES, stream>>>(tq, tk, tw, tu, x);
  else
    gdn_state_tc_kernel<2><<<dim3(a.nv, 1, a.groups), 192, SMEM_BYTES, stream>>>(tq, tk, tw, tu, x);
  count_launch();
  return true;
}

}  // namespace rf
