// Gated DeltaNet on sm_100a.
//
// gdn_prep           per token: depthwise causal conv (K taps, previous rows from the conv state) + SiLU over
//                    the q|k|v channels, rounded to bf16; q, k l2-normalised per head (q times dk^-0.5);
//                    beta = sigmoid(b), g = -exp(A_log) softplus(a + dt_bias) in fp32. Outputs head-major.
// gdn_chunk_scan     chunked gated delta rule (chunk C = 64), two kernels:
//   wy kernel        (parallel over value head x chunk) gamma = cumsum(g); A = strictly-lower(beta_i k_i.k_j
//                    e^(gamma_i - gamma_j)); T = (I + A)^-1 by forward substitution (one column per thread);
//                    W = T (beta e^gamma k), U = T (beta v) -> bf16 scratch
//   scan kernel      (parallel over value head x 64-column slice of the state, sequential over chunks)
//                    V' = U - W S;  O = (q e^gamma) S + (q k^T * decay) V'  (output mode);
//                    S <- e^(gamma_C) S + (k e^(gamma_C - gamma))^T V'.
//                    The fp32 state lives in mma accumulators for the whole sequence. Output mode computes O
//                    in the same pass (gdn_state_out_kernel); the older split form (the state pass stores the
//                    chunk-start states and V', a parallel pass reads them back) stays behind
//                    gdn_fused_output = 0. Fill mode (q == nullptr) skips the output.
// Matches the reference's chunk arithmetic (code/kva/ops.py:199-262) with bf16 tensor-core products and
// fp32 accumulation/state.
#include "kernels.h"
#include "mma.cuh"
#include "ptx.cuh"

namespace rf {

constexpr int GC = 64;  // chunk length

__device__ __forceinline__ float softplus_f(float x) { return x > 20.f ? x : log1pf(expf(x)); }
__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16(x)); }

// ---------------------------------------------------------------------------------------- prep
// grid: (token blocks of 64, head tasks); head task [0, nk) q heads, [nk, 2nk) k heads, [2nk, 2nk + nv) v
// heads. The CTA stages rows [t0 - (K-1), t0 + 64) of its head's channels in shared memory (earlier rows
// from the conv state), then each warp produces 16 tokens: lane j owns channels 4j..4j+3.
constexpr int PREP_T = 64;

__global__ void __launch_bounds__(128) gdn_prep_kernel(GdnPrepArgs a) {
  __shared__ __align__(16) __nv_bfloat16 rows[(PREP_T + 7) * 128];
  __shared__ float wsh[128 * 8];
  const int t0 = blockIdx.x * PREP_T;
  const int task = blockIdx.y + (a.q == nullptr ? a.nk : 0);   // no q heads in fill mode
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int C = 2 * a.nk * a.dk + a.nv * a.dv;
  int c0, dh;
  if (task < 2 * a.nk) {
    c0 = task * a.dk;
    dh = a.dk;
  } else {
    c0 = 2 * a.nk * a.dk + (task - 2 * a.nk) * a.dv;
    dh = a.dv;
  }
  const int K1 = a.K - 1;
  const int nrows = min(PREP_T, a.n - t0) + K1;
  // stage rows (16-byte vectors when the row pitches allow them)
  const bool vec = (a.proj_row % 8 == 0) && (C % 8 == 0);
  if (vec) {
    for (int v = threadIdx.x; v < nrows * (dh / 8); v += 128) {
      const int r = v / (dh / 8), c = (v % (dh / 8)) * 8;
      const int src = t0 - K1 + r;
      uint4 val = make_uint4(0, 0, 0, 0);
      if (src >= 0)
        val = *reinterpret_cast<const uint4*>(a.proj + (long)src * a.proj_row + c0 + c);
      else if (a.conv_state != nullptr)
        val = *reinterpret_cast<const uint4*>(a.conv_state + (long)(K1 + src) * C + c0 + c);
      *reinterpret_cast<uint4*>(&rows[r * 128 + c]) = val;
    }
  } else {
    for (int v = threadIdx.x; v < nrows * dh; v += 128) {
      const int r = v / dh, c = v % dh;
      const int src = t0 - K1 + r;
      __nv_bfloat16 val = __float2bfloat16(0.f);
      if (src >= 0)
        val = a.proj[(long)src * a.proj_row + c0 + c];
      else if (a.conv_state != nullptr)
        val = a.conv_state[(long)(K1 + src) * C + c0 + c];
      rows[r * 128 + c] = val;
    }
  }
  // weights transposed to [tap][channel] so lanes (consecutive channels) hit distinct banks
  for (int v = threadIdx.x; v < dh * a.K; v += 128) {
    const int ch = v / a.K, tap = v % a.K;
    wsh[tap * 128 + ch] = __bfloat162float(a.conv_w[(long)c0 * a.K + v]);
  }
  __syncthreads();
  const int per = dh / 32;   // channels per lane: lane + 32 j
  const bool is_qk = task < 2 * a.nk;
  const bool is_q = task < a.nk;
  const float qscale = rsqrtf((float)a.dk);
  for (int tt = warp; tt < PREP_T; tt += 4) {
    const int tkn = t0 + tt;
    if (tkn >= a.n) break;
    float val[4];
    float ss = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      if (j >= per) break;
      const int ch = j * 32 + lane;
      float acc = 0.f;
      for (int tap = 0; tap < a.K; ++tap) acc += __bfloat162float(rows[(tt + tap) * 128 + ch]) * wsh[tap * 128 + ch];
      const float y = bf16r(acc / (1.f + __expf(-acc)));
      val[j] = y;
      ss += y * y;
    }
    float scale = 1.f;
    if (is_qk) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      scale = rsqrtf(ss + 1e-6f) * (is_q ? qscale : 1.f);
    }
    __nv_bfloat16* dst;
    if (is_qk) {
      const int hh = is_q ? task : task - a.nk;
      dst = (is_q ? a.q : a.k) + ((long)hh * a.n + tkn) * a.dk;
    } else {
      dst = a.v + ((long)(task - 2 * a.nk) * a.n + tkn) * a.dv;
    }
#pragma unroll
    for (int j = 0; j < 4; ++j)
      if (j < per) dst[j * 32 + lane] = __float2bfloat16(val[j] * scale);
  }
  if (blockIdx.y == 0) {   // gates of this token block
    for (int v = threadIdx.x; v < PREP_T * a.nv; v += 128) {
      const int tt = v / a.nv, h = v % a.nv;
      const int tkn = t0 + tt;
      if (tkn >= a.n) continue;
      const __nv_bfloat16* prow = a.proj + (long)tkn * a.proj_row;
      const float b = __bfloat162float(prow[a.b_off + h]);
      const float av = __bfloat162float(prow[a.a_off + h]);
      a.beta[(long)h * a.n + tkn] = bf16r(1.f / (1.f + expf(-b)));
      a.g[(long)h * a.n + tkn] = -expf(a.A_log[h]) * softplus_f(av + a.dt_bias[h]);
    }
  }
}

// Register form of gdn_prep for head dims 64 / 128 (NCH = 2 / 4 channels per lane, one 4- or 8-byte load per lane
// per token) and 4 conv taps: each warp walks PREP_RUN consecutive tokens of one head and keeps the conv window (the
// previous K - 1 pre-conv rows of its channels) and the conv taps in registers, so a token costs one global load and one store
// per lane; SiLU on the fast reciprocal. Same arithmetic order as gdn_prep_kernel (taps oldest first, fp32 sum,
// bf16 rounding of the conv output before the l2 norm).
constexpr int PREP_RUN = 16;      // tokens per warp
constexpr int PREP_WARPS = 8;     // warps per CTA (tokens per CTA = 128)

template <int NCH, int K>
__global__ void __launch_bounds__(32 * PREP_WARPS) gdn_prep_fast_kernel(GdnPrepArgs a) {
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int task = blockIdx.y + (a.q == nullptr ? a.nk : 0);   // no q heads in fill mode
  const int C = 2 * a.nk * a.dk + a.nv * a.dv;
  const bool is_qk = task < 2 * a.nk;
  const bool is_q = task < a.nk;
  const int c0 = is_qk ? task * a.dk : 2 * a.nk * a.dk + (task - 2 * a.nk) * a.dv;
  const int ch = c0 + lane * NCH;                       // this lane's first channel
  const int t_begin = (blockIdx.x * PREP_WARPS + warp) * PREP_RUN;
  if (t_begin < a.n) {
    float w[NCH][K];
#pragma unroll
    for (int j = 0; j < NCH; ++j)
#pragma unroll
      for (int tap = 0; tap < K; ++tap) w[j][tap] = __bfloat162float(a.conv_w[(long)(ch + j) * K + tap]);
    auto load_row = [&](int tkn, float (&x)[NCH]) {
      const __nv_bfloat16* src = nullptr;
      if (tkn >= 0) src = a.proj + (long)tkn * a.proj_row + ch;
      else if (a.conv_state != nullptr) src = a.conv_state + (long)(K - 1 + tkn) * C + ch;
      if (src == nullptr) {
#pragma unroll
        for (int j = 0; j < NCH; ++j) x[j] = 0.f;
      } else if constexpr (NCH == 4) {
        const uint2 v = *reinterpret_cast<const uint2*>(src);
        x[0] = bf16_lo(v.x); x[1] = bf16_hi(v.x); x[2] = bf16_lo(v.y); x[3] = bf16_hi(v.y);
      } else {
        const uint32_t v = *reinterpret_cast<const uint32_t*>(src);
        x[0] = bf16_lo(v); x[1] = bf16_hi(v);
      }
    };
    // window[s] holds the row s + 1 - K relative to the current token (oldest first); window[K - 1] = current
    float win[K][NCH];
#pragma unroll
    for (int s = 0; s < K - 1; ++s) load_row(t_begin - (K - 1) + s, win[s]);
    const float qscale = rsqrtf((float)a.dk);
    const int t_end = min(a.n, t_begin + PREP_RUN);
    const int hh = is_qk ? (is_q ? task : task - a.nk) : task - 2 * a.nk;
    __nv_bfloat16* dst_base = is_qk ? (is_q ? a.q : a.k) + (long)hh * a.n * a.dk
                                    : a.v + (long)hh * a.n * a.dv;
    const int dh = is_qk ? a.dk : a.dv;
    for (int tkn = t_begin; tkn < t_end; ++tkn) {
      load_row(tkn, win[K - 1]);
      float y[NCH];
      float ss = 0.f;
#pragma unroll
      for (int j = 0; j < NCH; ++j) {
        float acc = 0.f;
#pragma unroll
        for (int tap = 0; tap < K; ++tap) acc += win[tap][j] * w[j][tap];
        y[j] = bf16r(__fdividef(acc, 1.f + __expf(-acc)));
        ss += y[j] * y[j];
      }
      float scale = 1.f;
      if (is_qk) {
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
        scale = rsqrtf(ss + 1e-6f) * (is_q ? qscale : 1.f);
      }
      __nv_bfloat16* dst = dst_base + (long)tkn * dh + lane * NCH;
      if constexpr (NCH == 4) {
        *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(y[0] * scale, y[1] * scale),
                                                   pack_bf16x2(y[2] * scale, y[3] * scale));
      } else {
        *reinterpret_cast<uint32_t*>(dst) = pack_bf16x2(y[0] * scale, y[1] * scale);
      }
#pragma unroll
      for (int s = 0; s < K - 1; ++s)
#pragma unroll
        for (int j = 0; j < NCH; ++j) win[s][j] = win[s + 1][j];
    }
  }
  if (blockIdx.y == 0) {   // gates of this CTA's tokens
    const int t0 = blockIdx.x * PREP_WARPS * PREP_RUN;
    for (int v = threadIdx.x; v < PREP_WARPS * PREP_RUN * a.nv; v += 32 * PREP_WARPS) {
      const int tt = v / a.nv, h = v % a.nv;
      const int tkn = t0 + tt;
      if (tkn >= a.n) continue;
      const __nv_bfloat16* prow = a.proj + (long)tkn * a.proj_row;
      const float b = __bfloat162float(prow[a.b_off + h]);
      const float av = __bfloat162float(prow[a.a_off + h]);
      a.beta[(long)h * a.n + tkn] = bf16r(1.f / (1.f + expf(-b)));
      a.g[(long)h * a.n + tkn] = -expf(a.A_log[h]) * softplus_f(av + a.dt_bias[h]);
    }
  }
}

void gdn_prep(const GdnPrepArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  const int C = 2 * a.nk * a.dk + a.nv * a.dv;
  const bool fast = a.dk == a.dv && (a.dk == 128 || a.dk == 64) && a.K == 4 && a.proj_row % 4 == 0 && C % 4 == 0 &&
                    reinterpret_cast<uintptr_t>(a.proj) % 8 == 0 &&
                    (a.conv_state == nullptr || reinterpret_cast<uintptr_t>(a.conv_state) % 8 == 0);
  if (fast) {
    const int per_cta = PREP_WARPS * PREP_RUN;
    dim3 grid((a.n + per_cta - 1) / per_cta, (a.q == nullptr ? 1 : 2) * a.nk + a.nv);
    if (a.dk == 128) gdn_prep_fast_kernel<4, 4><<<grid, 32 * PREP_WARPS, 0, stream>>>(a);
    else gdn_prep_fast_kernel<2, 4><<<grid, 32 * PREP_WARPS, 0, stream>>>(a);
    count_launch();
    return;
  }
  dim3 grid((a.n + PREP_T - 1) / PREP_T, (a.q == nullptr ? 1 : 2) * a.nk + a.nv);
  gdn_prep_kernel<<<grid, 128, 0, stream>>>(a);
  count_launch();
}

// new state = last K-1 rows of [old state; proj rows]
__global__ void gdn_conv_state_kernel(const __nv_bfloat16* proj, long proj_row, __nv_bfloat16* state, int n, int C,
                                      int K) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= C) return;
  __nv_bfloat16 tmp[8];
  for (int r = 0; r < K - 1; ++r) {
    const int idx = n - (K - 1) + r;
    tmp[r] = idx >= 0 ? proj[(long)idx * proj_row + c] : state[(long)(K - 1 + idx) * C + c];
  }
  for (int r = 0; r < K - 1; ++r) state[(long)r * C + c] = tmp[r];
}

void gdn_conv_state_update(const __nv_bfloat16* proj, long proj_row, __nv_bfloat16* state, int n, int C, int K,
                           cudaStream_t stream) {
  gdn_conv_state_kernel<<<(C + 255) / 256, 256, 0, stream>>>(proj, proj_row, state, n, C, K); count_launch();
}

// ------------------------------------------------------------------------------------ wy kernel
constexpr int DK = 128;           // key head dim supported by the chunk kernels
constexpr int PK = DK + 8;        // smem pitch of [64][dk] tiles
constexpr int PA = GC + 1;        // fp32 [64][64] pitch

constexpr int PT = GC + 8;        // bf16 pitch of the ta / tb tiles
struct WySmem {
  __nv_bfloat16 k[GC * PK];
  __nv_bfloat16 v[GC * PK];       // dv <= 128
  // strictly lower A, then scratch of the blocked inverse; once T is complete the same bytes hold
  // ta = T diag(beta e^gam) and tb = T diag(beta) (bf16 [64][PT] each), which keeps the block at 3 CTAs per SM
  float A[(2 * GC * PT * 2 + 3) / 4 > GC * PA ? (2 * GC * PT * 2 + 3) / 4 : GC * PA];
  float T[GC * PA];               // (I + A)^-1
  float gam[GC];
  float beta[GC];
  float eg[GC];
};

// One distance D of the blocked inverse: for every pair (i, j = i - D) at once, X_ij = sum_{k=j}^{i-1} A_ik T_kj
// into A's upper block (j, i), then T_ij = -T_ii X_ij. Thread = (row r, columns c, c + 1) of every pair's block; the
// pairs' and columns' sums are independent chains (accumulated in registers, the k order as blk_mm's).
template <int D>
__device__ __forceinline__ void wy_offdiag(float* A, float* T, int tid) {
  constexpr int NP = 4 - D;
  const int r = tid >> 3, c = (tid & 7) * 2;
  float acc[NP][2];
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    acc[p][0] = acc[p][1] = 0.f;
#pragma unroll
    for (int k = p; k < p + D; ++k) {
      const float* xr = A + ((p + D) * 16 + r) * PA + k * 16;
      const float* yc = T + (k * 16) * PA + p * 16 + c;
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        const float x = xr[e];
        acc[p][0] += x * yc[e * PA];
        acc[p][1] += x * yc[e * PA + 1];
      }
    }
  }
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    float* o = A + (p * 16 + r) * PA + (p + D) * 16 + c;
    o[0] = acc[p][0];
    o[1] = acc[p][1];
  }
  __syncthreads();
#pragma unroll
  for (int p = 0; p < NP; ++p) {
    const int i = p + D;
    const float* xr = T + (i * 16 + r) * PA + i * 16;
    const float* yc = A + (p * 16) * PA + i * 16 + c;
    float a0 = 0.f, a1 = 0.f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float x = xr[e];
      a0 += x * yc[e * PA];
      a1 += x * yc[e * PA + 1];
    }
    float* o = T + (i * 16 + r) * PA + p * 16 + c;
    o[0] = -a0;
    o[1] = -a1;
  }
  __syncthreads();
}

__global__ void __launch_bounds__(128) gdn_wy_kernel(GdnScanArgs a, int n_pad) {
  extern __shared__ __align__(16) uint8_t wy_raw[];
  WySmem& s = *reinterpret_cast<WySmem*>(wy_raw);
  const int chunk = blockIdx.x;
  const int h = blockIdx.y;
  const int kh = h / (a.nv / a.nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = chunk * GC;
  const int rows = min(GC, a.n - r0);
  const int dv = a.dv;

  const __nv_bfloat16* kp = a.k + ((long)kh * a.n + r0) * DK;
  const __nv_bfloat16* vp = a.v + ((long)h * a.n + r0) * dv;
  for (int v = tid; v < GC * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    const bool ok = r < rows;
    cp_async16(&s.k[r * PK + c], ok ? kp + (long)r * DK + c : kp, ok);
  }
  for (int v = tid; v < GC * (dv / 8); v += 128) {
    const int r = v / (dv / 8), c = (v % (dv / 8)) * 8;
    const bool ok = r < rows;
    cp_async16(&s.v[r * PK + c], ok ? vp + (long)r * dv + c : vp, ok);
  }
  cp_async_commit();
  if (tid < GC) {
    const bool ok = tid < rows;
    s.beta[tid] = ok ? a.beta[(long)h * a.n + r0 + tid] : 0.f;
    s.gam[tid] = ok ? a.g[(long)h * a.n + r0 + tid] : 0.f;
  }
  __syncthreads();
  if (warp == 0) {  // inclusive cumsum of 64 values, 2 per lane
    const float x0 = s.gam[2 * lane], x1 = s.gam[2 * lane + 1];
    const float pair = x0 + x1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s.gam[2 * lane] = incl - pair + x0;
    s.gam[2 * lane + 1] = incl;
    s.eg[2 * lane] = __expf(incl - pair + x0);
    s.eg[2 * lane + 1] = __expf(incl);
  }
  cp_async_wait<0>();
  __syncthreads();

  // A = strictly lower(beta_i * k_i.k_j * exp(gam_i - gam_j)) from KK^T (16 rows per warp)
  {
    float acc[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks) {
      uint32_t af[4];
      lda_row(af, s.k, PK, warp * 16, ks * 16, lane);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.k, PK, j2 * 16, ks * 16, lane);
        mma_bf16(acc[2 * j2], af, bf[0], bf[1]);
        mma_bf16(acc[2 * j2 + 1], af, bf[2], bf[3]);
      }
    }
    const int ra = warp * 16 + g, rb = ra + 8;
    const float ba = s.beta[ra], bb = s.beta[rb], ga = s.gam[ra], gb = s.gam[rb];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = (e >= 2) ? rb : ra;
        const int c = j * 8 + 2 * t + (e & 1);
        const float v = (r > c) ? ((e >= 2) ? bb : ba) * acc[j][e] * __expf(((e >= 2) ? gb : ga) - s.gam[c]) : 0.f;
        s.A[r * PA + c] = v;
        s.T[r * PA + c] = 0.f;
      }
    }
  }
  __syncthreads();
  // (I + A)^-1, blocked 4 x 4 in 16 x 16 blocks. Diagonal blocks by forward substitution: warp w inverts
  // block w, lane c < 16 owning column c, kept in registers (entries above the diagonal are zero, so the sum over
  // j < c adds nothing and the order of the nonzero terms is j = c .. r - 1, as before).
  if (lane < 16) {
    const int b0 = warp * 16;
    const int c = lane;
    float tc[16];
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float v = (r == c) ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < r; ++j) v -= s.A[(b0 + r) * PA + b0 + j] * tc[j];
      tc[r] = (r >= c) ? v : 0.f;
      s.T[(b0 + r) * PA + b0 + c] = tc[r];
    }
  }
  __syncthreads();
  // Off-diagonal blocks by distance: T_ij = -T_ii * sum_{k=j}^{i-1} A_ik T_kj (scratch X_ij in the zero
  // upper triangle of A: block (j, i)); every pair of one distance in flight at once.
  wy_offdiag<1>(s.A, s.T, tid);
  wy_offdiag<2>(s.A, s.T, tid);
  wy_offdiag<3>(s.A, s.T, tid);
  // ta = T diag(beta e^gam), tb = T diag(beta) (bf16, lower triangle incl. diagonal), over A's bytes
  __nv_bfloat16* s_ta = reinterpret_cast<__nv_bfloat16*>(s.A);
  __nv_bfloat16* s_tb = s_ta + GC * PT;
  for (int v = tid; v < GC * (GC / 2); v += 128) {
    const int r = v / (GC / 2), c = (v % (GC / 2)) * 2;
    const float t0 = r >= c ? s.T[r * PA + c] : 0.f;
    const float t1 = r >= c + 1 ? s.T[r * PA + c + 1] : 0.f;
    *reinterpret_cast<uint32_t*>(&s_ta[r * PT + c]) = pack2(t0 * s.beta[c] * s.eg[c], t1 * s.beta[c + 1] * s.eg[c + 1]);
    *reinterpret_cast<uint32_t*>(&s_tb[r * PT + c]) = pack2(t0 * s.beta[c], t1 * s.beta[c + 1]);
  }
  __syncthreads();
  // W = ta k [64 x dk] -> w_buf rows; U^T = v^T tb^T [dv x 64] -> u_buf as per-chunk [dv][64] tiles
  {
    __nv_bfloat16* wdst = a.w_buf + ((long)h * n_pad + r0) * DK;
    uint32_t af[4][4];
#pragma unroll
    for (int ks = 0; ks < GC / 16; ++ks) lda_row(af[ks], s_ta, PT, warp * 16, ks * 16, lane);
    for (int nb = 0; nb < DK; nb += 64) {
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < GC / 16; ++ks) {
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_kn(bf, s.k, PK, nb + j2 * 16, ks * 16, lane);
          mma_bf16(acc[2 * j2], af[ks], bf[0], bf[1]);
          mma_bf16(acc[2 * j2 + 1], af[ks], bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = warp * 16 + g;
        const int c = nb + j * 8 + 2 * t;
        *reinterpret_cast<uint32_t*>(wdst + (long)r * DK + c) = pack2(acc[j][0], acc[j][1]);
        *reinterpret_cast<uint32_t*>(wdst + (long)(r + 8) * DK + c) = pack2(acc[j][2], acc[j][3]);
      }
    }
  }
  {
    __nv_bfloat16* udst = a.u_buf + ((long)h * n_pad + r0) * dv;   // [dv][64] tile of this chunk
    for (int mb = warp * 16; mb < dv; mb += 64) {
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < GC / 16; ++ks) {
        uint32_t af[4];
        lda_trans(af, s.v, PK, mb, ks * 16, lane);        // A = v^T [dv][rows]
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_nk(bf, s_tb, PT, j2 * 16, ks * 16, lane);  // B[k][n] = tb[n][k]
          mma_bf16(acc[2 * j2], af, bf[0], bf[1]);
          mma_bf16(acc[2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int m = mb + g;
        const int c = j * 8 + 2 * t;
        *reinterpret_cast<uint32_t*>(udst + (long)m * GC + c) = pack2(acc[j][0], acc[j][1]);
        *reinterpret_cast<uint32_t*>(udst + (long)(m + 8) * GC + c) = pack2(acc[j][2], acc[j][3]);
      }
    }
  }
}

// ------------------------------------------------------------------------------ state pass kernel
// Sequential over chunks, parallel over (value head, 64-row slice of S^T); 4 warps, each owning 16 rows of
// the transposed state S^T [dv][dk] in mma accumulators. Per chunk, per warp (no inter-warp exchange):
//   V'^T = U^T - S^T W^T          (A = S^T straight from the accumulators, B = W rows from smem)
//   S^T  <- e^(gl) S^T + (V'^T diag(e^(gl - gam))) k     (A = scaled V'^T from the accumulators, B = k rows)
// The C-fragment layout of one product is the A-fragment layout of the next, so S and V' never leave the
// registers. Output mode stores the chunk-start S^T and the unscaled V'^T (bf16) for the output pass.
// Inputs of chunk c+2 are fetched (cp.async, 3 stages) while chunk c computes.
constexpr int SVS = 64;           // S^T rows (value dims) per CTA
constexpr int SST = 3;            // pipeline stages
constexpr int PU = GC + 8;        // pitch of the [dv][64] U^T tiles

struct StateSmem {
  __nv_bfloat16 w[SST][GC * PK];
  __nv_bfloat16 k[SST][GC * PK];
  __nv_bfloat16 ut[SST][SVS * PU];
  float g[SST][GC];
};

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem, bool pred) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  const int sz = pred ? 4 : 0;
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4, %2;" ::"r"(s), "l"(gmem), "r"(sz) : "memory");
}

__device__ __forceinline__ void state_issue_loads(StateSmem& s, const GdnScanArgs& a, int stage, int chunk, int h,
                                                  int kh, int m0, int n_pad, int tid) {
  const int r0 = chunk * GC;
  const int rows = min(GC, a.n - r0);
  const __nv_bfloat16* wp = a.w_buf + ((long)h * n_pad + r0) * DK;
  const __nv_bfloat16* up = a.u_buf + ((long)h * n_pad + r0) * a.dv + (long)m0 * GC;
  const __nv_bfloat16* kp = a.k + ((long)kh * a.n + r0) * DK;
  for (int v = tid; v < GC * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    cp_async16(&s.w[stage][r * PK + c], wp + (long)r * DK + c, true);   // padded rows hold zeros
    const bool ok = r < rows;
    cp_async16(&s.k[stage][r * PK + c], ok ? kp + (long)r * DK + c : kp, ok);
  }
  for (int v = tid; v < SVS * (GC / 8); v += 128) {
    const int r = v / (GC / 8), c = (v % (GC / 8)) * 8;
    cp_async16(&s.ut[stage][r * PU + c], up + (long)r * GC + c, true);
  }
  if (tid < GC) {
    const float* gp = a.g + (long)h * a.n + r0;
    cp_async4(&s.g[stage][tid], tid < rows ? gp + tid : gp, tid < rows);
  }
}

// MODE 0: sequential over every chunk from a.state (updated in place).
// MODE 1 (two-level scan, pass 1): blockIdx.z = chunk group; blockIdx.y < dv / SVS: the group's end state from a
//        zero start (R); blockIdx.y >= dv / SVS: the group's transfer matrix P (start from the identity, U = 0),
//        since S_end = S_start P + R is linear in S_start. Both go to grp_buf.
// MODE 2 (two-level scan, pass 3): blockIdx.z = chunk group, start from start_buf, output-mode stores only.
template <int MODE>
__global__ void __launch_bounds__(128, 1) gdn_state_kernel(GdnScanArgs a, int n_pad, __nv_bfloat16* s_buf,
                                                           __nv_bfloat16* vt_buf) {
  extern __shared__ __align__(16) uint8_t st_raw[];
  StateSmem& s = *reinterpret_cast<StateSmem*>(st_raw);
  const int h = blockIdx.x;
  const int slices = a.dv / SVS;
  const bool transfer = MODE == 1 && (int)blockIdx.y >= slices;   // computing P (U = 0, identity start)
  const int m0 = (MODE == 1 ? (int)blockIdx.y % slices : (int)blockIdx.y) * SVS;   // first value dim of this CTA
  const int kh = h / (a.nv / a.nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mrow = warp * 16;                      // this warp's rows within the slice
  const int n_chunks_all = (a.n + GC - 1) / GC;
  const int per_group = MODE == 0 ? n_chunks_all : (n_chunks_all + a.groups - 1) / a.groups;
  const int c_begin = MODE == 0 ? 0 : (int)blockIdx.z * per_group;
  const int c_end = MODE == 0 ? n_chunks_all : min(n_chunks_all, c_begin + per_group);
  const int n_chunks = n_chunks_all;               // chunk indexing of the scratch buffers
  float* state = a.state + (long)h * DK * a.dv;    // S [dk][dv]
  const long grp_mat = (long)a.dv * DK;            // one [dv][dk] matrix
  const long grp_idx = ((long)h * a.groups + blockIdx.z) * grp_mat;

  // S^T accumulators: rows m0 + mrow + (g, g+8), cols (dk) nt * 8 + 2t (+1)
  float S[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int m = m0 + mrow + g;
    const int c = nt * 8 + 2 * t;
    if constexpr (MODE == 0) {
      S[nt][0] = state[(long)c * a.dv + m];
      S[nt][1] = state[(long)(c + 1) * a.dv + m];
      S[nt][2] = state[(long)c * a.dv + m + 8];
      S[nt][3] = state[(long)(c + 1) * a.dv + m + 8];
    } else if constexpr (MODE == 1) {
      S[nt][0] = (transfer && c == m) ? 1.f : 0.f;
      S[nt][1] = (transfer && c + 1 == m) ? 1.f : 0.f;
      S[nt][2] = (transfer && c == m + 8) ? 1.f : 0.f;
      S[nt][3] = (transfer && c + 1 == m + 8) ? 1.f : 0.f;
    } else {
      const float* sp = a.start_buf + grp_idx;
      S[nt][0] = sp[(long)m * DK + c];
      S[nt][1] = sp[(long)m * DK + c + 1];
      S[nt][2] = sp[(long)(m + 8) * DK + c];
      S[nt][3] = sp[(long)(m + 8) * DK + c + 1];
    }
  }
  for (int p = 0; p < SST - 1; ++p) {
    if (c_begin + p < c_end) state_issue_loads(s, a, p, c_begin + p, h, kh, m0, n_pad, tid);
    cp_async_commit();
  }
  for (int ch = c_begin; ch < c_end; ++ch) {
    const int stage = (ch - c_begin) % SST;
    if (ch + SST - 1 < c_end)
      state_issue_loads(s, a, (ch - c_begin + SST - 1) % SST, ch + SST - 1, h, kh, m0, n_pad, tid);
    cp_async_commit();
    cp_async_wait<SST - 1>();
    __syncthreads();
    // S^T as bf16 A fragments (k = dk in steps of 16: n-tiles 2ks, 2ks + 1)
    uint32_t sa[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      sa[ks][0] = pack2(S[2 * ks][0], S[2 * ks][1]);
      sa[ks][1] = pack2(S[2 * ks][2], S[2 * ks][3]);
      sa[ks][2] = pack2(S[2 * ks + 1][0], S[2 * ks + 1][1]);
      sa[ks][3] = pack2(S[2 * ks + 1][2], S[2 * ks + 1][3]);
    }
    if (s_buf != nullptr) {   // chunk-start S^T, bf16 [dv][dk] per chunk
      __nv_bfloat16* sb = s_buf + (((long)h * n_chunks + ch) * a.dv + m0 + mrow) * DK;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const int c = ks * 16 + 2 * t;
        *reinterpret_cast<uint32_t*>(sb + (long)g * DK + c) = sa[ks][0];
        *reinterpret_cast<uint32_t*>(sb + (long)(g + 8) * DK + c) = sa[ks][1];
        *reinterpret_cast<uint32_t*>(sb + (long)g * DK + c + 8) = sa[ks][2];
        *reinterpret_cast<uint32_t*>(sb + (long)(g + 8) * DK + c + 8) = sa[ks][3];
      }
    }
    // gates: every warp scans the chunk's log decays (lane l holds gam[2l], gam[2l + 1])
    const float x0 = s.g[stage][2 * lane], x1 = s.g[stage][2 * lane + 1];
    const float pair = x0 + x1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float gl = __shfl_sync(0xffffffffu, incl, 31);
    const float f_even = __expf(gl - (incl - pair + x0)), f_odd = __expf(gl - incl);
    // V'^T = U^T - S^T W^T: [16 x 64], n-tiles over chunk rows
    float vt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) vt[j][0] = vt[j][1] = vt[j][2] = vt[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.w[stage], PK, j2 * 16, ks * 16, lane);   // B[k = dk][n = row] = W[row][dk]
        mma_bf16(vt[2 * j2], sa[ks], bf[0], bf[1]);
        mma_bf16(vt[2 * j2 + 1], sa[ks], bf[2], bf[3]);
      }
    }
    const __nv_bfloat16* ut = s.ut[stage];
    __nv_bfloat16* vtg = vt_buf != nullptr ? vt_buf + (((long)h * n_chunks + ch) * a.dv + m0 + mrow) * GC : nullptr;
    uint32_t va[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + 2 * t;                      // chunk rows c, c + 1
      float2 u0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[(mrow + g) * PU + c]));
      float2 u1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[(mrow + g + 8) * PU + c]));
      if (transfer) u0 = u1 = make_float2(0.f, 0.f);
      const float v0 = u0.x - vt[j][0], v1 = u0.y - vt[j][1], v2 = u1.x - vt[j][2], v3 = u1.y - vt[j][3];
      if (vtg != nullptr) {
        *reinterpret_cast<uint32_t*>(vtg + (long)g * GC + c) = pack2(v0, v1);
        *reinterpret_cast<uint32_t*>(vtg + (long)(g + 8) * GC + c) = pack2(v2, v3);
      }
      // decay factors of chunk rows c, c + 1 (= lane (c >> 1)'s pair)
      const float fc0 = __shfl_sync(0xffffffffu, f_even, c >> 1);
      const float fc1 = __shfl_sync(0xffffffffu, f_odd, c >> 1);
      const uint32_t lo = pack2(v0 * fc0, v1 * fc1), hi = pack2(v2 * fc0, v3 * fc1);
      va[j >> 1][(j & 1) ? 2 : 0] = lo;
      va[j >> 1][(j & 1) ? 3 : 1] = hi;
    }
    // S^T <- e^gl S^T + Vs^T k
    const float cd = __expf(gl);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      S[nt][0] *= cd;
      S[nt][1] *= cd;
      S[nt][2] *= cd;
      S[nt][3] *= cd;
    }
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 8; ++j2) {
        uint32_t bf[4];
        ldb_kn(bf, s.k[stage], PK, j2 * 16, ks * 16, lane);   // B[k = row][n = dk] = k[row][dk]
        mma_bf16(S[2 * j2], va[ks], bf[0], bf[1]);
        mma_bf16(S[2 * j2 + 1], va[ks], bf[2], bf[3]);
      }
    }
    __syncthreads();   // this stage is refilled two iterations later
  }
  cp_async_wait<0>();
  if constexpr (MODE == 2) return;                 // the group-end state is known from pass 2
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int m = m0 + mrow + g;
    const int c = nt * 8 + 2 * t;
    if constexpr (MODE == 0) {
      state[(long)c * a.dv + m] = S[nt][0];
      state[(long)(c + 1) * a.dv + m] = S[nt][1];
      state[(long)c * a.dv + m + 8] = S[nt][2];
      state[(long)(c + 1) * a.dv + m + 8] = S[nt][3];
    } else if (!transfer) {
      float* dst = a.grp_buf + grp_idx;
      *reinterpret_cast<float2*>(dst + (long)m * DK + c) = make_float2(S[nt][0], S[nt][1]);
      *reinterpret_cast<float2*>(dst + (long)(m + 8) * DK + c) = make_float2(S[nt][2], S[nt][3]);
    } else {
      // P as split bf16 (hi [dk][dk] then lo [dk][dk]) in its fp32 slot: pass 2 streams it with cp.async
      __nv_bfloat16* hi = reinterpret_cast<__nv_bfloat16*>(a.grp_buf + (long)a.nv * a.groups * grp_mat + grp_idx);
      __nv_bfloat16* lo = hi + (long)DK * DK;
      const float x[4] = {S[nt][0], S[nt][1], S[nt][2], S[nt][3]};
      float hx[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) hx[e] = __bfloat162float(__float2bfloat16(x[e]));
      *reinterpret_cast<uint32_t*>(hi + (long)m * DK + c) = pack2(hx[0], hx[1]);
      *reinterpret_cast<uint32_t*>(hi + (long)(m + 8) * DK + c) = pack2(hx[2], hx[3]);
      *reinterpret_cast<uint32_t*>(lo + (long)m * DK + c) = pack2(x[0] - hx[0], x[1] - hx[1]);
      *reinterpret_cast<uint32_t*>(lo + (long)(m + 8) * DK + c) = pack2(x[2] - hx[2], x[3] - hx[3]);
    }
  }
}

// ---------------------------------------------------------------------- two-level scan, pass 2
// Per (value head, 64-row slice of S^T): sequentially over the chunk groups, S_start(z + 1) = S_start(z) P_z + R_z
// (written to start_buf for pass 3 in output mode); the last one is the final state. The product runs on the
// tensor cores with split-bf16 operands (hi + lo; hi*hi + hi*lo + lo*hi), about fp32 accurate, so the state
// never passes through a single bf16 rounding. The next group's P halves stream in (cp.async, double buffer)
// while the current group's product runs.
constexpr int PP = DK + 8;        // pitch of the staged P halves
struct PropSmem {
  __nv_bfloat16 hi[2][DK * PP];
  __nv_bfloat16 lo[2][DK * PP];
};

__device__ __forceinline__ void prop_issue(PropSmem& s, const __nv_bfloat16* src, int buf, int tid) {
  for (int v = tid; v < DK * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    cp_async16(&s.hi[buf][r * PP + c], src + (long)r * DK + c, true);
    cp_async16(&s.lo[buf][r * PP + c], src + (long)DK * DK + (long)r * DK + c, true);
  }
}

__global__ void __launch_bounds__(128, 1) gdn_group_prop_kernel(GdnScanArgs a, int write_starts) {
  extern __shared__ __align__(16) uint8_t pp_raw[];
  PropSmem& s = *reinterpret_cast<PropSmem*>(pp_raw);
  const int h = blockIdx.x, m0 = blockIdx.y * SVS;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mrow = warp * 16;
  float* state = a.state + (long)h * DK * a.dv;
  const long mat = (long)a.dv * DK;
  const float* R = a.grp_buf;
  const float* Pbase = a.grp_buf + (long)a.nv * a.groups * mat;
  float S[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int m = m0 + mrow + g, c = nt * 8 + 2 * t;
    S[nt][0] = state[(long)c * a.dv + m];
    S[nt][1] = state[(long)(c + 1) * a.dv + m];
    S[nt][2] = state[(long)c * a.dv + m + 8];
    S[nt][3] = state[(long)(c + 1) * a.dv + m + 8];
  }
  prop_issue(s, reinterpret_cast<const __nv_bfloat16*>(Pbase + (long)h * a.groups * mat), 0, tid);
  cp_async_commit();
  for (int z = 0; z < a.groups; ++z) {
    const long idx = ((long)h * a.groups + z) * mat;
    const int buf = z & 1;
    if (z + 1 < a.groups)
      prop_issue(s, reinterpret_cast<const __nv_bfloat16*>(Pbase + idx + mat), buf ^ 1, tid);
    cp_async_commit();
    if (write_starts) {
      float* sp = a.start_buf + idx;
#pragma unroll
      for (int nt = 0; nt < 16; ++nt) {
        const int m = m0 + mrow + g, c = nt * 8 + 2 * t;
        *reinterpret_cast<float2*>(sp + (long)m * DK + c) = make_float2(S[nt][0], S[nt][1]);
        *reinterpret_cast<float2*>(sp + (long)(m + 8) * DK + c) = make_float2(S[nt][2], S[nt][3]);
      }
    }
    float acc[16][4];
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int m = m0 + mrow + g, c = nt * 8 + 2 * t;
      const float2 r0 = *reinterpret_cast<const float2*>(R + idx + (long)m * DK + c);
      const float2 r1 = *reinterpret_cast<const float2*>(R + idx + (long)(m + 8) * DK + c);
      acc[nt][0] = r0.x;
      acc[nt][1] = r0.y;
      acc[nt][2] = r1.x;
      acc[nt][3] = r1.y;
    }
    // A fragments of S^T (hi and lo), K = dk in 8 steps of 16
    uint32_t ah[8][4], al[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float* src = S[2 * ks + (e >> 1)];
        const float x0 = src[(e & 1) * 2], x1 = src[(e & 1) * 2 + 1];
        const float h0 = __bfloat162float(__float2bfloat16(x0)), h1 = __bfloat162float(__float2bfloat16(x1));
        ah[ks][e] = pack2(h0, h1);
        al[ks][e] = pack2(x0 - h0, x1 - h1);
      }
    }
    cp_async_wait<1>();
    __syncthreads();
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 8; ++j2) {
        uint32_t bh[4], bl[4];
        ldb_kn(bh, s.hi[buf], PP, j2 * 16, ks * 16, lane);   // B[k = row of P][n = col of P]
        ldb_kn(bl, s.lo[buf], PP, j2 * 16, ks * 16, lane);
        mma_bf16(acc[2 * j2], ah[ks], bh[0], bh[1]);
        mma_bf16(acc[2 * j2 + 1], ah[ks], bh[2], bh[3]);
        mma_bf16(acc[2 * j2], ah[ks], bl[0], bl[1]);
        mma_bf16(acc[2 * j2 + 1], ah[ks], bl[2], bl[3]);
        mma_bf16(acc[2 * j2], al[ks], bh[0], bh[1]);
        mma_bf16(acc[2 * j2 + 1], al[ks], bh[2], bh[3]);
      }
    }
    __syncthreads();   // buffer `buf` is refilled by the next iteration's prefetch
#pragma unroll
    for (int nt = 0; nt < 16; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) S[nt][e] = acc[nt][e];
  }
  cp_async_wait<0>();
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int m = m0 + mrow + g, c = nt * 8 + 2 * t;
    state[(long)c * a.dv + m] = S[nt][0];
    state[(long)(c + 1) * a.dv + m] = S[nt][1];
    state[(long)c * a.dv + m + 8] = S[nt][2];
    state[(long)(c + 1) * a.dv + m + 8] = S[nt][3];
  }
}

// -------------------------------------------------------------------------- fused state + output pass
// Output mode without the chunk-state round trip: the sequential state pass itself produces every chunk's output
// rows for its 64 value dims, so the chunk-start states (bf16 [dv][dk] per chunk) and V' never go to memory and
// the separate output pass disappears. Per chunk, warp w (value dims m0 + 16w .. + 16):
//   P      = rows 16w.. of the chunk's (q k^T) * e^(gam_r - gam_c) (r >= c), bf16 -> shared memory (all warps)
//   O^T    = S^T q^T, column r scaled by e^(gam_r)               (A = S^T from the accumulators, B = q rows)
//   V'^T   = U^T - S^T W^T                                        (as in the state pass)
//   O^T   += V'^T P^T                                             (A = V'^T from the accumulators, B = P rows)
//   S^T   <- e^(gl) S^T + (V'^T diag(e^(gl - gam))) k             (as in the state pass)
// O^T is staged transposed in shared memory and stored as whole 128-byte row segments. The recurrence's chain is
// unchanged; the output products are independent of it and fill its latency.
// MODE 0: sequential over every chunk from a.state (updated in place); MODE 2: one chunk group of the two-level
// scan from start_buf (its end state is known from pass 2).
constexpr int PQ = GC + 8;        // pitch of the P tile and of the output staging tile

struct StateOutSmem {
  __nv_bfloat16 w[SST][GC * PK];
  __nv_bfloat16 k[SST][GC * PK];
  __nv_bfloat16 q[SST][GC * PK];
  __nv_bfloat16 ut[SST][SVS * PU];
  float g[SST][GC];
  __nv_bfloat16 p[GC * PQ];       // masked, decayed q k^T of the chunk
  __nv_bfloat16 o[GC * PQ];       // output rows x this CTA's 64 value dims
};

__device__ __forceinline__ void state_out_issue_loads(StateOutSmem& s, const GdnScanArgs& a, int stage, int chunk,
                                                      int h, int kh, int m0, int n_pad, int tid) {
  const int r0 = chunk * GC;
  const int rows = min(GC, a.n - r0);
  const __nv_bfloat16* wp = a.w_buf + ((long)h * n_pad + r0) * DK;
  const __nv_bfloat16* up = a.u_buf + ((long)h * n_pad + r0) * a.dv + (long)m0 * GC;
  const __nv_bfloat16* kp = a.k + ((long)kh * a.n + r0) * DK;
  const __nv_bfloat16* qp = a.q + ((long)kh * a.n + r0) * DK;
  for (int v = tid; v < GC * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    cp_async16(&s.w[stage][r * PK + c], wp + (long)r * DK + c, true);   // padded rows hold zeros
    const bool ok = r < rows;
    cp_async16(&s.k[stage][r * PK + c], ok ? kp + (long)r * DK + c : kp, ok);
    cp_async16(&s.q[stage][r * PK + c], ok ? qp + (long)r * DK + c : qp, ok);
  }
  for (int v = tid; v < SVS * (GC / 8); v += 128) {
    const int r = v / (GC / 8), c = (v % (GC / 8)) * 8;
    cp_async16(&s.ut[stage][r * PU + c], up + (long)r * GC + c, true);
  }
  if (tid < GC) {
    const float* gp = a.g + (long)h * a.n + r0;
    cp_async4(&s.g[stage][tid], tid < rows ? gp + tid : gp, tid < rows);
  }
}

template <int MODE>
__global__ void __launch_bounds__(128, 1) gdn_state_out_kernel(GdnScanArgs a, int n_pad) {
  static_assert(MODE == 0 || MODE == 2, "sequential scan or the two-level scan's output pass");
  extern __shared__ __align__(16) uint8_t so_raw[];
  StateOutSmem& s = *reinterpret_cast<StateOutSmem*>(so_raw);
  const int h = blockIdx.x;
  const int m0 = (int)blockIdx.y * SVS;
  const int kh = h / (a.nv / a.nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int mrow = warp * 16;
  const int n_chunks_all = (a.n + GC - 1) / GC;
  const int per_group = MODE == 0 ? n_chunks_all : (n_chunks_all + a.groups - 1) / a.groups;
  const int c_begin = MODE == 0 ? 0 : (int)blockIdx.z * per_group;
  const int c_end = MODE == 0 ? n_chunks_all : min(n_chunks_all, c_begin + per_group);
  float* state = a.state + (long)h * DK * a.dv;
  const long grp_idx = ((long)h * a.groups + blockIdx.z) * ((long)a.dv * DK);

  float S[16][4];
#pragma unroll
  for (int nt = 0; nt < 16; ++nt) {
    const int m = m0 + mrow + g;
    const int c = nt * 8 + 2 * t;
    if constexpr (MODE == 0) {
      S[nt][0] = state[(long)c * a.dv + m];
      S[nt][1] = state[(long)(c + 1) * a.dv + m];
      S[nt][2] = state[(long)c * a.dv + m + 8];
      S[nt][3] = state[(long)(c + 1) * a.dv + m + 8];
    } else {
      const float* sp = a.start_buf + grp_idx;
      S[nt][0] = sp[(long)m * DK + c];
      S[nt][1] = sp[(long)m * DK + c + 1];
      S[nt][2] = sp[(long)(m + 8) * DK + c];
      S[nt][3] = sp[(long)(m + 8) * DK + c + 1];
    }
  }
  for (int p = 0; p < SST - 1; ++p) {
    if (c_begin + p < c_end) state_out_issue_loads(s, a, p, c_begin + p, h, kh, m0, n_pad, tid);
    cp_async_commit();
  }
  for (int ch = c_begin; ch < c_end; ++ch) {
    const int stage = (ch - c_begin) % SST;
    const int r0 = ch * GC;
    const int rows = min(GC, a.n - r0);
    if (ch + SST - 1 < c_end)
      state_out_issue_loads(s, a, (ch - c_begin + SST - 1) % SST, ch + SST - 1, h, kh, m0, n_pad, tid);
    cp_async_commit();
    cp_async_wait<SST - 1>();
    __syncthreads();
    // gates: every warp scans the chunk's log decays (lane l holds gam[2l] = ge, gam[2l + 1] = go)
    const float x0 = s.g[stage][2 * lane], x1 = s.g[stage][2 * lane + 1];
    const float pair = x0 + x1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float ge = incl - x1, go = incl;
    const float gl = __shfl_sync(0xffffffffu, incl, 31);
    const float f_even = __expf(gl - ge), f_odd = __expf(gl - go);
    const float e_even = __expf(ge), e_odd = __expf(go);
    // P rows mrow.. (all 64 columns): q k^T over dk, causal mask and decay, bf16 into s.p
    {
      float pa[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) pa[j][0] = pa[j][1] = pa[j][2] = pa[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t af[4];
        lda_row(af, s.q[stage], PK, mrow, ks * 16, lane);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_nk(bf, s.k[stage], PK, j2 * 16, ks * 16, lane);
          mma_bf16(pa[2 * j2], af, bf[0], bf[1]);
          mma_bf16(pa[2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
      const int ra = mrow + g, rb = ra + 8;
      const float gae = __shfl_sync(0xffffffffu, ge, ra >> 1), gao = __shfl_sync(0xffffffffu, go, ra >> 1);
      const float gbe = __shfl_sync(0xffffffffu, ge, rb >> 1), gbo = __shfl_sync(0xffffffffu, go, rb >> 1);
      const float gra = (ra & 1) ? gao : gae, grb = (rb & 1) ? gbo : gbe;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = (e >= 2) ? rb : ra;
          const int c = j * 8 + 2 * t + (e & 1);
          const float gc = __shfl_sync(0xffffffffu, (e & 1) ? go : ge, c >> 1);
          pa[j][e] = (r >= c) ? pa[j][e] * __expf(((e >= 2) ? grb : gra) - gc) : 0.f;
        }
        *reinterpret_cast<uint32_t*>(&s.p[ra * PQ + j * 8 + 2 * t]) = pack2(pa[j][0], pa[j][1]);
        *reinterpret_cast<uint32_t*>(&s.p[rb * PQ + j * 8 + 2 * t]) = pack2(pa[j][2], pa[j][3]);
      }
    }
    // S^T as bf16 A fragments (k = dk in steps of 16: n-tiles 2ks, 2ks + 1)
    uint32_t sa[8][4];
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
      sa[ks][0] = pack2(S[2 * ks][0], S[2 * ks][1]);
      sa[ks][1] = pack2(S[2 * ks][2], S[2 * ks][3]);
      sa[ks][2] = pack2(S[2 * ks + 1][0], S[2 * ks + 1][1]);
      sa[ks][3] = pack2(S[2 * ks + 1][2], S[2 * ks + 1][3]);
    }
    // O^T = S^T q^T [16 x 64 chunk rows], then column r times e^(gam_r)
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.q[stage], PK, j2 * 16, ks * 16, lane);   // B[k = dk][n = row] = q[row][dk]
        mma_bf16(o[2 * j2], sa[ks], bf[0], bf[1]);
        mma_bf16(o[2 * j2 + 1], sa[ks], bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + 2 * t;                      // chunk rows c, c + 1 (= lane (c >> 1)'s pair)
      const float s0 = __shfl_sync(0xffffffffu, e_even, c >> 1);
      const float s1 = __shfl_sync(0xffffffffu, e_odd, c >> 1);
      o[j][0] *= s0;
      o[j][1] *= s1;
      o[j][2] *= s0;
      o[j][3] *= s1;
    }
    // V'^T = U^T - S^T W^T: [16 x 64], n-tiles over chunk rows
    float vt[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) vt[j][0] = vt[j][1] = vt[j][2] = vt[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < 8; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.w[stage], PK, j2 * 16, ks * 16, lane);   // B[k = dk][n = row] = W[row][dk]
        mma_bf16(vt[2 * j2], sa[ks], bf[0], bf[1]);
        mma_bf16(vt[2 * j2 + 1], sa[ks], bf[2], bf[3]);
      }
    }
    const __nv_bfloat16* ut = s.ut[stage];
    uint32_t va[4][4], vu[4][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + 2 * t;
      const float2 u0 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[(mrow + g) * PU + c]));
      const float2 u1 = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&ut[(mrow + g + 8) * PU + c]));
      const float v0 = u0.x - vt[j][0], v1 = u0.y - vt[j][1], v2 = u1.x - vt[j][2], v3 = u1.y - vt[j][3];
      vu[j >> 1][(j & 1) ? 2 : 0] = pack2(v0, v1);
      vu[j >> 1][(j & 1) ? 3 : 1] = pack2(v2, v3);
      const float fc0 = __shfl_sync(0xffffffffu, f_even, c >> 1);
      const float fc1 = __shfl_sync(0xffffffffu, f_odd, c >> 1);
      va[j >> 1][(j & 1) ? 2 : 0] = pack2(v0 * fc0, v1 * fc1);
      va[j >> 1][(j & 1) ? 3 : 1] = pack2(v2 * fc0, v3 * fc1);
    }
    __syncthreads();   // every warp's P rows are in s.p
    // O^T += V'^T P^T (B[k = row'][n = row] = P[row][row'])
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.p, PQ, j2 * 16, kk * 16, lane);
        mma_bf16(o[2 * j2], vu[kk], bf[0], bf[1]);
        mma_bf16(o[2 * j2 + 1], vu[kk], bf[2], bf[3]);
      }
    }
    // O^T -> s.o[row][value dim]
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = j * 8 + 2 * t;
      const int m = mrow + g;
      s.o[c * PQ + m] = __float2bfloat16(o[j][0]);
      s.o[(c + 1) * PQ + m] = __float2bfloat16(o[j][1]);
      s.o[c * PQ + m + 8] = __float2bfloat16(o[j][2]);
      s.o[(c + 1) * PQ + m + 8] = __float2bfloat16(o[j][3]);
    }
    // S^T <- e^gl S^T + Vs^T k
    const float cd = __expf(gl);
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      S[nt][0] *= cd;
      S[nt][1] *= cd;
      S[nt][2] *= cd;
      S[nt][3] *= cd;
    }
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 8; ++j2) {
        uint32_t bf[4];
        ldb_kn(bf, s.k[stage], PK, j2 * 16, ks * 16, lane);   // B[k = row][n = dk] = k[row][dk]
        mma_bf16(S[2 * j2], va[ks], bf[0], bf[1]);
        mma_bf16(S[2 * j2 + 1], va[ks], bf[2], bf[3]);
      }
    }
    __syncthreads();   // s.o is complete; this stage and s.p are free again
    // output rows of the chunk, this CTA's 64 value dims: 8 x 16-byte segments per row
    for (int v = tid; v < GC * (SVS / 8); v += 128) {
      const int r = v / (SVS / 8), c = (v % (SVS / 8)) * 8;
      if (r < rows)
        *reinterpret_cast<uint4*>(a.out + (long)(r0 + r) * a.out_row + (long)h * a.dv + m0 + c) =
            *reinterpret_cast<const uint4*>(&s.o[r * PQ + c]);
    }
  }
  cp_async_wait<0>();
  if constexpr (MODE == 0) {
#pragma unroll
    for (int nt = 0; nt < 16; ++nt) {
      const int m = m0 + mrow + g;
      const int c = nt * 8 + 2 * t;
      state[(long)c * a.dv + m] = S[nt][0];
      state[(long)(c + 1) * a.dv + m] = S[nt][1];
      state[(long)c * a.dv + m + 8] = S[nt][2];
      state[(long)(c + 1) * a.dv + m + 8] = S[nt][3];
    }
  }
}

// ---------------------------------------------------------------------------------- output pass
// Parallel over (chunk, value head): O = (q e^gam) S_c + (q k^T * decay) V' for the chunk's rows, with
// S_c^T [dv][dk] and V'^T [dv][64] from the state pass read as [N][K] B operands.
struct OutSmem {
  __nv_bfloat16 q[GC * PK];
  __nv_bfloat16 k[GC * PK];
  __nv_bfloat16 vt[128 * PU];     // V'^T [dv][64]
  __nv_bfloat16 st[128 * PK];     // S_c^T [dv][dk]
  float gam[GC];
  float eg[GC];
};

__global__ void __launch_bounds__(128) gdn_output_kernel(GdnScanArgs a, int n_pad, const __nv_bfloat16* s_buf,
                                                         const __nv_bfloat16* vt_buf) {
  extern __shared__ __align__(16) uint8_t out_raw[];
  OutSmem& s = *reinterpret_cast<OutSmem*>(out_raw);
  const int chunk = blockIdx.x;
  const int h = blockIdx.y;
  const int kh = h / (a.nv / a.nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int r0 = chunk * GC;
  const int rows = min(GC, a.n - r0);
  const int dv = a.dv;
  const int n_chunks = n_pad / GC;
  const __nv_bfloat16* qp = a.q + ((long)kh * a.n + r0) * DK;
  const __nv_bfloat16* kp = a.k + ((long)kh * a.n + r0) * DK;
  const __nv_bfloat16* vp = vt_buf + ((long)h * n_chunks + chunk) * dv * GC;
  const __nv_bfloat16* sp = s_buf + ((long)h * n_chunks + chunk) * dv * DK;
  for (int v = tid; v < GC * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    const bool ok = r < rows;
    cp_async16(&s.q[r * PK + c], ok ? qp + (long)r * DK + c : qp, ok);
    cp_async16(&s.k[r * PK + c], ok ? kp + (long)r * DK + c : kp, ok);
  }
  for (int v = tid; v < dv * (GC / 8); v += 128) {
    const int r = v / (GC / 8), c = (v % (GC / 8)) * 8;
    cp_async16(&s.vt[r * PU + c], vp + (long)r * GC + c, true);
  }
  for (int v = tid; v < dv * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    cp_async16(&s.st[r * PK + c], sp + (long)r * DK + c, true);
  }
  cp_async_commit();
  if (warp == 0) {
    const float x0 = (2 * lane < rows) ? a.g[(long)h * a.n + r0 + 2 * lane] : 0.f;
    const float x1 = (2 * lane + 1 < rows) ? a.g[(long)h * a.n + r0 + 2 * lane + 1] : 0.f;
    const float pair = x0 + x1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    s.gam[2 * lane] = incl - pair + x0;
    s.gam[2 * lane + 1] = incl;
    s.eg[2 * lane] = __expf(incl - pair + x0);
    s.eg[2 * lane + 1] = __expf(incl);
  }
  cp_async_wait<0>();
  __syncthreads();
  const int ra = warp * 16 + g, rb = ra + 8;
  float qk[8][4];
#pragma unroll
  for (int j = 0; j < 8; ++j) qk[j][0] = qk[j][1] = qk[j][2] = qk[j][3] = 0.f;
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    uint32_t af[4];
    lda_row(af, s.q, PK, warp * 16, ks * 16, lane);
#pragma unroll
    for (int j2 = 0; j2 < 4; ++j2) {
      uint32_t bf[4];
      ldb_nk(bf, s.k, PK, j2 * 16, ks * 16, lane);
      mma_bf16(qk[2 * j2], af, bf[0], bf[1]);
      mma_bf16(qk[2 * j2 + 1], af, bf[2], bf[3]);
    }
  }
  const float ga = s.gam[ra], gb = s.gam[rb];
#pragma unroll
  for (int j = 0; j < 8; ++j)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int r = (e >= 2) ? rb : ra;
      const int c = j * 8 + 2 * t + (e & 1);
      qk[j][e] = (r >= c) ? qk[j][e] * __expf(((e >= 2) ? gb : ga) - s.gam[c]) : 0.f;
    }
  uint32_t pf[4][4];
#pragma unroll
  for (int kk = 0; kk < 4; ++kk) {
    pf[kk][0] = pack2(qk[2 * kk][0], qk[2 * kk][1]);
    pf[kk][1] = pack2(qk[2 * kk][2], qk[2 * kk][3]);
    pf[kk][2] = pack2(qk[2 * kk + 1][0], qk[2 * kk + 1][1]);
    pf[kk][3] = pack2(qk[2 * kk + 1][2], qk[2 * kk + 1][3]);
  }
  uint32_t qa[8][4];
  const float ea = s.eg[ra], eb = s.eg[rb];
#pragma unroll
  for (int ks = 0; ks < DK / 16; ++ks) {
    lda_row(qa[ks], s.q, PK, warp * 16, ks * 16, lane);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float sc = (e & 1) ? eb : ea;
      float2 f = __bfloat1622float2(*reinterpret_cast<__nv_bfloat162*>(&qa[ks][e]));
      qa[ks][e] = pack2(f.x * sc, f.y * sc);
    }
  }
  for (int nb = 0; nb < dv; nb += 64) {
    float o[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.st, PK, nb + j2 * 16, ks * 16, lane);   // B[k = dk][n = dv] = S^T[dv][dk]
        mma_bf16(o[2 * j2], qa[ks], bf[0], bf[1]);
        mma_bf16(o[2 * j2 + 1], qa[ks], bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int kk = 0; kk < 4; ++kk) {
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_nk(bf, s.vt, PU, nb + j2 * 16, kk * 16, lane);   // B[k = row][n = dv] = V'^T[dv][row]
        mma_bf16(o[2 * j2], pf[kk], bf[0], bf[1]);
        mma_bf16(o[2 * j2 + 1], pf[kk], bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int c = nb + j * 8 + 2 * t;
      if (ra < rows)
        *reinterpret_cast<uint32_t*>(a.out + (long)(r0 + ra) * a.out_row + (long)h * dv + c) = pack2(o[j][0], o[j][1]);
      if (rb < rows)
        *reinterpret_cast<uint32_t*>(a.out + (long)(r0 + rb) * a.out_row + (long)h * dv + c) = pack2(o[j][2], o[j][3]);
    }
  }
}

int gdn_fused_output = 1;

void gdn_chunk_scan(const GdnScanArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  // output mode on the fused state + output pass unless switched off or the output rows are not 16-byte aligned
  const bool fused = a.q != nullptr && gdn_fused_output && a.out != nullptr &&
                     reinterpret_cast<uintptr_t>(a.out) % 16 == 0 && a.out_row % 8 == 0;
  if (a.dk != DK || a.dv % SVS != 0 || a.dv > 128 || a.nv % a.nk != 0 ||
      (a.q != nullptr && !fused && (a.s_buf == nullptr || a.vt_buf == nullptr))) {
    record_error_async(a.err, kErrBadShape, stream);
    return;
  }
  const int n_chunks = (a.n + GC - 1) / GC;
  const int n_pad = n_chunks * GC;
  static PerDeviceOnce once;
  once([] {
    cudaFuncSetAttribute(gdn_wy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(WySmem));
    cudaFuncSetAttribute(gdn_state_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(StateSmem));
    cudaFuncSetAttribute(gdn_state_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(StateSmem));
    cudaFuncSetAttribute(gdn_state_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(StateSmem));
    cudaFuncSetAttribute(gdn_group_prop_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(PropSmem));
    cudaFuncSetAttribute(gdn_output_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(OutSmem));
    cudaFuncSetAttribute(gdn_state_out_kernel<0>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(StateOutSmem));
    cudaFuncSetAttribute(gdn_state_out_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                         (int)sizeof(StateOutSmem));
  });
  gdn_wy_kernel<<<dim3(n_chunks, a.nv), 128, sizeof(WySmem), stream>>>(a, n_pad);
  count_launch();
  const bool two_level = a.groups > 1 && a.dv == DK && a.grp_buf != nullptr &&
                         (a.q == nullptr || a.start_buf != nullptr) && n_chunks >= 2 * a.groups;
  if (!two_level) {
    if (fused) {
      if (!gdn_state_out_tc(a, n_pad, 0, stream))
        gdn_state_out_kernel<0><<<dim3(a.nv, a.dv / SVS), 128, sizeof(StateOutSmem), stream>>>(a, n_pad);
    } else
      gdn_state_kernel<0><<<dim3(a.nv, a.dv / SVS), 128, sizeof(StateSmem), stream>>>(a, n_pad, a.q ? a.s_buf : nullptr,
                                                                                    a.q ? a.vt_buf : nullptr);
    count_launch();
  } else {
    gdn_state_kernel<1><<<dim3(a.nv, 2 * a.dv / SVS, a.groups), 128, sizeof(StateSmem), stream>>>(a, n_pad, nullptr,
                                                                                               nullptr);
    gdn_group_prop_kernel<<<dim3(a.nv, a.dv / SVS), 128, sizeof(PropSmem), stream>>>(a, a.q != nullptr ? 1 : 0);
    count_launch(2);
    if (a.q != nullptr) {
      if (fused) {
        if (!gdn_state_out_tc(a, n_pad, 2, stream))
          gdn_state_out_kernel<2><<<dim3(a.nv, a.dv / SVS, a.groups), 128, sizeof(StateOutSmem), stream>>>(a, n_pad);
      } else
        gdn_state_kernel<2><<<dim3(a.nv, a.dv / SVS, a.groups), 128, sizeof(StateSmem), stream>>>(a, n_pad, a.s_buf,
                                                                                                a.vt_buf);
      count_launch();
    }
  }
  if (a.q != nullptr && !fused) {
    gdn_output_kernel<<<dim3(n_chunks, a.nv), 128, sizeof(OutSmem), stream>>>(a, n_pad, a.s_buf, a.vt_buf);
    count_launch();
  }
}

}  // namespace rf
