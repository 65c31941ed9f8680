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
//                    The fp32 state lives in mma accumulators for the whole sequence; its bf16 copy in shared
//                    memory feeds the products. Fill mode (q == nullptr) skips the output.
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
// grid: n tokens; block 256 threads (8 warps) loop over head tasks: [0, nk) q heads, [nk, 2nk) k heads,
// [2nk, 2nk + nv) v heads.
__global__ void __launch_bounds__(256) gdn_prep_kernel(GdnPrepArgs a) {
  const int tkn = blockIdx.x;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int C = 2 * a.nk * a.dk + a.nv * a.dv;
  const int tasks = 2 * a.nk + a.nv;
  const __nv_bfloat16* prow = a.proj + (long)tkn * a.proj_row;
  for (int task = warp; task < tasks; task += 8) {
    int c0, dh;
    if (task < 2 * a.nk) {
      c0 = task * a.dk;
      dh = a.dk;
    } else {
      c0 = 2 * a.nk * a.dk + (task - 2 * a.nk) * a.dv;
      dh = a.dv;
    }
    const int per = dh / 32;
    float val[8];
    float ss = 0.f;
    for (int j = 0; j < per; ++j) {
      const int c = c0 + lane * per + j;
      float acc = 0.f;
      for (int tap = 0; tap < a.K; ++tap) {
        const int r = tkn - (a.K - 1) + tap;   // source row (negative: conv state)
        float x;
        if (r >= 0)
          x = __bfloat162float(a.proj[(long)r * a.proj_row + c]);
        else
          x = a.conv_state != nullptr ? __bfloat162float(a.conv_state[(long)(a.K - 1 + r) * C + c]) : 0.f;
        acc += x * __bfloat162float(a.conv_w[(long)c * a.K + tap]);
      }
      const float y = bf16r(acc / (1.f + expf(-acc)));
      val[j] = y;
      ss += y * y;
    }
    if (task < 2 * a.nk) {
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
      float inv = rsqrtf(ss + 1e-6f);
      const bool is_q = task < a.nk;
      if (is_q) inv *= rsqrtf((float)a.dk);
      const int hh = is_q ? task : task - a.nk;
      __nv_bfloat16* dst = (is_q ? a.q : a.k) + ((long)hh * a.n + tkn) * a.dk;
      for (int j = 0; j < per; ++j) dst[lane * per + j] = __float2bfloat16(val[j] * inv);
    } else {
      const int hh = task - 2 * a.nk;
      __nv_bfloat16* dst = a.v + ((long)hh * a.n + tkn) * a.dv;
      for (int j = 0; j < per; ++j) dst[lane * per + j] = __float2bfloat16(val[j]);
    }
  }
  for (int h = threadIdx.x; h < a.nv; h += blockDim.x) {
    const float b = __bfloat162float(prow[a.b_off + h]);
    const float av = __bfloat162float(prow[a.a_off + h]);
    a.beta[(long)h * a.n + tkn] = bf16r(1.f / (1.f + expf(-b)));
    a.g[(long)h * a.n + tkn] = -expf(a.A_log[h]) * softplus_f(av + a.dt_bias[h]);
  }
}

void gdn_prep(const GdnPrepArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  gdn_prep_kernel<<<a.n, 256, 0, stream>>>(a); count_launch();
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

struct WySmem {
  __nv_bfloat16 k[GC * PK];
  __nv_bfloat16 kb[GC * PK];
  __nv_bfloat16 vb[GC * PK];      // dv <= 128
  __nv_bfloat16 t16[GC * (GC + 8)];
  float A[GC * (GC + 1)];
  float gam[GC];
  float beta[GC];
};

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

  // loads
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
    cp_async16(&s.vb[r * PK + c], ok ? vp + (long)r * dv + c : vp, ok);
  }
  cp_async_commit();
  if (tid < GC) {
    const bool ok = tid < rows;
    s.beta[tid] = ok ? a.beta[(long)h * a.n + r0 + tid] : 0.f;
    s.gam[tid] = ok ? a.g[(long)h * a.n + r0 + tid] : 0.f;
  }
  __syncthreads();
  if (warp == 0) {  // inclusive cumsum of 64 values, 2 per lane
    float x0 = s.gam[2 * lane], x1 = s.gam[2 * lane + 1];
    float pair = x0 + x1;
    float incl = pair;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const float y = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += y;
    }
    const float excl = incl - pair;
    s.gam[2 * lane] = excl + x0;
    s.gam[2 * lane + 1] = incl;
  }
  cp_async_wait<0>();
  __syncthreads();

  // KK^T (16 rows per warp) -> A = strictly lower, beta_i * kk * exp(gam_i - gam_j)
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
#pragma unroll
    for (int j = 0; j < 8; ++j) {
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 16 + g + (e >= 2 ? 8 : 0);
        const int c = j * 8 + 2 * t + (e & 1);
        const float v = (r > c) ? s.beta[r] * acc[j][e] * expf(s.gam[r] - s.gam[c]) : 0.f;
        s.A[r * (GC + 1) + c] = v;
      }
    }
  }
  // scaled operands: kb = beta e^gam k, vb = beta v (in place over the loaded v)
  for (int v = tid; v < GC * DK; v += 128) {
    const int r = v / DK, c = v % DK;
    s.kb[r * PK + c] = __float2bfloat16(s.beta[r] * expf(s.gam[r]) * __bfloat162float(s.k[r * PK + c]));
  }
  for (int v = tid; v < GC * dv; v += 128) {
    const int r = v / dv, c = v % dv;
    s.vb[r * PK + c] = __float2bfloat16(s.beta[r] * __bfloat162float(s.vb[r * PK + c]));
  }
  __syncthreads();
  // T = (I + A)^-1, column c by thread c: T[i][c] = [i == c] - sum_{c <= j < i} A[i][j] T[j][c]
  if (tid < GC) {
    const int c = tid;
    float col[GC];
#pragma unroll
    for (int i = 0; i < GC; ++i) col[i] = 0.f;
#pragma unroll
    for (int i = 0; i < GC; ++i) {
      if (i < c) continue;
      float v = (i == c) ? 1.f : 0.f;
#pragma unroll
      for (int j = 0; j < i; ++j)
        if (j >= c) v -= s.A[i * (GC + 1) + j] * col[j];
      col[i] = v;
    }
#pragma unroll
    for (int i = 0; i < GC; ++i) s.t16[i * (GC + 8) + c] = __float2bfloat16(col[i]);
  }
  __syncthreads();
  // W = T kb [64 x dk], U = T vb [64 x dv]
  __nv_bfloat16* wdst = a.w_buf + ((long)h * n_pad + r0) * DK;
  __nv_bfloat16* udst = a.u_buf + ((long)h * n_pad + r0) * dv;
#pragma unroll
  for (int which = 0; which < 2; ++which) {
    const __nv_bfloat16* B = which == 0 ? s.kb : s.vb;
    const int ncols = which == 0 ? DK : dv;
    __nv_bfloat16* dst = which == 0 ? wdst : udst;
    for (int nb = 0; nb < ncols; nb += 64) {
      float acc[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) acc[j][0] = acc[j][1] = acc[j][2] = acc[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < GC / 16; ++ks) {
        uint32_t af[4];
        lda_row(af, s.t16, GC + 8, warp * 16, ks * 16, lane);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_kn(bf, B, PK, nb + j2 * 16, ks * 16, lane);
          mma_bf16(acc[2 * j2], af, bf[0], bf[1]);
          mma_bf16(acc[2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int r = warp * 16 + g;
        const int c = nb + j * 8 + 2 * t;
        *reinterpret_cast<uint32_t*>(dst + (long)r * ncols + c) = pack2(acc[j][0], acc[j][1]);
        *reinterpret_cast<uint32_t*>(dst + (long)(r + 8) * ncols + c) = pack2(acc[j][2], acc[j][3]);
      }
    }
  }
}

// ---------------------------------------------------------------------------------- scan kernel
constexpr int DVS = 64;           // state columns per CTA
constexpr int PV = DVS + 8;

struct ScanSmem {
  __nv_bfloat16 w[2][GC * PK];
  __nv_bfloat16 k[2][GC * PK];
  __nv_bfloat16 q[2][GC * PK];
  __nv_bfloat16 u[2][GC * PV];
  __nv_bfloat16 vn[GC * PV];
  __nv_bfloat16 kd[GC * PK];
  __nv_bfloat16 st[DK * PV];
  float gam[2][GC];
};

__device__ __forceinline__ void scan_issue_loads(ScanSmem& s, const GdnScanArgs& a, int buf, int chunk, int h, int kh,
                                                 int col0, int n_pad, int tid) {
  const int r0 = chunk * GC;
  const int rows = min(GC, a.n - r0);
  const __nv_bfloat16* wp = a.w_buf + ((long)h * n_pad + r0) * DK;
  const __nv_bfloat16* up = a.u_buf + ((long)h * n_pad + r0) * a.dv + col0;
  const __nv_bfloat16* kp = a.k + ((long)kh * a.n + r0) * DK;
  const __nv_bfloat16* qp = a.q != nullptr ? a.q + ((long)kh * a.n + r0) * DK : nullptr;
  for (int v = tid; v < GC * (DK / 8); v += 128) {
    const int r = v / (DK / 8), c = (v % (DK / 8)) * 8;
    cp_async16(&s.w[buf][r * PK + c], wp + (long)r * DK + c, true);   // padded rows hold zeros
    const bool ok = r < rows;
    cp_async16(&s.k[buf][r * PK + c], ok ? kp + (long)r * DK + c : kp, ok);
    if (qp != nullptr) cp_async16(&s.q[buf][r * PK + c], ok ? qp + (long)r * DK + c : qp, ok);
  }
  for (int v = tid; v < GC * (DVS / 8); v += 128) {
    const int r = v / (DVS / 8), c = (v % (DVS / 8)) * 8;
    cp_async16(&s.u[buf][r * PV + c], up + (long)r * a.dv + c, true);
  }
  cp_async_commit();
}

__global__ void __launch_bounds__(128, 1) gdn_scan_kernel(GdnScanArgs a, int n_pad) {
  extern __shared__ __align__(16) uint8_t scan_raw[];
  ScanSmem& s = *reinterpret_cast<ScanSmem*>(scan_raw);
  const int h = blockIdx.x;
  const int col0 = blockIdx.y * DVS;
  const int kh = h / (a.nv / a.nk);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, t = lane & 3;
  const int n_chunks = (a.n + GC - 1) / GC;
  const bool out_mode = a.q != nullptr;
  float* state = a.state + (long)h * DK * a.dv;

  // state accumulators: warp rows [32w, 32w+32) (2 m-tiles) x 64 cols (8 n-tiles)
  float S[2][8][4];
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + g + (e >= 2 ? 8 : 0);
        const int c = nt * 8 + 2 * t + (e & 1);
        S[mt][nt][e] = state[(long)r * a.dv + col0 + c];
      }

  if (n_chunks > 0) scan_issue_loads(s, a, 0, 0, h, kh, col0, n_pad, tid);
  for (int ch = 0; ch < n_chunks; ++ch) {
    const int buf = ch & 1;
    const int r0 = ch * GC;
    const int rows = min(GC, a.n - r0);
    // bf16 state copy + gamma of this chunk
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt) {
        const int r = warp * 32 + mt * 16 + g;
        const int c = nt * 8 + 2 * t;
        *reinterpret_cast<uint32_t*>(&s.st[r * PV + c]) = pack2(S[mt][nt][0], S[mt][nt][1]);
        *reinterpret_cast<uint32_t*>(&s.st[(r + 8) * PV + c]) = pack2(S[mt][nt][2], S[mt][nt][3]);
      }
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
      s.gam[buf][2 * lane] = incl - pair + x0;
      s.gam[buf][2 * lane + 1] = incl;
    }
    if (ch + 1 < n_chunks) scan_issue_loads(s, a, buf ^ 1, ch + 1, h, kh, col0, n_pad, tid);
    else cp_async_commit();
    cp_async_wait<1>();
    __syncthreads();
    const float* gam = s.gam[buf];
    const float gl = gam[GC - 1];

    // V' = U - W S  (warp rows [16w, 16w + 16) x 64)
    float vn[8][4];
#pragma unroll
    for (int j = 0; j < 8; ++j) vn[j][0] = vn[j][1] = vn[j][2] = vn[j][3] = 0.f;
#pragma unroll
    for (int ks = 0; ks < DK / 16; ++ks) {
      uint32_t af[4];
      lda_row(af, s.w[buf], PK, warp * 16, ks * 16, lane);
#pragma unroll
      for (int j2 = 0; j2 < 4; ++j2) {
        uint32_t bf[4];
        ldb_kn(bf, s.st, PV, j2 * 16, ks * 16, lane);
        mma_bf16(vn[2 * j2], af, bf[0], bf[1]);
        mma_bf16(vn[2 * j2 + 1], af, bf[2], bf[3]);
      }
    }
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int r = warp * 16 + g;
      const int c = j * 8 + 2 * t;
      const __nv_bfloat16* ur = s.u[buf];
      const float u0 = __bfloat162float(ur[r * PV + c]), u1 = __bfloat162float(ur[r * PV + c + 1]);
      const float u2 = __bfloat162float(ur[(r + 8) * PV + c]), u3 = __bfloat162float(ur[(r + 8) * PV + c + 1]);
      *reinterpret_cast<uint32_t*>(&s.vn[r * PV + c]) = pack2(u0 - vn[j][0], u1 - vn[j][1]);
      *reinterpret_cast<uint32_t*>(&s.vn[(r + 8) * PV + c]) = pack2(u2 - vn[j][2], u3 - vn[j][3]);
    }
    // Kd = k e^(gl - gam) (bf16)
    for (int v = tid; v < GC * DK; v += 128) {
      const int r = v / DK, c = v % DK;
      s.kd[r * PK + c] = __float2bfloat16(__bfloat162float(s.k[buf][r * PK + c]) * expf(gl - gam[r]));
    }
    __syncthreads();

    if (out_mode) {
      // O = (q e^gam) S + (q k^T * decay) V'
      float o[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
      const int ra = warp * 16 + g, rb = ra + 8;
      const float ea = expf(gam[ra]), eb = expf(gam[rb]);
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t af[4];
        lda_row(af, s.q[buf], PK, warp * 16, ks * 16, lane);
        // scale rows: a0, a2 -> row ra; a1, a3 -> row rb
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          __nv_bfloat162 p = *reinterpret_cast<__nv_bfloat162*>(&af[e]);
          const float sc = (e & 1) ? eb : ea;
          float2 f = __bfloat1622float2(p);
          af[e] = pack2(f.x * sc, f.y * sc);
        }
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_kn(bf, s.st, PV, j2 * 16, ks * 16, lane);
          mma_bf16(o[2 * j2], af, bf[0], bf[1]);
          mma_bf16(o[2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
      float qk[8][4];
#pragma unroll
      for (int j = 0; j < 8; ++j) qk[j][0] = qk[j][1] = qk[j][2] = qk[j][3] = 0.f;
#pragma unroll
      for (int ks = 0; ks < DK / 16; ++ks) {
        uint32_t af[4];
        lda_row(af, s.q[buf], PK, warp * 16, ks * 16, lane);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_nk(bf, s.k[buf], PK, j2 * 16, ks * 16, lane);
          mma_bf16(qk[2 * j2], af, bf[0], bf[1]);
          mma_bf16(qk[2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int r = (e >= 2) ? rb : ra;
          const int c = j * 8 + 2 * t + (e & 1);
          qk[j][e] = (r >= c) ? qk[j][e] * expf(gam[r] - gam[c]) : 0.f;
        }
      }
#pragma unroll
      for (int kk = 0; kk < 4; ++kk) {
        uint32_t pf[4];
        pf[0] = pack2(qk[2 * kk][0], qk[2 * kk][1]);
        pf[1] = pack2(qk[2 * kk][2], qk[2 * kk][3]);
        pf[2] = pack2(qk[2 * kk + 1][0], qk[2 * kk + 1][1]);
        pf[3] = pack2(qk[2 * kk + 1][2], qk[2 * kk + 1][3]);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_kn(bf, s.vn, PV, j2 * 16, kk * 16, lane);
          mma_bf16(o[2 * j2], pf, bf[0], bf[1]);
          mma_bf16(o[2 * j2 + 1], pf, bf[2], bf[3]);
        }
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const int c = col0 + j * 8 + 2 * t;
        if (ra < rows)
          *reinterpret_cast<uint32_t*>(a.out + (long)(r0 + ra) * a.out_row + (long)h * a.dv + c) =
              pack2(o[j][0], o[j][1]);
        if (rb < rows)
          *reinterpret_cast<uint32_t*>(a.out + (long)(r0 + rb) * a.out_row + (long)h * a.dv + c) =
              pack2(o[j][2], o[j][3]);
      }
    }

    // S <- e^gl S + Kd^T V'
    const float cd = expf(gl);
#pragma unroll
    for (int mt = 0; mt < 2; ++mt)
#pragma unroll
      for (int nt = 0; nt < 8; ++nt)
#pragma unroll
        for (int e = 0; e < 4; ++e) S[mt][nt][e] *= cd;
#pragma unroll
    for (int ks = 0; ks < GC / 16; ++ks) {
#pragma unroll
      for (int mt = 0; mt < 2; ++mt) {
        uint32_t af[4];
        lda_trans(af, s.kd, PK, warp * 32 + mt * 16, ks * 16, lane);
#pragma unroll
        for (int j2 = 0; j2 < 4; ++j2) {
          uint32_t bf[4];
          ldb_kn(bf, s.vn, PV, j2 * 16, ks * 16, lane);
          mma_bf16(S[mt][2 * j2], af, bf[0], bf[1]);
          mma_bf16(S[mt][2 * j2 + 1], af, bf[2], bf[3]);
        }
      }
    }
    __syncthreads();
  }
  cp_async_wait<0>();
#pragma unroll
  for (int mt = 0; mt < 2; ++mt)
#pragma unroll
    for (int nt = 0; nt < 8; ++nt)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int r = warp * 32 + mt * 16 + g + (e >= 2 ? 8 : 0);
        const int c = nt * 8 + 2 * t + (e & 1);
        state[(long)r * a.dv + col0 + c] = S[mt][nt][e];
      }
}

void gdn_chunk_scan(const GdnScanArgs& a, cudaStream_t stream) {
  if (a.n <= 0) return;
  if (a.dk != DK || a.dv % DVS != 0 || a.dv > 128 || a.nv % a.nk != 0) {
    if (a.err) cudaMemsetAsync(a.err, kErrBadShape, 1, stream);
    return;
  }
  const int n_chunks = (a.n + GC - 1) / GC;
  const int n_pad = n_chunks * GC;
  static bool set = false;
  if (!set) {
    cudaFuncSetAttribute(gdn_wy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(WySmem));
    cudaFuncSetAttribute(gdn_scan_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(ScanSmem));
    set = true;
  }
  gdn_wy_kernel<<<dim3(n_chunks, a.nv), 128, sizeof(WySmem), stream>>>(a, n_pad); count_launch();
  gdn_scan_kernel<<<dim3(a.nv, a.dv / DVS), 128, sizeof(ScanSmem), stream>>>(a, n_pad); count_launch();
}

}  // namespace rf
