// Vocabulary reductions over logits rows (the scorer: teacher-forced log-probs, top-1 and KL between two arms).
//
//  score_rows   one CTA per row of fp32 logits [rows][V]: the row max and first argmax (ties to the lower index),
//               the log-sum-exp accumulated in fp64 (max + log sum exp(x - max)), the target's log-probability
//               x[t] - lse, and with a reference row q (the exact arm's logits) KL(q || p) = sum softmax(q) (log
//               softmax(q) - log softmax(p)) in fp64. The reference computes the same quantities with torch
//               log_softmax over the vocabulary (code/kva/kva.py:463-467, code/kva/agree.py:59-62) and its native
//               scorer with an fp64 log-softmax on the host (code/qwen38-27b-kit/exact_score.cpp:13-65).
// Three passes over the row (max, sums, KL); a row of 248,320 fp32 logits is ~1 MB, read from L2 after pass 1.
#include "kernels.h"
#include "ptx.cuh"

namespace rf {

constexpr int kScoreThreads = 512;

template <typename T>
__device__ __forceinline__ T warp_sum(T v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

// block-wide (max, argmax) with ties to the lower index
__device__ void block_argmax(float& v, int& idx, float* sv, int* si) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, v, o);
    const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
    if (ov > v || (ov == v && oi < idx)) {
      v = ov;
      idx = oi;
    }
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) {
    sv[warp] = v;
    si[warp] = idx;
  }
  __syncthreads();
  if (warp == 0) {
    v = lane < kScoreThreads / 32 ? sv[lane] : -INFINITY;
    idx = lane < kScoreThreads / 32 ? si[lane] : 0x7fffffff;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, v, o);
      const int oi = __shfl_xor_sync(0xffffffffu, idx, o);
      if (ov > v || (ov == v && oi < idx)) {
        v = ov;
        idx = oi;
      }
    }
    if (lane == 0) {
      sv[0] = v;
      si[0] = idx;
    }
  }
  __syncthreads();
  v = sv[0];
  idx = si[0];
  __syncthreads();
}

__device__ double block_sum(double v, double* sd) {
  v = warp_sum(v);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sd[warp] = v;
  __syncthreads();
  if (warp == 0) {
    v = lane < kScoreThreads / 32 ? sd[lane] : 0.0;
    v = warp_sum(v);
    if (lane == 0) sd[0] = v;
  }
  __syncthreads();
  v = sd[0];
  __syncthreads();
  return v;
}

__global__ void __launch_bounds__(kScoreThreads) score_rows_kernel(ScoreArgs a) {
  __shared__ float sv[kScoreThreads / 32];
  __shared__ int si[kScoreThreads / 32];
  __shared__ double sd[kScoreThreads / 32];
  const long r = blockIdx.x;
  const float* x = a.logits + r * a.ld;
  const float* q = a.ref != nullptr ? a.ref + r * a.ld_ref : nullptr;

  float mx = -INFINITY, mq = -INFINITY;
  int ix = 0x7fffffff, iq = 0x7fffffff;
  for (int j = threadIdx.x; j < a.V; j += kScoreThreads) {
    const float v = x[j];
    if (v > mx) {
      mx = v;
      ix = j;
    }
    if (q != nullptr) {
      const float u = q[j];
      if (u > mq) {
        mq = u;
        iq = j;
      }
    }
  }
  block_argmax(mx, ix, sv, si);
  if (q != nullptr) block_argmax(mq, iq, sv, si);

  double sx = 0.0, sq = 0.0;
  for (int j = threadIdx.x; j < a.V; j += kScoreThreads) {
    sx += exp((double)x[j] - (double)mx);
    if (q != nullptr) sq += exp((double)q[j] - (double)mq);
  }
  sx = block_sum(sx, sd);
  const double lse_x = (double)mx + log(sx);
  double lse_q = 0.0;
  if (q != nullptr) {
    sq = block_sum(sq, sd);
    lse_q = (double)mq + log(sq);
  }
  if (q != nullptr && a.kl != nullptr) {
    double acc = 0.0;
    for (int j = threadIdx.x; j < a.V; j += kScoreThreads) {
      const double lq = (double)q[j] - lse_q;
      acc += exp(lq) * (lq - ((double)x[j] - lse_x));
    }
    acc = block_sum(acc, sd);
    if (threadIdx.x == 0) a.kl[r] = acc;
  }
  if (threadIdx.x == 0) {
    if (a.lse != nullptr) a.lse[r] = lse_x;
    if (a.argmax != nullptr) a.argmax[r] = ix;
    if (a.ref_argmax != nullptr && q != nullptr) a.ref_argmax[r] = iq;
    if (a.targets != nullptr && a.logprob != nullptr) {
      const long t = a.targets[r];
      a.logprob[r] = (t >= 0 && t < a.V) ? (double)x[t] - lse_x : NAN;
    }
  }
}

void score_rows(const ScoreArgs& a, cudaStream_t stream) {
  if (a.rows <= 0) return;
  score_rows_kernel<<<a.rows, kScoreThreads, 0, stream>>>(a);
  count_launch();
}

}  // namespace rf
