// Native identity check of the ridge-map fill GEMM (the role of code/qwen38-27b-kit/identity_native.cpp:9-43):
// with W = I and c = 0, x = h W^T + c must reproduce h bit for bit (bf16), for both N-tile widths, with the bias
// epilogue and without it, on ragged shapes. A standalone program: no Python, no torch, links only the GEMM
// translation unit and the CUDA runtime / driver.
//
//   identity_check [rows] [dim]      exit 0 and one JSON line when every case is bitwise exact
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <vector>

#include "../gemm.h"

#define CHECK(x)                                                                   \
  do {                                                                             \
    cudaError_t e_ = (x);                                                          \
    if (e_ != cudaSuccess) {                                                       \
      std::fprintf(stderr, "%s:%d %s\n", __FILE__, __LINE__, cudaGetErrorString(e_)); \
      std::exit(2);                                                                \
    }                                                                              \
  } while (0)

static uint16_t bits(__nv_bfloat16 v) {
  uint16_t u;
  std::memcpy(&u, &v, 2);
  return u;
}

int main(int argc, char** argv) {
  const int rows = argc > 1 ? std::atoi(argv[1]) : 777;
  const int dim = argc > 2 ? std::atoi(argv[2]) : 1024;
  std::vector<__nv_bfloat16> h(size_t(rows) * dim), eye(size_t(dim) * dim), zero(dim);
  uint32_t s = 12345u;
  for (auto& v : h) {
    s = s * 1664525u + 1013904223u;
    // values across many binades, both signs, including exact zeros
    const int e = int((s >> 8) % 24) - 12;
    const float m = 1.0f + float((s >> 16) & 0x7f) / 128.0f;
    v = __float2bfloat16(((s & 1u) ? -1.0f : 1.0f) * ((s >> 20) % 97 == 0 ? 0.0f : std::ldexp(m, e)));
  }
  for (int i = 0; i < dim; ++i) {
    for (int j = 0; j < dim; ++j) eye[size_t(i) * dim + j] = __float2bfloat16(i == j ? 1.0f : 0.0f);
    zero[i] = __float2bfloat16(0.0f);
  }
  __nv_bfloat16 *dh, *dw, *dz, *dx;
  int* derr;
  CHECK(cudaMalloc(&dh, h.size() * 2));
  CHECK(cudaMalloc(&dw, eye.size() * 2));
  CHECK(cudaMalloc(&dz, zero.size() * 2));
  CHECK(cudaMalloc(&dx, h.size() * 2));
  CHECK(cudaMalloc(&derr, sizeof(int)));
  CHECK(cudaMemcpy(dh, h.data(), h.size() * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(dw, eye.data(), eye.size() * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemcpy(dz, zero.data(), zero.size() * 2, cudaMemcpyHostToDevice));
  CHECK(cudaMemset(derr, 0, sizeof(int)));
  std::vector<__nv_bfloat16> got(h.size());
  long bad_total = 0;
  int cases = 0;
  for (int bn : {256, 128}) {
    for (int with_bias : {0, 1}) {
      CHECK(cudaMemset(dx, 0xff, h.size() * 2));
      rf::GemmOperands op{dh, dim, false, dw, dim, false};
      rf::GemmArgs a{};
      a.M = rows;
      a.N = dim;
      a.K = dim;
      a.k_splits = 1;
      a.k_chunk = dim;
      a.out = dx;
      a.ldo = dim;
      a.bias = with_bias ? dz : nullptr;
      a.vec_ok = dim % 8 == 0;
      a.err = derr;
      rf::gemm_bf16(op, a, rf::kEpiStore, bn, 0, 0);
      CHECK(cudaGetLastError());
      CHECK(cudaDeviceSynchronize());
      CHECK(cudaMemcpy(got.data(), dx, got.size() * 2, cudaMemcpyDeviceToHost));
      long bad = 0;
      for (size_t i = 0; i < got.size(); ++i) {
        // -0 * 1 + 0 sums to +0 in the fp32 accumulator: compare zeros by value, everything else by bits
        const bool both_zero = (bits(got[i]) & 0x7fff) == 0 && (bits(h[i]) & 0x7fff) == 0;
        bad += !(both_zero || bits(got[i]) == bits(h[i]));
      }
      if (bad) std::fprintf(stderr, "bn %d bias %d: %ld of %zu values differ\n", bn, with_bias, bad, got.size());
      bad_total += bad;
      ++cases;
    }
  }
  int err = 0;
  CHECK(cudaMemcpy(&err, derr, sizeof(int), cudaMemcpyDeviceToHost));
  std::printf("{\"check\": \"identity_fill\", \"rows\": %d, \"dim\": %d, \"cases\": %d, \"mismatches\": %ld, "
              "\"error_word\": %d}\n", rows, dim, cases, bad_total, err);
  return (bad_total == 0 && err == 0) ? 0 : 1;
}
