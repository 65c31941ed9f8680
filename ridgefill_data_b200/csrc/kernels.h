// Launchers of the non-GEMM sm_100a kernels (norms, RoPE, attention, Gated DeltaNet, ridge linear
// algebra, MoE routing, peer-memory collectives). Raw pointers + a stream; no torch types.
#pragma once
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <cstdint>

namespace rf {}  // namespace rf
