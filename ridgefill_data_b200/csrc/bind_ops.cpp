// Python bindings of the non-GEMM kernels (kernels.h).
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "kernels.h"

void register_ops(pybind11::module_& m) { (void)m; }
