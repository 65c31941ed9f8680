// Python bindings of the sm_100a kernels (torch tensors -> raw pointers + the current stream).
#include <torch/extension.h>
#include <algorithm>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include "gemm.h"
#include "kernels.h"

// One int32 error word per device: kernels with bounded waits (and gather bounds checks) record a code here.
// Outside the anonymous namespace: bind_ops.cpp uses it too.
torch::Tensor& err_word(int dev) {
  static std::vector<torch::Tensor> words(64);
  if (!words[dev].defined())
    words[dev] = torch::zeros({1}, torch::dtype(torch::kInt32).device(torch::kCUDA, dev));
  return words[dev];
}

namespace {

#define CHECK_CUDA(x) TORCH_CHECK((x).is_cuda(), #x " must be a CUDA tensor")
#define CHECK_BF16(x) TORCH_CHECK((x).scalar_type() == at::kBFloat16, #x " must be bf16")

cudaStream_t stream() { return at::cuda::getCurrentCUDAStream().stream(); }


int* err_ptr(const torch::Tensor& like) { return err_word(like.get_device()).data_ptr<int>(); }

torch::Tensor error_word(int64_t dev) { return err_word((int)dev); }

// out = epilogue(A x B^T). A: [M, K] (a_mn: [K, M]); B: [N, K] (b_mn: [K, N]); leading stride of each
// operand may exceed its logical width (row pitch = stride(0)).
void gemm(torch::Tensor a, torch::Tensor b, torch::Tensor out, c10::optional<torch::Tensor> bias,
          c10::optional<torch::Tensor> residual, int64_t epi, int64_t bn, bool a_mn, bool b_mn, int64_t k_splits,
          int64_t k_chunk, int64_t max_ctas) {
  CHECK_CUDA(a); CHECK_CUDA(b); CHECK_CUDA(out);
  CHECK_BF16(a); CHECK_BF16(b);
  TORCH_CHECK(a.dim() == 2 && b.dim() == 2 && out.dim() == 2, "gemm: 2-D operands");
  TORCH_CHECK(a.stride(1) == 1 && b.stride(1) == 1 && out.stride(1) == 1, "gemm: unit inner stride");
  c10::cuda::CUDAGuard g(a.device());
  rf::GemmOperands op;
  op.A = a.data_ptr(); op.lda = a.stride(0); op.a_mn = a_mn;
  op.B = b.data_ptr(); op.ldb = b.stride(0); op.b_mn = b_mn;
  rf::GemmArgs args{};
  args.M = (int)(a_mn ? a.size(1) : a.size(0));
  args.K = (int)(a_mn ? a.size(0) : a.size(1));
  args.N = (int)(b_mn ? b.size(1) : b.size(0));
  TORCH_CHECK((b_mn ? b.size(0) : b.size(1)) == args.K, "gemm: K mismatch");
  args.k_splits = (int)k_splits;
  args.k_chunk = (int)k_chunk;
  args.out = out.data_ptr();
  args.ldo = out.stride(0);
  const int64_t out_cols = epi == rf::kEpiSwiGLU ? args.N / 2 : args.N;
  TORCH_CHECK(out.size(0) == args.M && out.size(1) == out_cols, "gemm: output shape");
  if (epi == rf::kEpiStore || epi == rf::kEpiSwiGLU) CHECK_BF16(out);
  if (epi == rf::kEpiF32) TORCH_CHECK(out.scalar_type() == at::kFloat, "gemm: fp32 output");
  if (epi == rf::kEpiF64Acc) TORCH_CHECK(out.scalar_type() == at::kDouble, "gemm: fp64 output");
  bool vec = (reinterpret_cast<uintptr_t>(args.out) % 16 == 0) && ((args.ldo * out.element_size()) % 16 == 0);
  if (bias.has_value()) {
    CHECK_BF16(*bias);
    TORCH_CHECK(bias->is_contiguous() && bias->numel() == args.N, "gemm: bias [N]");
    args.bias = reinterpret_cast<const __nv_bfloat16*>(bias->data_ptr());
  }
  if (residual.has_value()) {
    CHECK_BF16(*residual);
    TORCH_CHECK(residual->dim() == 2 && residual->stride(1) == 1 && residual->size(0) == args.M &&
                    residual->size(1) == args.N, "gemm: residual [M, N]");
    args.residual = reinterpret_cast<const __nv_bfloat16*>(residual->data_ptr());
    args.ldr = residual->stride(0);
    vec = vec && (reinterpret_cast<uintptr_t>(args.residual) % 16 == 0) && ((args.ldr * 2) % 16 == 0);
  }
  args.vec_ok = vec ? 1 : 0;
  args.err = err_ptr(a);
  rf::gemm_bf16(op, args, (int)epi, (int)bn, (int)max_ctas, stream());
  C10_CUDA_KERNEL_LAUNCH_CHECK();
}

int64_t sm_count(int64_t dev) { return rf::num_sms((int)dev); }
int64_t launch_count() { return rf::launch_counter().load(); }

// Whether 256-column store / SwiGLU products run on the two-SM kernel (gemm2sm.cu); returns the previous setting.
bool set_gemm_2sm(bool on) {
  const bool was = rf::gemm_2sm_enabled;
  rf::gemm_2sm_enabled = on;
  return was;
}

}  // namespace

void register_ops(pybind11::module_& m);   // bind_ops.cpp

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "ridgefill_data_b200 sm_100a kernels";
  m.def("error_word", &error_word);
  m.def("sm_count", &sm_count);
  m.def("launch_count", &launch_count);
  m.def("set_gemv", [](bool on) {
    const bool was = rf::gemv_enabled;
    rf::gemv_enabled = on;
    return was;
  });
  m.def("set_gemv_max_rows", [](int64_t n) {
    const int was = rf::gemv_max_rows;
    rf::gemv_max_rows = (int)std::max<int64_t>(0, std::min<int64_t>(16, n));
    return was;
  });
  m.def("set_gemv_mma", [](bool on) {
    const bool was = rf::gemv_mma;
    rf::gemv_mma = on;
    return was;
  });
  m.def("set_gemm_2sm", &set_gemm_2sm);
  m.def("set_attn_poly", [](int64_t n) {
    const int was = rf::attn_poly;
    rf::attn_poly = (n == 2 || n == 4) ? (int)n : 0;
    return was;
  });
  m.def("set_gdn_fused_output", [](int64_t n) {
    const int was = rf::gdn_fused_output;
    rf::gdn_fused_output = n ? 1 : 0;
    return was;
  });
  m.def("gdn_fused_output", []() { return rf::gdn_fused_output; });
  // phase trace of the tcgen05 GDN state pass: an int64 CUDA tensor of >= 128 * 16 stamps, or None
  m.def("set_gdn_tc_trace", [](c10::optional<at::Tensor> t) {
    rf::gdn_tc_trace = t.has_value() ? reinterpret_cast<unsigned long long*>(t->data_ptr<int64_t>()) : nullptr;
  });
  m.def("set_gdn_state_tc", [](int64_t n) {
    const int was = rf::gdn_state_tc;
    rf::gdn_state_tc = n ? 1 : 0;
    return was;
  });
  m.def("set_attn_softmax_groups", [](int64_t n) {
    const int was = rf::attn_softmax_groups;
    rf::attn_softmax_groups = n == 2 ? 2 : 1;
    return was;
  });
  m.def("set_attn_q_tmem", [](int64_t n) {
    const int was = rf::attn_q_tmem;
    rf::attn_q_tmem = n ? 1 : 0;
    return was;
  });
  m.def("set_attn_rotate", [](int64_t n) {
    const int was = rf::attn_rotate;
    rf::attn_rotate = n ? 1 : 0;
    return was;
  });
  m.def("set_attn_s_buffers", [](int64_t n) {
    const int was = rf::attn_s_buffers;
    rf::attn_s_buffers = (n == 2 || n == 3) ? (int)n : 0;
    return was;
  });
  m.def("set_attn_p_buffers", [](int64_t n) {
    const int was = rf::attn_p_buffers;
    rf::attn_p_buffers = n == 1 ? 1 : 2;
    return was;
  });
  m.def("gemm", &gemm, py::arg("a"), py::arg("b"), py::arg("out"), py::arg("bias") = py::none(),
        py::arg("residual") = py::none(), py::arg("epi") = 0, py::arg("bn") = 256, py::arg("a_mn") = false,
        py::arg("b_mn") = false, py::arg("k_splits") = 1, py::arg("k_chunk") = 0, py::arg("max_ctas") = 0);
  register_ops(m);
}
