// rmsnorm: PyTorch extension module with the Python-facing API of the upstream
// Tools/rmsnorm extension (rmsnorm.cu:123-143):
//   forward(input, weight, eps, residual=None) -> [out, rms]
// The kernel and its C ABI live in libqwen_b200.so (include/qwen_b200_ops.h);
// this file only checks tensors and allocates the outputs, as upstream's
// wrapper does.  fp16 only.  `backward` (training) is not part of this build
// and raises.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <optional>
#include <vector>

#include "qwen_b200.h"
#include "qwen_b200_ops.h"

namespace {

void check_half_cuda(const torch::Tensor &t, const char *name) {
  TORCH_CHECK(t.defined() && t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.scalar_type() == torch::kHalf, name, " must be float16 (this build is fp16 only), got ",
              t.scalar_type());
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

std::vector<torch::Tensor> forward(torch::Tensor input, torch::Tensor weight, double eps,
                                   std::optional<torch::Tensor> residual) {
  check_half_cuda(input, "input");
  check_half_cuda(weight, "weight");
  TORCH_CHECK(input.dim() >= 1 && input.size(-1) > 0, "input must have a non-empty last dimension");
  const int64_t C = input.size(-1);
  const int64_t N = input.numel() / C;
  TORCH_CHECK(weight.numel() == C, "weight has ", weight.numel(), " elements, expected ", C);
  TORCH_CHECK(weight.device() == input.device(), "weight must be on ", input.device());
  // Upstream selects the fused add form for a defined, non-empty residual.
  const bool fused = residual.has_value() && residual->defined() && residual->numel() > 0;
  if (fused) {
    check_half_cuda(*residual, "residual");
    TORCH_CHECK(residual->numel() == input.numel(), "residual must have the shape of input");
    TORCH_CHECK(residual->device() == input.device(), "residual must be on ", input.device());
  }
  const c10::cuda::CUDAGuard guard(input.device());
  auto out = torch::empty_like(input);
  auto rms = torch::empty({N}, input.options().dtype(torch::kFloat));
  const int rc = qwen_b200_rmsnorm_forward(
      out.data_ptr(), rms.data_ptr<float>(), input.data_ptr(), weight.data_ptr(),
      fused ? residual->data_ptr() : nullptr, N, static_cast<int>(C), static_cast<float>(eps),
      c10::cuda::getCurrentCUDAStream(input.device().index()).stream());
  if (rc != 0) {
    char msg[512];
    qwen_b200_last_error(msg, sizeof(msg));
    TORCH_CHECK(false, "rmsnorm.forward failed (code ", rc, "): ", msg);
  }
  return {out, rms};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &forward, "RMSNorm forward (B200)", py::arg("input"), py::arg("weight"),
        py::arg("eps"), py::arg("residual") = py::none());
  m.def(
      "backward",
      [](py::args, py::kwargs) {
        TORCH_CHECK(false, "rmsnorm.backward is not part of this inference build");
      },
      "not available: this build implements the forward operators only");
}
