// swiglu_fused: PyTorch extension module with the Python-facing API of the
// upstream Tools/swiglu extension (swiglu_binding.cpp:5-31):
//   forward(x, w_gate, w_up, b_gate=None, b_up=None) -> [out, gate_cache, up_cache]
//   forward_down(x, w_gate, w_up, w_down, b_gate=None, b_up=None, b_down=None) -> out
// x is [batch, seq, hidden] as upstream requires (swiglu.cu:323-326); weights
// in the upstream layout w_gate, w_up [hidden, inter], w_down [inter, hidden].
// Plus one call with no upstream counterpart as a single call:
//   rmsnorm_forward_down(x, norm_weight, eps, w_gate, w_up, w_down,
//                        residual=None, b_gate=None, b_up=None, b_down=None)
//     -> [out, normed, rms]  (rmsnorm.forward followed by forward_down)
// Kernels and C ABI in libqwen_b200.so (include/qwen_b200_ops.h).  fp16 only;
// `backward` (training) is not part of this build and raises.
// forward_down and rmsnorm_forward_down take one keyword more, `exact`:
//   None (default)  tensor cores (tcgen05, fp32 accumulation) from 64 rows on,
//                   upstream's fp16 accumulation chain (bit-identical) below;
//   True            the fp16 chain at every size (bit-identical to upstream);
//   False           the tensor cores at every size.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>

#include <optional>
#include <vector>

#include "qwen_b200.h"
#include "qwen_b200_ops.h"

namespace {

using OptT = std::optional<torch::Tensor>;

void check_half_cuda(const torch::Tensor &t, const char *name, const torch::Device &dev) {
  TORCH_CHECK(t.defined() && t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == dev, name, " must be on ", dev);
  TORCH_CHECK(t.scalar_type() == torch::kHalf, name, " must be float16 (this build is fp16 only), got ",
              t.scalar_type());
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
}

const void *opt_ptr(const OptT &t, const char *name, int64_t numel, const torch::Device &dev) {
  if (!t.has_value() || !t->defined()) return nullptr;
  check_half_cuda(*t, name, dev);
  TORCH_CHECK(t->numel() == numel, name, " has ", t->numel(), " elements, expected ", numel);
  return t->data_ptr();
}

void raise_if(int rc, const char *what) {
  if (rc == 0) return;
  char msg[512];
  qwen_b200_last_error(msg, sizeof(msg));
  TORCH_CHECK(false, what, " failed (code ", rc, "): ", msg);
}

void check_weights(const torch::Tensor &x, const torch::Tensor &wg, const torch::Tensor &wu,
                   int64_t H) {
  const auto dev = x.device();
  check_half_cuda(wg, "w_gate", dev);
  check_half_cuda(wu, "w_up", dev);
  TORCH_CHECK(wg.dim() == 2 && wg.size(0) == H, "w_gate must be [hidden=", H, ", inter]");
  TORCH_CHECK(wu.sizes() == wg.sizes(), "w_up must have the shape of w_gate");
}

cudaStream_t stream_of(const torch::Tensor &x) {
  return c10::cuda::getCurrentCUDAStream(x.device().index()).stream();
}

std::vector<torch::Tensor> forward(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up,
                                   OptT b_gate, OptT b_up) {
  TORCH_CHECK(x.dim() == 3, "x must be [batch, seq, hidden], got ", x.dim(), " dimensions");
  const auto dev = x.device();
  check_half_cuda(x, "x", dev);
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2);
  check_weights(x, w_gate, w_up, H);
  const int64_t I = w_gate.size(1);
  const c10::cuda::CUDAGuard guard(dev);
  const void *bg = opt_ptr(b_gate, "b_gate", I, dev);
  const void *bu = opt_ptr(b_up, "b_up", I, dev);
  auto out = torch::empty({B, S, I}, x.options());
  auto gc = torch::empty({B, S, I}, x.options());
  auto uc = torch::empty({B, S, I}, x.options());
  raise_if(qwen_b200_swiglu_forward(x.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(), bg, bu,
                                    out.data_ptr(), gc.data_ptr(), uc.data_ptr(), B * S,
                                    static_cast<int>(H), static_cast<int>(I), stream_of(x)),
           "swiglu_fused.forward");
  return {out, gc, uc};
}

int mode_of(std::optional<bool> exact) { return !exact.has_value() ? -1 : (*exact ? 1 : 0); }

torch::Tensor forward_down(torch::Tensor x, torch::Tensor w_gate, torch::Tensor w_up,
                           torch::Tensor w_down, OptT b_gate, OptT b_up, OptT b_down,
                           std::optional<bool> exact) {
  TORCH_CHECK(x.dim() == 3, "x must be [batch, seq, hidden], got ", x.dim(), " dimensions");
  const auto dev = x.device();
  check_half_cuda(x, "x", dev);
  const int64_t B = x.size(0), S = x.size(1), H = x.size(2);
  check_weights(x, w_gate, w_up, H);
  const int64_t I = w_gate.size(1);
  check_half_cuda(w_down, "w_down", dev);
  TORCH_CHECK(w_down.dim() == 2 && w_down.size(0) == I && w_down.size(1) == H,
              "w_down must be [inter=", I, ", hidden=", H, "]");
  const c10::cuda::CUDAGuard guard(dev);
  const void *bg = opt_ptr(b_gate, "b_gate", I, dev);
  const void *bu = opt_ptr(b_up, "b_up", I, dev);
  const void *bd = opt_ptr(b_down, "b_down", H, dev);
  auto out = torch::empty({B, S, H}, x.options());
  auto ws = torch::empty({qwen_b200_swiglu_forward_down_workspace(B * S, static_cast<int>(I))},
                         x.options().dtype(torch::kByte));
  raise_if(qwen_b200_swiglu_forward_down_ex(x.data_ptr(), w_gate.data_ptr(), w_up.data_ptr(),
                                            w_down.data_ptr(), bg, bu, bd, out.data_ptr(),
                                            ws.data_ptr(), B * S, static_cast<int>(H),
                                            static_cast<int>(I), mode_of(exact), stream_of(x)),
           "swiglu_fused.forward_down");
  return out;
}

std::vector<torch::Tensor> rmsnorm_forward_down(torch::Tensor x, torch::Tensor norm_weight,
                                                double eps, torch::Tensor w_gate,
                                                torch::Tensor w_up, torch::Tensor w_down,
                                                OptT residual, OptT b_gate, OptT b_up,
                                                OptT b_down, std::optional<bool> exact) {
  const auto dev = x.device();
  check_half_cuda(x, "x", dev);
  TORCH_CHECK(x.dim() >= 1 && x.size(-1) > 0, "x must have a non-empty last dimension");
  const int64_t H = x.size(-1), rows = x.numel() / H;
  check_half_cuda(norm_weight, "norm_weight", dev);
  TORCH_CHECK(norm_weight.numel() == H, "norm_weight must have ", H, " elements");
  check_weights(x, w_gate, w_up, H);
  const int64_t I = w_gate.size(1);
  check_half_cuda(w_down, "w_down", dev);
  TORCH_CHECK(w_down.dim() == 2 && w_down.size(0) == I && w_down.size(1) == H,
              "w_down must be [inter=", I, ", hidden=", H, "]");
  const c10::cuda::CUDAGuard guard(dev);
  void *res = nullptr;
  if (residual.has_value() && residual->defined() && residual->numel() > 0) {
    check_half_cuda(*residual, "residual", dev);
    TORCH_CHECK(residual->numel() == x.numel(), "residual must have the shape of x");
    res = residual->data_ptr();
  }
  const void *bg = opt_ptr(b_gate, "b_gate", I, dev);
  const void *bu = opt_ptr(b_up, "b_up", I, dev);
  const void *bd = opt_ptr(b_down, "b_down", H, dev);
  auto out = torch::empty_like(x);
  auto normed = torch::empty_like(x);
  auto rms = torch::empty({rows}, x.options().dtype(torch::kFloat));
  auto ws = torch::empty(
      {qwen_b200_rmsnorm_swiglu_down_workspace(rows, static_cast<int>(H), static_cast<int>(I))},
      x.options().dtype(torch::kByte));
  raise_if(qwen_b200_rmsnorm_swiglu_down_ex(
               x.data_ptr(), norm_weight.data_ptr(), res, static_cast<float>(eps),
               w_gate.data_ptr(), w_up.data_ptr(), w_down.data_ptr(), bg, bu, bd,
               normed.data_ptr(), rms.data_ptr<float>(), out.data_ptr(), ws.data_ptr(), rows,
               static_cast<int>(H), static_cast<int>(I), mode_of(exact), stream_of(x)),
           "swiglu_fused.rmsnorm_forward_down");
  return {out, normed, rms};
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("forward", &forward, "Fused SwiGLU forward (B200)", py::arg("x"), py::arg("w_gate"),
        py::arg("w_up"), py::arg("b_gate") = py::none(), py::arg("b_up") = py::none());
  m.def("forward_down", &forward_down, "Fused SwiGLU + down projection forward (B200)",
        py::arg("x"), py::arg("w_gate"), py::arg("w_up"), py::arg("w_down"),
        py::arg("b_gate") = py::none(), py::arg("b_up") = py::none(),
        py::arg("b_down") = py::none(), py::arg("exact") = py::none());
  m.def("rmsnorm_forward_down", &rmsnorm_forward_down,
        "RMSNorm followed by SwiGLU + down projection (B200)", py::arg("x"),
        py::arg("norm_weight"), py::arg("eps"), py::arg("w_gate"), py::arg("w_up"),
        py::arg("w_down"), py::arg("residual") = py::none(), py::arg("b_gate") = py::none(),
        py::arg("b_up") = py::none(), py::arg("b_down") = py::none(),
        py::arg("exact") = py::none());
  m.def(
      "backward",
      [](py::args, py::kwargs) {
        TORCH_CHECK(false, "swiglu_fused.backward is not part of this inference build");
      },
      "not available: this build implements the forward operators only");
}
