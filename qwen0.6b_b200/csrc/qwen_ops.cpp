// qwen_megakernel_C: PyTorch extension module with the same Python-facing
// API as the upstream binding (Tools/megakernel/qwen_ops.cpp:30-170):
// decode(), generate_nosync(), abi_version() (+ built_torch_version(), which
// the upstream Python layer probes at Model/Qwen06B_architecture.py:76-81).
// It only converts tensors to raw pointers and calls the C ABI of
// libqwen_b200.so (include/qwen_b200.h); no computation happens here.
//
// Differences from the upstream binding, all in error handling: arguments
// are validated (device, dtype, size, 16-byte alignment) and every failure
// raises RuntimeError instead of surfacing later as a CUDA fault.
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>
#include <torch/version.h>

#include <cstdint>
#include <string>

#include "qwen_b200.h"

namespace {

constexpr int64_t kHidden = 1024, kInter = 3072, kQ = 2048, kKV = 1024, kHeadDim = 128;
constexpr int64_t kVocab = 151936, kKVHeads = 8;

void check_tensor(const torch::Tensor &t, const char *name, torch::ScalarType dt, int64_t min_numel,
                  const torch::Device &dev) {
  TORCH_CHECK(t.defined(), name, " is undefined");
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.device() == dev, name, " is on ", t.device(), " but embed_weight is on ", dev);
  TORCH_CHECK(t.scalar_type() == dt, name, " must have dtype ", dt, ", got ", t.scalar_type());
  TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  TORCH_CHECK(t.numel() >= min_numel, name, " has ", t.numel(), " elements, needs >= ", min_numel);
  TORCH_CHECK(reinterpret_cast<uintptr_t>(t.data_ptr()) % 16 == 0, name,
              " must be 16-byte aligned (address ends in ",
              reinterpret_cast<uintptr_t>(t.data_ptr()) % 16, ")");
}

void raise_if_failed(const char *what) {
  char msg[512];
  const int rc = qwen_b200_last_error(msg, sizeof(msg));
  TORCH_CHECK(rc == 0, what, " failed (code ", rc, "): ", msg);
}

int num_sms(const torch::Device &dev) {
  int sms = 0;
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev.index());
  return sms;
}

struct Bufs {
  torch::Tensor embed, packed, final_norm, lm_head, cos, sin, kc, vc, hidden, act, res, q, k, v,
      attn, inter, norm, bvals, bidx;
};

void validate(const Bufs &b, int num_layers, int max_seq_len) {
  const auto dev = b.embed.device();
  TORCH_CHECK(num_layers >= 1, "num_layers must be >= 1");
  TORCH_CHECK(max_seq_len >= 1, "max_seq_len must be >= 1");
  const auto f16 = torch::kHalf, f32 = torch::kFloat, i32 = torch::kInt, i64 = torch::kLong;
  check_tensor(b.embed, "embed_weight", f16, kVocab * kHidden, dev);
  // Upstream guard (qwen_ops.cpp:64-65): the packed table must be 16-byte aligned.
  check_tensor(b.packed, "layer_weights_packed", i64, 12LL * num_layers, dev);
  check_tensor(b.final_norm, "final_norm_weight", f16, kHidden, dev);
  check_tensor(b.lm_head, "lm_head_weight", f16, kVocab * kHidden, dev);
  check_tensor(b.cos, "cos_table", f16, int64_t(max_seq_len) * kHeadDim, dev);
  check_tensor(b.sin, "sin_table", f16, int64_t(max_seq_len) * kHeadDim, dev);
  const int64_t kv = int64_t(num_layers) * kKVHeads * max_seq_len * kHeadDim;
  check_tensor(b.kc, "k_cache", f16, kv, dev);
  check_tensor(b.vc, "v_cache", f16, kv, dev);
  check_tensor(b.hidden, "hidden", f16, kHidden, dev);
  check_tensor(b.act, "act", f32, kHidden, dev);
  check_tensor(b.res, "res", f32, kHidden, dev);
  check_tensor(b.q, "q", f16, kQ, dev);
  check_tensor(b.k, "k", f16, kKV, dev);
  check_tensor(b.v, "v", f16, kKV, dev);
  check_tensor(b.attn, "attn_out", f16, kQ, dev);
  check_tensor(b.inter, "mlp_inter", f32, kInter, dev);
  check_tensor(b.norm, "norm_out", f32, kHidden, dev);
  const int sms = num_sms(dev);
  check_tensor(b.bvals, "bmax_vals", f32, sms, dev);
  check_tensor(b.bidx, "bmax_idxs", i32, sms, dev);
}

}  // namespace

int abi_version() { return qwen_b200_abi_version(); }

std::string built_torch_version() { return std::string(TORCH_VERSION); }

torch::Tensor decode(int input_token_id, torch::Tensor embed_weight,
                     torch::Tensor layer_weights_packed, torch::Tensor final_norm_weight,
                     torch::Tensor lm_head_weight, torch::Tensor cos_table,
                     torch::Tensor sin_table, torch::Tensor k_cache, torch::Tensor v_cache,
                     torch::Tensor hidden, torch::Tensor act, torch::Tensor res, torch::Tensor q,
                     torch::Tensor k, torch::Tensor v, torch::Tensor attn_out,
                     torch::Tensor mlp_inter, torch::Tensor norm_out, torch::Tensor bmax_vals,
                     torch::Tensor bmax_idxs, int num_layers, int position, int max_seq_len,
                     float attn_scale) {
  Bufs b{embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
         sin_table, k_cache, v_cache, hidden, act, res, q, k, v, attn_out, mlp_inter, norm_out,
         bmax_vals, bmax_idxs};
  validate(b, num_layers, max_seq_len);
  const c10::cuda::CUDAGuard guard(embed_weight.device());
  auto out = torch::empty({1}, torch::dtype(torch::kInt32).device(embed_weight.device()));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(embed_weight.device().index());
  launch_ldg_decode_direct(
      input_token_id, out.data_ptr<int>(), embed_weight.data_ptr(),
      reinterpret_cast<const LDGLayerWeight *>(layer_weights_packed.data_ptr()),
      final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
      sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), hidden.data_ptr(),
      act.data_ptr(), res.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
      attn_out.data_ptr(), mlp_inter.data_ptr(), norm_out.data_ptr(), bmax_vals.data_ptr(),
      bmax_idxs.data_ptr(), num_layers, position, max_seq_len, attn_scale, stream);
  raise_if_failed("qwen_megakernel_C.decode");
  return out;
}

torch::Tensor generate_nosync(int first_token_id, int num_steps, torch::Tensor embed_weight,
                              torch::Tensor layer_weights_packed, torch::Tensor final_norm_weight,
                              torch::Tensor lm_head_weight, torch::Tensor cos_table,
                              torch::Tensor sin_table, torch::Tensor k_cache,
                              torch::Tensor v_cache, torch::Tensor hidden, torch::Tensor act,
                              torch::Tensor res, torch::Tensor q, torch::Tensor k, torch::Tensor v,
                              torch::Tensor attn_out, torch::Tensor mlp_inter,
                              torch::Tensor norm_out, torch::Tensor bmax_vals,
                              torch::Tensor bmax_idxs, int num_layers, int start_position,
                              int max_seq_len, float attn_scale) {
  Bufs b{embed_weight, layer_weights_packed, final_norm_weight, lm_head_weight, cos_table,
         sin_table, k_cache, v_cache, hidden, act, res, q, k, v, attn_out, mlp_inter, norm_out,
         bmax_vals, bmax_idxs};
  validate(b, num_layers, max_seq_len);
  TORCH_CHECK(num_steps >= 1, "num_steps must be >= 1");
  const c10::cuda::CUDAGuard guard(embed_weight.device());
  auto out = torch::empty({num_steps}, torch::dtype(torch::kInt32).device(embed_weight.device()));
  cudaStream_t stream = c10::cuda::getCurrentCUDAStream(embed_weight.device().index());
  launch_ldg_generate_nosync(
      first_token_id, num_steps, embed_weight.data_ptr(),
      reinterpret_cast<const LDGLayerWeight *>(layer_weights_packed.data_ptr()),
      final_norm_weight.data_ptr(), lm_head_weight.data_ptr(), cos_table.data_ptr(),
      sin_table.data_ptr(), k_cache.data_ptr(), v_cache.data_ptr(), hidden.data_ptr(),
      act.data_ptr(), res.data_ptr(), q.data_ptr(), k.data_ptr(), v.data_ptr(),
      attn_out.data_ptr(), mlp_inter.data_ptr(), norm_out.data_ptr(), bmax_vals.data_ptr(),
      bmax_idxs.data_ptr(), out.data_ptr<int>(), num_layers, start_position, max_seq_len,
      attn_scale, stream);
  raise_if_failed("qwen_megakernel_C.generate_nosync");
  return out;
}

// Device-side status of the last launch on `device` (synchronises that
// device): 0 = ok, else the code of the bounded wait that gave up.
int64_t device_status(int device) {
  uint64_t detail = 0;
  const int rc = qwen_b200_device_status(device, &detail);
  return rc == 0 ? 0 : static_cast<int64_t>(detail & 0xffffffffull) | (int64_t(rc) << 32);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("decode", &decode, "Qwen3 single token decode (B200 persistent kernel)");
  m.def("generate_nosync", &generate_nosync,
        "Qwen3 greedy generation, all steps in one device-resident launch");
  m.def("abi_version", &abi_version, "ABI version of the packed weight table");
  m.def("built_torch_version", &built_torch_version, "torch version this module was built with");
  m.def("device_status", &device_status, "status word of the last decode launch on a device");
  m.def("set_wait_timeout_ns", &qwen_b200_set_wait_timeout_ns, "bound for every device-side wait");
}
