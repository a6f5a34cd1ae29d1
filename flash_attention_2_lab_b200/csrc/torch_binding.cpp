// PyTorch extension module `flash_attention_cuda`: the drop-in boundary.
//
// Exposes the reference's production entry point
//   tensorcore_attention_forward_production_128x128(query, key, value, causal)
// (reference csrc/bindings.cpp:63-68, :136-140) with the same argument
// meaning, the same input checks and error messages
// (csrc/tensorcore_attention.cu:2731-2823, :3035-3038), the same output
// allocation (empty_like(query), :2991) and the same stream (the current
// stream of query's device, :3084-3087). The arithmetic runs in the sm_100a
// kernel behind the C ABI in include/fa_sm100.h; this file holds no device
// code and has no fallback.
//
// The reference's older noncausal entry points (bindings.cpp:112-134) are
// kept with their own divisibility checks and routed to the same kernel.
// `attention_forward` is the general form: any sequence length, different
// query/key lengths, optional scale.

#include <torch/extension.h>
#include <vector>

#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>

#include <cmath>
#include <optional>

#include "fa_sm100.h"

namespace {

constexpr int64_t kHeadDimension = 64;

// Checks of validate_tensorcore_attention_inputs<kKeyTileSize>
// (reference csrc/tensorcore_attention.cu:2731-2823), same order and text.
void validate_inputs(const torch::Tensor& query, const torch::Tensor& key,
                     const torch::Tensor& value, int64_t key_tile) {
  TORCH_CHECK(query.is_cuda(), "query must be a CUDA tensor");
  TORCH_CHECK(key.is_cuda(), "key must be a CUDA tensor");
  TORCH_CHECK(value.is_cuda(), "value must be a CUDA tensor");
  TORCH_CHECK(query.device() == key.device() && query.device() == value.device(),
              "query, key, and value must be on the same device");
  TORCH_CHECK(query.scalar_type() == at::kHalf, "query must have dtype torch.float16");
  TORCH_CHECK(key.scalar_type() == at::kHalf, "key must have dtype torch.float16");
  TORCH_CHECK(value.scalar_type() == at::kHalf, "value must have dtype torch.float16");
  TORCH_CHECK(query.dim() == 4, "query must have shape [B, H, N, D]");
  TORCH_CHECK(key.dim() == 4, "key must have shape [B, H, N, D]");
  TORCH_CHECK(value.dim() == 4, "value must have shape [B, H, N, D]");
  TORCH_CHECK(query.sizes() == key.sizes(), "query and key must have identical shapes");
  TORCH_CHECK(query.sizes() == value.sizes(), "query and value must have identical shapes");
  TORCH_CHECK(query.is_contiguous(), "query must be contiguous");
  TORCH_CHECK(key.is_contiguous(), "key must be contiguous");
  TORCH_CHECK(value.is_contiguous(), "value must be contiguous");
  TORCH_CHECK(query.size(3) == kHeadDimension, "head dimension must equal 64");
  TORCH_CHECK(query.size(2) % key_tile == 0, "sequence length must be divisible by ", key_tile);
}

void check_status(int rc) {
  TORCH_CHECK(rc == FA_OK, "fa_fwd_sm100 failed (", rc, "): ", fa_last_error());
}

torch::Tensor run_fixed(const torch::Tensor& query, const torch::Tensor& key,
                        const torch::Tensor& value, bool causal, int64_t key_tile,
                        bool grid_y_check) {
  validate_inputs(query, key, value, key_tile);
  const c10::cuda::CUDAGuard device_guard(query.device());
  torch::Tensor output = torch::empty_like(query);
  const int64_t batch = query.size(0), heads = query.size(1), seq = query.size(2);
  if (batch == 0 || heads == 0 || seq == 0) return output;
  if (grid_y_check) {
    // The reference grid puts batch*heads on grid.y (:3035-3038); the
    // persistent kernel has no such limit, but the drop-in keeps the check.
    TORCH_CHECK(batch * heads <= 65535, "batch * heads exceeds CUDA grid.y limit");
  }
  const float scale = 1.0f / std::sqrt(static_cast<float>(kHeadDimension));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(query.get_device()).stream();
  check_status(fa_fwd_sm100(query.data_ptr(), key.data_ptr(), value.data_ptr(),
                            output.data_ptr(), batch, heads, seq, causal ? 1 : 0, scale, stream));
  return output;
}

}  // namespace

torch::Tensor tensorcore_attention_forward_production_128x128(torch::Tensor query,
                                                              torch::Tensor key,
                                                              torch::Tensor value, bool causal) {
  return run_fixed(query, key, value, causal, 128, true);
}

torch::Tensor tensorcore_attention_forward(torch::Tensor query, torch::Tensor key,
                                           torch::Tensor value) {
  return run_fixed(query, key, value, false, 16, true);
}

torch::Tensor tensorcore_attention_forward_bc32(torch::Tensor query, torch::Tensor key,
                                                torch::Tensor value) {
  return run_fixed(query, key, value, false, 32, true);
}

torch::Tensor tensorcore_attention_forward_bc32_raw_pv(torch::Tensor query, torch::Tensor key,
                                                       torch::Tensor value) {
  return run_fixed(query, key, value, false, 32, true);
}

torch::Tensor tensorcore_attention_forward_bc32_raw_qk_raw_pv(torch::Tensor query,
                                                              torch::Tensor key,
                                                              torch::Tensor value) {
  return run_fixed(query, key, value, false, 32, true);
}

// General form: q [B,H,Nq,64], k/v [B,H,Nk,64], any Nq, Nk >= 1.
torch::Tensor attention_forward(torch::Tensor query, torch::Tensor key, torch::Tensor value,
                                bool causal, std::optional<double> scale) {
  TORCH_CHECK(query.is_cuda(), "query must be a CUDA tensor");
  TORCH_CHECK(key.is_cuda(), "key must be a CUDA tensor");
  TORCH_CHECK(value.is_cuda(), "value must be a CUDA tensor");
  TORCH_CHECK(query.device() == key.device() && query.device() == value.device(),
              "query, key, and value must be on the same device");
  TORCH_CHECK(query.scalar_type() == at::kHalf && key.scalar_type() == at::kHalf &&
                  value.scalar_type() == at::kHalf,
              "query, key and value must have dtype torch.float16");
  TORCH_CHECK(query.dim() == 4 && key.dim() == 4 && value.dim() == 4,
              "query, key and value must have shape [B, H, N, D]");
  TORCH_CHECK(query.size(0) == key.size(0) && query.size(0) == value.size(0),
              "query, key, and value must have the same batch size");
  TORCH_CHECK(query.size(1) == key.size(1) && query.size(1) == value.size(1),
              "query, key, and value must have the same number of heads");
  TORCH_CHECK(key.sizes() == value.sizes(), "key and value must have identical shapes");
  TORCH_CHECK(query.size(3) == kHeadDimension && key.size(3) == kHeadDimension,
              "head dimension must equal 64");
  TORCH_CHECK(query.is_contiguous() && key.is_contiguous() && value.is_contiguous(),
              "query, key and value must be contiguous");
  const c10::cuda::CUDAGuard device_guard(query.device());
  torch::Tensor output = torch::empty_like(query);
  const int64_t batch = query.size(0), heads = query.size(1);
  const int64_t nq = query.size(2), nk = key.size(2);
  if (batch == 0 || heads == 0 || nq == 0) return output;
  TORCH_CHECK(nk > 0, "key length must be positive when there are queries");
  const float s = scale.has_value() ? static_cast<float>(*scale)
                                    : 1.0f / std::sqrt(static_cast<float>(kHeadDimension));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(query.get_device()).stream();
  check_status(fa_fwd_sm100_varlen(query.data_ptr(), key.data_ptr(), value.data_ptr(),
                                   output.data_ptr(), batch, heads, nq, nk, causal ? 1 : 0, s,
                                   stream));
  return output;
}

namespace {

// Tensors shaped like query [B, H, Nq, 64] (query, output, grad_output) and
// like key [B, H, Nk, 64] (key, value).
void check_training_inputs(const std::vector<std::pair<const char*, const torch::Tensor*>>& qs,
                           const std::vector<std::pair<const char*, const torch::Tensor*>>& ks) {
  const torch::Tensor& ref = *qs.front().second;
  TORCH_CHECK(ref.dim() == 4, "query must have shape [B, H, N, D]");
  TORCH_CHECK(ref.size(3) == kHeadDimension, "head dimension must equal 64");
  auto common = [&](const char* name, const torch::Tensor& t) {
    TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
    TORCH_CHECK(t.device() == ref.device(), name, " must be on the same device as query");
    TORCH_CHECK(t.scalar_type() == at::kHalf, name, " must have dtype torch.float16");
    TORCH_CHECK(t.is_contiguous(), name, " must be contiguous");
  };
  for (const auto& nt : qs) {
    common(nt.first, *nt.second);
    TORCH_CHECK(nt.second->sizes() == ref.sizes(), nt.first, " must have the shape of query");
  }
  const torch::Tensor& kref = *ks.front().second;
  for (const auto& nt : ks) {
    const torch::Tensor& t = *nt.second;
    common(nt.first, t);
    TORCH_CHECK(t.dim() == 4 && t.size(0) == ref.size(0) && t.size(1) == ref.size(1) &&
                    t.size(3) == kHeadDimension,
                nt.first, " must have shape [B, H, N_kv, 64] with query's B and H");
    TORCH_CHECK(t.sizes() == kref.sizes(), nt.first, " must have the shape of key");
  }
}

}  // namespace

// Forward that also returns the row log-sum-exp [B, H, Nq] (fp32) for the
// backward; key length may differ from the query length.  No counterpart in
// the reference.
std::vector<torch::Tensor> attention_forward_lse(torch::Tensor query, torch::Tensor key,
                                                 torch::Tensor value, bool causal,
                                                 std::optional<double> scale) {
  check_training_inputs({{"query", &query}}, {{"key", &key}, {"value", &value}});
  const c10::cuda::CUDAGuard device_guard(query.device());
  torch::Tensor output = torch::empty_like(query);
  torch::Tensor lse = torch::empty({query.size(0), query.size(1), query.size(2)},
                                   query.options().dtype(at::kFloat));
  const int64_t batch = query.size(0), heads = query.size(1), nq = query.size(2),
                nk = key.size(2);
  if (batch == 0 || heads == 0 || nq == 0) return {output, lse};
  const float s = scale.has_value() ? static_cast<float>(*scale)
                                    : 1.0f / std::sqrt(static_cast<float>(kHeadDimension));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(query.get_device()).stream();
  check_status(fa_fwd_sm100_lse(query.data_ptr(), key.data_ptr(), value.data_ptr(),
                                output.data_ptr(), lse.data_ptr<float>(), batch, heads, nq, nk,
                                causal ? 1 : 0, s, stream));
  return {output, lse};
}

// Backward of attention_forward_lse: (dq, dk, dv).  No counterpart in the
// reference.
std::vector<torch::Tensor> attention_backward(torch::Tensor query, torch::Tensor key,
                                              torch::Tensor value, torch::Tensor output,
                                              torch::Tensor grad_output, torch::Tensor lse,
                                              bool causal, std::optional<double> scale) {
  check_training_inputs({{"query", &query}, {"output", &output}, {"grad_output", &grad_output}},
                        {{"key", &key}, {"value", &value}});
  TORCH_CHECK(lse.is_cuda() && lse.device() == query.device(), "lse must be on query's device");
  TORCH_CHECK(lse.scalar_type() == at::kFloat && lse.is_contiguous() && lse.dim() == 3 &&
                  lse.size(0) == query.size(0) && lse.size(1) == query.size(1) &&
                  lse.size(2) == query.size(2),
              "lse must be a contiguous float32 tensor of shape [B, H, N_q]");
  const c10::cuda::CUDAGuard device_guard(query.device());
  torch::Tensor dq = torch::empty_like(query), dk = torch::empty_like(key),
                dv = torch::empty_like(value);
  const int64_t batch = query.size(0), heads = query.size(1), nq = query.size(2),
                nk = key.size(2);
  if (batch == 0 || heads == 0 || (nq == 0 && nk == 0)) return {dq, dk, dv};
  const float s = scale.has_value() ? static_cast<float>(*scale)
                                    : 1.0f / std::sqrt(static_cast<float>(kHeadDimension));
  cudaStream_t stream = at::cuda::getCurrentCUDAStream(query.get_device()).stream();
  check_status(fa_bwd_sm100_varlen(query.data_ptr(), key.data_ptr(), value.data_ptr(),
                                   output.data_ptr(), grad_output.data_ptr(),
                                   lse.data_ptr<float>(), dq.data_ptr(), dk.data_ptr(),
                                   dv.data_ptr(), batch, heads, nq, nk, causal ? 1 : 0, s,
                                   stream));
  return {dq, dk, dv};
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, module) {
  module.def("attention_forward_lse", &attention_forward_lse,
             "Attention forward returning (output, row log-sum-exp) (sm_100a)",
             py::arg("query"), py::arg("key"), py::arg("value"), py::arg("causal") = false,
             py::arg("scale") = py::none());
  module.def("attention_backward", &attention_backward,
             "Attention backward: (dq, dk, dv) (sm_100a)", py::arg("query"), py::arg("key"),
             py::arg("value"), py::arg("output"), py::arg("grad_output"), py::arg("lse"),
             py::arg("causal") = false, py::arg("scale") = py::none());
  module.def("tensorcore_attention_forward_production_128x128",
             &tensorcore_attention_forward_production_128x128, "Production kernel",
             py::arg("query"), py::arg("key"), py::arg("value"), py::arg("causal"));
  module.def("tensorcore_attention_forward", &tensorcore_attention_forward,
             "Fused FP16 Tensor Core attention forward pass");
  module.def("tensorcore_attention_forward_bc32", &tensorcore_attention_forward_bc32,
             "Fused FP16 Tensor core attention forward with Bc=32");
  module.def("tensorcore_attention_forward_bc32_raw_pv", &tensorcore_attention_forward_bc32_raw_pv,
             "Fused FP16 Tensor Core attention with raw MMA PV");
  module.def("tensorcore_attention_forward_bc32_raw_qk_raw_pv",
             &tensorcore_attention_forward_bc32_raw_qk_raw_pv,
             "Fused FP16 Tensor Core attention with raw MMA QK");
  module.def("attention_forward", &attention_forward,
             "Attention forward, any sequence lengths (sm_100a)", py::arg("query"),
             py::arg("key"), py::arg("value"), py::arg("causal") = false,
             py::arg("scale") = py::none());
}
