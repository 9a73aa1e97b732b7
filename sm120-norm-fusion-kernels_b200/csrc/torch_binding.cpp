// torch_binding.cpp -- the reference's Python-facing surface on top of the C ABI.
//
// Exposes exactly what the reference's csrc/bindings.cpp exposes (paths in the
// reference project):
//   * pybind11 module sm120_rmsnorm._C with rms_norm, rms_norm_out,
//     fused_add_rms_norm, fused_add_rms_norm_out, fused_add_rms_norm_inplace,
//     fused_qk_rms_norm_rope, fused_qk_rms_norm_rope_kv   (bindings.cpp:83-106)
//   * TORCH_LIBRARY(sm120_norm) with the two mutating schemas, verbatim, and
//     CUDA implementations                                 (bindings.cpp:66-81)
// Tensor validation raises RuntimeError with the reference's messages
// (csrc/rmsnorm_kernels.cu:439-452, 488-492, 548-583, 624-676, 732-745).
// Everything else -- version checks, shape dispatch, launch -- happens behind
// the C ABI in include/sm120norm_b200.h, on the tensors' device and on the
// current PyTorch stream. No host synchronisation; only rms_norm and
// fused_add_rms_norm allocate (their outputs).
#include <c10/cuda/CUDAGuard.h>
#include <c10/cuda/CUDAStream.h>
#include <torch/extension.h>
#include <torch/library.h>

#include <vector>

#include "sm120norm_b200.h"

namespace {

int dtype_code(const torch::Tensor& t) {
  switch (t.scalar_type()) {
    case torch::kFloat32: return SM120N_F32;
    case torch::kFloat16: return SM120N_F16;
    case torch::kBFloat16: return SM120N_BF16;
    default: return -1;
  }
}

void raise_if_failed(int status) {
  TORCH_CHECK(status == SM120N_OK, sm120n_last_error());
}

void* current_stream() {
  return static_cast<void*>(c10::cuda::getCurrentCUDAStream().stream());
}

void check_activation_and_weight(const torch::Tensor& input, const torch::Tensor& weight) {
  TORCH_CHECK(input.is_cuda(), "input must be a CUDA tensor");
  TORCH_CHECK(weight.is_cuda(), "weight must be a CUDA tensor");
  TORCH_CHECK(input.is_contiguous(), "input must be contiguous");
  TORCH_CHECK(weight.is_contiguous(), "weight must be contiguous");
  TORCH_CHECK(input.dim() >= 2, "input must have at least two dimensions");
  TORCH_CHECK(weight.dim() == 1, "weight must be one-dimensional");
  TORCH_CHECK(input.size(-1) == weight.numel(), "weight size must equal input hidden size");
  TORCH_CHECK(input.scalar_type() == weight.scalar_type(), "input and weight dtypes must match");
  TORCH_CHECK(dtype_code(input) >= 0, "supported dtypes are float16, bfloat16, and float32");
  TORCH_CHECK(input.device() == weight.device(), "all tensors must be on the same CUDA device");
}

void check_like_input(const torch::Tensor& t, const torch::Tensor& input, const char* name) {
  TORCH_CHECK(t.is_cuda() && t.is_contiguous(), name, " must be contiguous CUDA");
  TORCH_CHECK(t.sizes() == input.sizes(), name, " shape must match input");
  TORCH_CHECK(t.scalar_type() == input.scalar_type(), name, " dtype must match input");
  TORCH_CHECK(t.device() == input.device(), "all tensors must be on the same CUDA device");
}

}  // namespace

void b200_rms_norm_out(torch::Tensor input, torch::Tensor weight, torch::Tensor output,
                       double epsilon, int64_t version) {
  check_activation_and_weight(input, weight);
  TORCH_CHECK(output.is_cuda() && output.is_contiguous(), "output must be contiguous CUDA");
  TORCH_CHECK(output.sizes() == input.sizes(), "output shape must match input");
  TORCH_CHECK(output.scalar_type() == input.scalar_type(), "output dtype must match input");
  TORCH_CHECK(output.device() == input.device(), "all tensors must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(input.device());
  const int64_t hidden = input.size(-1);
  const int64_t rows = hidden == 0 ? 0 : input.numel() / hidden;
  raise_if_failed(sm120n_rms_norm(input.data_ptr(), weight.data_ptr(), output.data_ptr(), rows,
                                  hidden, dtype_code(input), static_cast<float>(epsilon),
                                  static_cast<int>(version), current_stream()));
}

torch::Tensor b200_rms_norm(torch::Tensor input, torch::Tensor weight, double epsilon,
                            int64_t version) {
  auto output = torch::empty_like(input);
  b200_rms_norm_out(input, weight, output, epsilon, version);
  return output;
}

void b200_fused_add_rms_norm_out(torch::Tensor input, torch::Tensor residual, torch::Tensor weight,
                                 torch::Tensor output, torch::Tensor residual_output,
                                 double epsilon, int64_t version) {
  check_activation_and_weight(input, weight);
  TORCH_CHECK(residual.is_cuda() && residual.is_contiguous(), "residual must be contiguous CUDA");
  TORCH_CHECK(residual.sizes() == input.sizes(), "residual shape must match input");
  TORCH_CHECK(residual.scalar_type() == input.scalar_type(), "residual dtype must match input");
  TORCH_CHECK(residual.device() == input.device(), "all tensors must be on the same CUDA device");
  check_like_input(output, input, "output");
  check_like_input(residual_output, input, "residual_output");
  c10::cuda::CUDAGuard guard(input.device());
  const int64_t hidden = input.size(-1);
  const int64_t rows = hidden == 0 ? 0 : input.numel() / hidden;
  raise_if_failed(sm120n_fused_add_rms_norm(
      input.data_ptr(), residual.data_ptr(), weight.data_ptr(), output.data_ptr(),
      residual_output.data_ptr(), rows, hidden, dtype_code(input), static_cast<float>(epsilon),
      static_cast<int>(version), current_stream()));
}

std::vector<torch::Tensor> b200_fused_add_rms_norm(torch::Tensor input, torch::Tensor residual,
                                                   torch::Tensor weight, double epsilon,
                                                   int64_t version) {
  auto output = torch::empty_like(input);
  auto residual_output = torch::empty_like(input);
  b200_fused_add_rms_norm_out(input, residual, weight, output, residual_output, epsilon, version);
  return {output, residual_output};
}

// residual += input; input = RMSNorm(residual) * weight.
void b200_fused_add_rms_norm_inplace(torch::Tensor input, torch::Tensor residual,
                                     torch::Tensor weight, double epsilon, int64_t version) {
  b200_fused_add_rms_norm_out(input, residual, weight, input, residual, epsilon, version);
}

namespace {

void check_qk(const torch::Tensor& query, const torch::Tensor& key,
              const torch::Tensor& query_weight, const torch::Tensor& key_weight,
              const torch::Tensor& positions, const torch::Tensor& cos_sin_cache,
              const char* head_dim_message) {
  TORCH_CHECK(query.is_cuda() && key.is_cuda(), "query and key must be CUDA tensors");
  TORCH_CHECK(query.is_contiguous() && key.is_contiguous(), "query and key must be contiguous");
  TORCH_CHECK(query.dim() == 3 && key.dim() == 3,
              "query and key must have shape [tokens, heads, head_dim]");
  TORCH_CHECK(query.size(0) == key.size(0), "query and key token counts must match");
  TORCH_CHECK(query.size(2) == 128 && key.size(2) == 128, head_dim_message);
  TORCH_CHECK(query.scalar_type() == key.scalar_type(), "query and key dtypes must match");
  TORCH_CHECK(dtype_code(query) >= 0, "supported dtypes are float16, bfloat16, and float32");
  TORCH_CHECK(query_weight.is_cuda() && key_weight.is_cuda(), "Q/K weights must be CUDA tensors");
  TORCH_CHECK(query_weight.is_contiguous() && key_weight.is_contiguous(),
              "Q/K weights must be contiguous");
  TORCH_CHECK(query_weight.numel() == 128 && key_weight.numel() == 128,
              "Q/K weights must contain 128 elements");
  TORCH_CHECK(query_weight.scalar_type() == query.scalar_type() &&
                  key_weight.scalar_type() == query.scalar_type(),
              "Q/K weight dtypes must match activations");
  TORCH_CHECK(positions.is_cuda() && positions.is_contiguous(),
              "positions must be a contiguous CUDA tensor");
  TORCH_CHECK(positions.scalar_type() == torch::kInt64, "positions must use int64 dtype");
  TORCH_CHECK(positions.numel() == query.size(0), "positions length must match token count");
  TORCH_CHECK(cos_sin_cache.is_cuda() && cos_sin_cache.is_contiguous(),
              "cos/sin cache must be a contiguous CUDA tensor");
  TORCH_CHECK(cos_sin_cache.scalar_type() == torch::kFloat32, "cos/sin cache must use float32 dtype");
  TORCH_CHECK(cos_sin_cache.dim() >= 1 && cos_sin_cache.size(-1) == 128,
              "cos/sin cache last dimension must be 128");
  TORCH_CHECK(query.device() == key.device() && query.device() == query_weight.device() &&
                  query.device() == key_weight.device() && query.device() == positions.device() &&
                  query.device() == cos_sin_cache.device(),
              "all tensors must be on the same CUDA device");
}

}  // namespace

void b200_fused_qk_rms_norm_rope(torch::Tensor query, torch::Tensor key, torch::Tensor query_weight,
                                 torch::Tensor key_weight, torch::Tensor positions,
                                 torch::Tensor cos_sin_cache, double epsilon, int64_t version) {
  check_qk(query, key, query_weight, key_weight, positions, cos_sin_cache,
           "fused QK Norm+RoPE requires head_dim=128");
  TORCH_CHECK(version == 1 || version == 2, "QK Norm+RoPE version must be 1 or 2");
  c10::cuda::CUDAGuard guard(query.device());
  raise_if_failed(sm120n_fused_qk_rms_norm_rope(
      query.data_ptr(), key.data_ptr(), query_weight.data_ptr(), key_weight.data_ptr(),
      positions.data_ptr<int64_t>(), cos_sin_cache.data_ptr<float>(), query.size(0), query.size(1),
      key.size(1), query.size(2), cos_sin_cache.numel() / 128, dtype_code(query),
      static_cast<float>(epsilon), static_cast<int>(version), current_stream()));
}

void b200_fused_qk_rms_norm_rope_kv(torch::Tensor query, torch::Tensor key, torch::Tensor value,
                                    torch::Tensor query_weight, torch::Tensor key_weight,
                                    torch::Tensor positions, torch::Tensor cos_sin_cache,
                                    torch::Tensor key_cache, torch::Tensor value_cache,
                                    torch::Tensor slot_mapping, double epsilon, int64_t version) {
  TORCH_CHECK(query.is_cuda() && key.is_cuda() && value.is_cuda(), "Q/K/V must be CUDA tensors");
  TORCH_CHECK(query.is_contiguous() && key.is_contiguous() && value.is_contiguous(),
              "Q/K/V must be contiguous");
  TORCH_CHECK(query.dim() == 3 && key.dim() == 3 && value.dim() == 3,
              "Q/K/V must have shape [tokens, heads, head_dim]");
  TORCH_CHECK(query.size(0) == key.size(0) && key.sizes() == value.sizes(),
              "Q/K/V token and KV shapes must match");
  TORCH_CHECK(query.scalar_type() == key.scalar_type() && key.scalar_type() == value.scalar_type(),
              "Q/K/V dtypes must match");
  check_qk(query, key, query_weight, key_weight, positions, cos_sin_cache,
           "fused QK Norm+RoPE+KV requires head_dim=128");
  TORCH_CHECK(key_cache.is_cuda() && value_cache.is_cuda() && key_cache.is_contiguous() &&
                  value_cache.is_contiguous(),
              "KV caches must be contiguous CUDA tensors");
  TORCH_CHECK(key_cache.sizes() == value_cache.sizes() &&
                  key_cache.scalar_type() == query.scalar_type() &&
                  value_cache.scalar_type() == query.scalar_type(),
              "KV cache shapes and dtypes must match activations");
  TORCH_CHECK(key_cache.dim() >= 2 && key_cache.size(-2) == key.size(1) &&
                  key_cache.size(-1) == 128,
              "KV cache must end in [key_heads, 128]");
  TORCH_CHECK(slot_mapping.is_cuda() && slot_mapping.is_contiguous() &&
                  slot_mapping.scalar_type() == torch::kInt &&
                  slot_mapping.numel() == query.size(0),
              "slot_mapping must be contiguous CUDA int32 with one entry per token");
  TORCH_CHECK(version == 1 || version == 4,
              "QK Norm+RoPE+KV version must be 1 or 4 warps per block");
  TORCH_CHECK(query.device() == value.device() && query.device() == key_cache.device() &&
                  query.device() == value_cache.device() &&
                  query.device() == slot_mapping.device(),
              "all tensors must be on the same CUDA device");
  c10::cuda::CUDAGuard guard(query.device());
  const int64_t slot_elems = key.size(1) * 128;
  const int64_t cache_slots = slot_elems == 0 ? 0 : key_cache.numel() / slot_elems;
  raise_if_failed(sm120n_fused_qk_rms_norm_rope_kv(
      query.data_ptr(), key.data_ptr(), value.data_ptr(), query_weight.data_ptr(),
      key_weight.data_ptr(), positions.data_ptr<int64_t>(), cos_sin_cache.data_ptr<float>(),
      key_cache.data_ptr(), value_cache.data_ptr(), slot_mapping.data_ptr<int32_t>(),
      query.size(0), query.size(1), key.size(1), query.size(2), cos_sin_cache.numel() / 128,
      cache_slots, dtype_code(query), static_cast<float>(epsilon), static_cast<int>(version),
      current_stream()));
}

TORCH_LIBRARY(sm120_norm, m) {
  m.def(
      "fused_qk_rms_norm_rope_(Tensor(a!) query, Tensor(b!) key, "
      "Tensor query_weight, Tensor key_weight, Tensor positions, "
      "Tensor cos_sin_cache, float epsilon=1e-6, int version=2) -> ()");
  m.def(
      "fused_qk_rms_norm_rope_kv_(Tensor(a!) query, Tensor(b!) key, Tensor value, "
      "Tensor query_weight, Tensor key_weight, Tensor positions, "
      "Tensor cos_sin_cache, Tensor(c!) key_cache, Tensor(d!) value_cache, "
      "Tensor slot_mapping, float epsilon=1e-6, int version=1) -> ()");
}

TORCH_LIBRARY_IMPL(sm120_norm, CUDA, m) {
  m.impl("fused_qk_rms_norm_rope_", &b200_fused_qk_rms_norm_rope);
  m.impl("fused_qk_rms_norm_rope_kv_", &b200_fused_qk_rms_norm_rope_kv);
}

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.doc() = "B200 (sm_100a) fused normalisation kernels behind the sm120_rmsnorm._C interface";
  m.def("rms_norm", &b200_rms_norm, "RMSNorm forward (CUDA)");
  m.def("rms_norm_out", &b200_rms_norm_out, "RMSNorm forward into preallocated output (CUDA)");
  m.def("fused_add_rms_norm", &b200_fused_add_rms_norm, "Fused residual add + RMSNorm forward (CUDA)");
  m.def("fused_add_rms_norm_out", &b200_fused_add_rms_norm_out,
        "Fused residual add + RMSNorm into preallocated outputs (CUDA)");
  m.def("fused_add_rms_norm_inplace", &b200_fused_add_rms_norm_inplace,
        "In-place fused residual add + RMSNorm (CUDA)");
  m.def("fused_qk_rms_norm_rope", &b200_fused_qk_rms_norm_rope,
        "In-place fused Q/K RMSNorm + RoPE (CUDA)");
  m.def("fused_qk_rms_norm_rope_kv", &b200_fused_qk_rms_norm_rope_kv,
        "In-place fused Q/K RMSNorm + RoPE + paged KV store (CUDA)");
}
