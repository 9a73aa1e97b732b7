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
//
// Beyond the reference: TORCH_LIBRARY(sm120_norm_ext) with the engine-side
// extensions of the same path (generalised Q/K norm + RoPE + cache store;
// RMSNorm with fp8 quantisation, under the operator names and argument order
// fp8 inference engines use for those fusions). The reference's namespace is
// left exactly as it is.
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

// ---------------------------------------------------------------------------
// Extensions
// ---------------------------------------------------------------------------
namespace {

bool is_fp8_storage(const torch::Tensor& t) {
  return t.scalar_type() == torch::kFloat8_e4m3fn || t.scalar_type() == torch::kByte;
}

// [tokens, heads, head_dim] with adjacent heads and elements; any token stride.
void check_head_rows(const torch::Tensor& t, const char* name) {
  TORCH_CHECK(t.is_cuda(), name, " must be a CUDA tensor");
  TORCH_CHECK(t.dim() == 3, name, " must have shape [tokens, heads, head_dim]");
  TORCH_CHECK(t.size(2) <= 1 || t.stride(2) == 1, name, " must have unit element stride");
  TORCH_CHECK(t.size(1) <= 1 || t.stride(1) == t.size(2), name,
              " heads must be adjacent (head stride == head_dim)");
}

int64_t token_stride(const torch::Tensor& t) {
  return t.size(0) <= 1 ? t.size(1) * t.size(2) : t.stride(0);
}

}  // namespace

void b200_qk_norm_rope_cache(torch::Tensor query, torch::Tensor key,
                             c10::optional<torch::Tensor> value, torch::Tensor query_weight,
                             torch::Tensor key_weight, torch::Tensor positions,
                             torch::Tensor cos_sin_cache, c10::optional<torch::Tensor> key_cache,
                             c10::optional<torch::Tensor> value_cache,
                             c10::optional<torch::Tensor> slot_mapping,
                             c10::optional<torch::Tensor> k_scale,
                             c10::optional<torch::Tensor> v_scale, bool is_neox,
                             c10::string_view kv_cache_layout, double epsilon) {
  check_head_rows(query, "query");
  check_head_rows(key, "key");
  TORCH_CHECK(query.size(0) == key.size(0), "query and key token counts must match");
  TORCH_CHECK(query.size(2) == key.size(2), "query and key head sizes must match");
  TORCH_CHECK(query.scalar_type() == key.scalar_type(), "query and key dtypes must match");
  TORCH_CHECK(dtype_code(query) >= 0, "supported dtypes are float16, bfloat16, and float32");
  const int64_t head_dim = query.size(2);
  TORCH_CHECK(query_weight.is_cuda() && key_weight.is_cuda() && query_weight.is_contiguous() &&
                  key_weight.is_contiguous(),
              "Q/K weights must be contiguous CUDA tensors");
  TORCH_CHECK(query_weight.numel() == head_dim && key_weight.numel() == head_dim,
              "Q/K weights must contain head_dim elements");
  TORCH_CHECK(query_weight.scalar_type() == query.scalar_type() &&
                  key_weight.scalar_type() == query.scalar_type(),
              "Q/K weight dtypes must match activations");
  TORCH_CHECK(positions.is_cuda() && positions.is_contiguous() &&
                  positions.scalar_type() == torch::kInt64 && positions.numel() == query.size(0),
              "positions must be contiguous CUDA int64 with one entry per token");
  TORCH_CHECK(cos_sin_cache.is_cuda() && cos_sin_cache.is_contiguous() &&
                  cos_sin_cache.scalar_type() == torch::kFloat32 && cos_sin_cache.dim() >= 1,
              "cos/sin cache must be a contiguous CUDA float32 tensor");
  const int64_t rotary_dim = cos_sin_cache.size(-1);
  const auto device = query.device();
  TORCH_CHECK(key.device() == device && query_weight.device() == device &&
                  key_weight.device() == device && positions.device() == device &&
                  cos_sin_cache.device() == device,
              "all tensors must be on the same CUDA device");

  sm120n_qk_cache_args a{};
  a.struct_size = sizeof(a);
  a.dtype = dtype_code(query);
  a.tokens = query.size(0);
  a.query_heads = query.size(1);
  a.key_heads = key.size(1);
  a.head_dim = head_dim;
  a.rotary_dim = rotary_dim;
  a.rope_style = is_neox ? SM120N_ROPE_NEOX : SM120N_ROPE_INTERLEAVED;
  a.cache_dtype = SM120N_CACHE_AUTO;
  a.query = query.data_ptr();
  a.query_token_stride = token_stride(query);
  a.key = key.data_ptr();
  a.key_token_stride = token_stride(key);
  a.query_weight = query_weight.data_ptr();
  a.key_weight = key_weight.data_ptr();
  a.positions = positions.data_ptr<int64_t>();
  a.cos_sin_cache = cos_sin_cache.data_ptr<float>();
  a.rope_positions = rotary_dim == 0 ? 0 : cos_sin_cache.numel() / rotary_dim;
  a.epsilon = static_cast<float>(epsilon);

  const bool store = key_cache.has_value() || value_cache.has_value();
  if (store) {
    TORCH_CHECK(key_cache.has_value() && value_cache.has_value() && value.has_value() &&
                    slot_mapping.has_value(),
                "a KV store needs value, key_cache, value_cache and slot_mapping");
    const auto& v = *value;
    const auto& kc = *key_cache;
    const auto& vc = *value_cache;
    const auto& slots = *slot_mapping;
    check_head_rows(v, "value");
    TORCH_CHECK(v.sizes() == key.sizes() && v.scalar_type() == key.scalar_type(),
                "value shape and dtype must match key");
    const bool nhd = kv_cache_layout == "NHD";
    TORCH_CHECK(nhd || kv_cache_layout == "HND", "kv_cache_layout must be \"NHD\" or \"HND\"");
    TORCH_CHECK(kc.is_cuda() && vc.is_cuda() && kc.dim() == 4 && vc.sizes() == kc.sizes() &&
                    vc.strides() == kc.strides() && vc.scalar_type() == kc.scalar_type(),
                "key_cache and value_cache must be 4-D CUDA tensors of one shape, stride "
                "and dtype");
    const int64_t head_axis = nhd ? 2 : 1;
    const int64_t slot_axis = nhd ? 1 : 2;
    TORCH_CHECK(kc.size(head_axis) == key.size(1) && kc.size(3) == head_dim,
                nhd ? "NHD caches must be [blocks, block_size, key_heads, head_dim]"
                    : "HND caches must be [blocks, key_heads, block_size, head_dim]");
    TORCH_CHECK(kc.stride(3) == 1, "KV caches must have unit element stride");
    const bool fp8 = is_fp8_storage(kc);
    TORCH_CHECK(fp8 || kc.scalar_type() == query.scalar_type(),
                "KV caches must use the activation dtype or fp8 e4m3 (float8_e4m3fn / uint8)");
    TORCH_CHECK(slots.is_cuda() && slots.is_contiguous() && slots.scalar_type() == torch::kInt &&
                    slots.numel() == query.size(0),
                "slot_mapping must be contiguous CUDA int32 with one entry per token");
    TORCH_CHECK(v.device() == device && kc.device() == device && vc.device() == device &&
                    slots.device() == device,
                "all tensors must be on the same CUDA device");
    if (fp8) {
      TORCH_CHECK(k_scale.has_value() && v_scale.has_value(), "fp8 caches need k_scale and v_scale");
      for (const auto* scale : {&*k_scale, &*v_scale}) {
        TORCH_CHECK(scale->is_cuda() && scale->scalar_type() == torch::kFloat32 &&
                        scale->numel() == 1 && scale->device() == device,
                    "k_scale and v_scale must be one-element CUDA float32 tensors");
      }
      a.cache_dtype = SM120N_CACHE_FP8_E4M3;
      a.k_scale = k_scale->data_ptr<float>();
      a.v_scale = v_scale->data_ptr<float>();
    }
    a.value = v.data_ptr();
    a.value_token_stride = token_stride(v);
    a.key_cache = kc.data_ptr();
    a.value_cache = vc.data_ptr();
    a.slot_mapping = slots.data_ptr<int32_t>();
    a.num_blocks = kc.size(0);
    a.block_size = kc.size(slot_axis);
    a.cache_block_stride = kc.stride(0);
    a.cache_slot_stride = kc.stride(slot_axis);
    a.cache_head_stride = kc.stride(head_axis);
  }
  c10::cuda::CUDAGuard guard(device);
  raise_if_failed(sm120n_qk_norm_rope_cache(&a, current_stream()));
}

namespace {

void check_quant_output(const torch::Tensor& result, const torch::Tensor& input) {
  TORCH_CHECK(result.is_cuda() && result.is_contiguous() && is_fp8_storage(result),
              "result must be a contiguous CUDA float8_e4m3fn (or uint8) tensor");
  TORCH_CHECK(result.sizes() == input.sizes(), "result shape must match input");
  TORCH_CHECK(result.device() == input.device(), "all tensors must be on the same CUDA device");
}

void check_scalar_scale(const torch::Tensor& scale, const torch::Tensor& input, const char* name) {
  TORCH_CHECK(scale.is_cuda() && scale.scalar_type() == torch::kFloat32 && scale.numel() == 1 &&
                  scale.device() == input.device(),
              name, " must be a one-element CUDA float32 tensor");
}

void run_norm_quant(torch::Tensor& result, const torch::Tensor& input,
                    const c10::optional<torch::Tensor>& residual, const torch::Tensor& weight,
                    const float* scale, float* token_scales, const float* scale_ub,
                    double epsilon) {
  check_activation_and_weight(input, weight);
  check_quant_output(result, input);
  const void* residual_ptr = nullptr;
  if (residual.has_value()) {
    check_like_input(*residual, input, "residual");
    residual_ptr = residual->data_ptr();
  }
  c10::cuda::CUDAGuard guard(input.device());
  const int64_t hidden = input.size(-1);
  const int64_t rows = hidden == 0 ? 0 : input.numel() / hidden;
  raise_if_failed(sm120n_rms_norm_fp8_quant(
      input.data_ptr(), residual_ptr, weight.data_ptr(), const_cast<void*>(residual_ptr),
      result.data_ptr(), scale, token_scales, scale_ub, rows, hidden, dtype_code(input),
      static_cast<float>(epsilon), current_stream()));
}

}  // namespace

void b200_rms_norm_static_fp8_quant(torch::Tensor result, torch::Tensor input,
                                    torch::Tensor weight, torch::Tensor scale, double epsilon) {
  check_scalar_scale(scale, input, "scale");
  run_norm_quant(result, input, c10::nullopt, weight, scale.data_ptr<float>(), nullptr, nullptr,
                 epsilon);
}

// residual = input + residual (in place); result = quant(RMSNorm(residual)).
void b200_fused_add_rms_norm_static_fp8_quant(torch::Tensor result, torch::Tensor input,
                                              torch::Tensor residual, torch::Tensor weight,
                                              torch::Tensor scale, double epsilon) {
  check_scalar_scale(scale, input, "scale");
  run_norm_quant(result, input, residual, weight, scale.data_ptr<float>(), nullptr, nullptr,
                 epsilon);
}

void b200_rms_norm_dynamic_per_token_quant(torch::Tensor result, torch::Tensor input,
                                           torch::Tensor weight, torch::Tensor scale,
                                           double epsilon, c10::optional<torch::Tensor> scale_ub,
                                           c10::optional<torch::Tensor> residual) {
  const int64_t hidden = input.size(-1);
  const int64_t rows = hidden == 0 ? 0 : input.numel() / hidden;
  TORCH_CHECK(scale.is_cuda() && scale.is_contiguous() && scale.scalar_type() == torch::kFloat32 &&
                  scale.numel() == rows && scale.device() == input.device(),
              "scale must be a contiguous CUDA float32 tensor with one entry per row");
  const float* ub = nullptr;
  if (scale_ub.has_value()) {
    check_scalar_scale(*scale_ub, input, "scale_ub");
    ub = scale_ub->data_ptr<float>();
  }
  run_norm_quant(result, input, residual, weight, nullptr, scale.data_ptr<float>(), ub, epsilon);
}

// RMSNorm (+ residual add) with NVFP4 output: `result` holds two e2m1 codes
// per byte ([..., hidden / 2] bytes), `block_scale` one e4m3 byte per 16
// elements (row-major, or the 128 x 4 tiled layout when `swizzled_scales`; any
// dtype, e.g. the int32 buffers engines allocate for it, as long as it is
// contiguous and large enough).
void b200_rms_norm_nvfp4_quant(torch::Tensor result, torch::Tensor block_scale,
                               torch::Tensor input, torch::Tensor weight,
                               torch::Tensor global_scale, double epsilon,
                               c10::optional<torch::Tensor> residual, bool swizzled_scales) {
  check_activation_and_weight(input, weight);
  const int64_t hidden = input.size(-1);
  const int64_t rows = hidden == 0 ? 0 : input.numel() / hidden;
  TORCH_CHECK(hidden % 16 == 0, "NVFP4 needs hidden_size to be a multiple of 16");
  TORCH_CHECK(result.is_cuda() && result.is_contiguous() &&
                  (result.scalar_type() == torch::kByte ||
                   result.scalar_type() == at::ScalarType::Float4_e2m1fn_x2) &&
                  result.numel() == rows * hidden / 2,
              "result must be a contiguous CUDA uint8 tensor of rows x hidden / 2 bytes");
  const int64_t blocks = hidden / 16;
  const int64_t scale_bytes = swizzled_scales ? (rows + 127) / 128 * 128 * ((blocks + 3) / 4 * 4)
                                              : rows * blocks;
  TORCH_CHECK(block_scale.is_cuda() && block_scale.is_contiguous() &&
                  block_scale.numel() * block_scale.element_size() >= scale_bytes,
              "block_scale must be a contiguous CUDA tensor of at least ", scale_bytes, " bytes");
  check_scalar_scale(global_scale, input, "global_scale");
  TORCH_CHECK(result.device() == input.device() && block_scale.device() == input.device(),
              "all tensors must be on the same CUDA device");
  const void* residual_ptr = nullptr;
  if (residual.has_value()) {
    check_like_input(*residual, input, "residual");
    residual_ptr = residual->data_ptr();
  }
  c10::cuda::CUDAGuard guard(input.device());
  raise_if_failed(sm120n_rms_norm_fp4_quant(
      input.data_ptr(), residual_ptr, weight.data_ptr(), const_cast<void*>(residual_ptr),
      result.data_ptr(), block_scale.data_ptr(), global_scale.data_ptr<float>(), rows, hidden,
      dtype_code(input), static_cast<float>(epsilon),
      swizzled_scales ? SM120N_SCALES_TILED_128X4 : SM120N_SCALES_ROW_MAJOR, current_stream()));
}

// QKV projection (tensor cores) with the Q/K norm + RoPE + KV store fused
// into the epilogue (fuse_norm) or as a plain GEMM.
void b200_qkv_proj_norm_rope_cache(torch::Tensor hidden, torch::Tensor qkv_weight,
                                   torch::Tensor qkv, int64_t query_heads, int64_t key_heads,
                                   c10::optional<torch::Tensor> query_weight,
                                   c10::optional<torch::Tensor> key_weight,
                                   c10::optional<torch::Tensor> positions,
                                   c10::optional<torch::Tensor> cos_sin_cache,
                                   c10::optional<torch::Tensor> key_cache,
                                   c10::optional<torch::Tensor> value_cache,
                                   c10::optional<torch::Tensor> slot_mapping, double epsilon,
                                   bool fuse_norm) {
  for (const auto* t : {&hidden, &qkv_weight, &qkv}) {
    TORCH_CHECK(t->is_cuda() && t->is_contiguous() && t->scalar_type() == torch::kBFloat16 &&
                    t->dim() == 2 && t->device() == hidden.device(),
                "hidden, qkv_weight and qkv must be contiguous 2-D bf16 CUDA tensors on one device");
  }
  const int64_t n = (query_heads + 2 * key_heads) * 128;
  TORCH_CHECK(qkv_weight.size(0) == n && qkv_weight.size(1) == hidden.size(1),
              "qkv_weight must be [(query_heads + 2 * key_heads) * 128, hidden_size]");
  TORCH_CHECK(qkv.size(0) == hidden.size(0) && qkv.size(1) == n,
              "qkv must be [tokens, (query_heads + 2 * key_heads) * 128]");
  const void* qw = nullptr;
  const void* kw = nullptr;
  const int64_t* pos = nullptr;
  const float* table = nullptr;
  int64_t rope_positions = 0;
  void* kc = nullptr;
  void* vc = nullptr;
  const int32_t* slots = nullptr;
  int64_t cache_slots = 0;
  if (fuse_norm) {
    TORCH_CHECK(query_weight.has_value() && key_weight.has_value() && positions.has_value() &&
                    cos_sin_cache.has_value(),
                "the fused norm needs query_weight, key_weight, positions and cos_sin_cache");
    TORCH_CHECK(query_weight->is_cuda() && key_weight->is_cuda() &&
                    query_weight->scalar_type() == torch::kBFloat16 &&
                    key_weight->scalar_type() == torch::kBFloat16 &&
                    query_weight->numel() == 128 && key_weight->numel() == 128 &&
                    query_weight->is_contiguous() && key_weight->is_contiguous(),
                "Q/K weights must be contiguous bf16 CUDA tensors of 128 elements");
    TORCH_CHECK(positions->is_cuda() && positions->is_contiguous() &&
                    positions->scalar_type() == torch::kInt64 &&
                    positions->numel() == hidden.size(0),
                "positions must be contiguous CUDA int64 with one entry per token");
    TORCH_CHECK(cos_sin_cache->is_cuda() && cos_sin_cache->is_contiguous() &&
                    cos_sin_cache->scalar_type() == torch::kFloat32 &&
                    cos_sin_cache->size(-1) == 128,
                "cos/sin cache must be contiguous CUDA float32 with last dimension 128");
    qw = query_weight->data_ptr();
    kw = key_weight->data_ptr();
    pos = positions->data_ptr<int64_t>();
    table = cos_sin_cache->data_ptr<float>();
    rope_positions = cos_sin_cache->numel() / 128;
    if (key_cache.has_value() || value_cache.has_value()) {
      TORCH_CHECK(key_cache.has_value() && value_cache.has_value() && slot_mapping.has_value(),
                  "a KV store needs key_cache, value_cache and slot_mapping");
      TORCH_CHECK(key_cache->is_cuda() && value_cache->is_cuda() && key_cache->is_contiguous() &&
                      value_cache->is_contiguous() &&
                      key_cache->scalar_type() == torch::kBFloat16 &&
                      key_cache->sizes() == value_cache->sizes() && key_cache->dim() >= 2 &&
                      key_cache->size(-2) == key_heads && key_cache->size(-1) == 128,
                  "KV caches must be contiguous bf16 CUDA tensors ending in [key_heads, 128]");
      TORCH_CHECK(slot_mapping->is_cuda() && slot_mapping->is_contiguous() &&
                      slot_mapping->scalar_type() == torch::kInt &&
                      slot_mapping->numel() == hidden.size(0),
                  "slot_mapping must be contiguous CUDA int32 with one entry per token");
      kc = key_cache->data_ptr();
      vc = value_cache->data_ptr();
      slots = slot_mapping->data_ptr<int32_t>();
      cache_slots = key_heads == 0 ? 0 : key_cache->numel() / (key_heads * 128);
    }
  }
  c10::cuda::CUDAGuard guard(hidden.device());
  raise_if_failed(sm120n_qkv_proj_norm_rope_cache(
      hidden.data_ptr(), qkv_weight.data_ptr(), qkv.data_ptr(), hidden.size(0), hidden.size(1),
      query_heads, key_heads, qw, kw, pos, table, rope_positions, kc, vc, slots, cache_slots,
      static_cast<float>(epsilon), fuse_norm ? 1 : 0, current_stream()));
}

TORCH_LIBRARY(sm120_norm_ext, m) {
  m.def(
      "qk_norm_rope_cache_(Tensor(a!) query, Tensor(b!) key, Tensor? value, "
      "Tensor query_weight, Tensor key_weight, Tensor positions, Tensor cos_sin_cache, "
      "Tensor(c!)? key_cache, Tensor(d!)? value_cache, Tensor? slot_mapping, "
      "Tensor? k_scale, Tensor? v_scale, bool is_neox=True, str kv_cache_layout=\"NHD\", "
      "float epsilon=1e-6) -> ()");
  m.def(
      "rms_norm_static_fp8_quant(Tensor(a!) result, Tensor input, Tensor weight, "
      "Tensor scale, float epsilon) -> ()");
  m.def(
      "fused_add_rms_norm_static_fp8_quant(Tensor(a!) result, Tensor input, "
      "Tensor(b!) residual, Tensor weight, Tensor scale, float epsilon) -> ()");
  m.def(
      "rms_norm_dynamic_per_token_quant(Tensor(a!) result, Tensor input, Tensor weight, "
      "Tensor(b!) scale, float epsilon, Tensor? scale_ub, Tensor(c!)? residual) -> ()");
  m.def(
      "rms_norm_nvfp4_quant(Tensor(a!) result, Tensor(b!) block_scale, Tensor input, "
      "Tensor weight, Tensor global_scale, float epsilon=1e-6, Tensor(c!)? residual=None, "
      "bool swizzled_scales=True) -> ()");
  m.def(
      "qkv_proj_norm_rope_cache_(Tensor hidden, Tensor qkv_weight, Tensor(a!) qkv, "
      "int query_heads, int key_heads, Tensor? query_weight=None, Tensor? key_weight=None, "
      "Tensor? positions=None, Tensor? cos_sin_cache=None, Tensor(b!)? key_cache=None, "
      "Tensor(c!)? value_cache=None, Tensor? slot_mapping=None, float epsilon=1e-6, "
      "bool fuse_norm=True) -> ()");
}

TORCH_LIBRARY_IMPL(sm120_norm_ext, CUDA, m) {
  m.impl("qk_norm_rope_cache_", &b200_qk_norm_rope_cache);
  m.impl("rms_norm_static_fp8_quant", &b200_rms_norm_static_fp8_quant);
  m.impl("fused_add_rms_norm_static_fp8_quant", &b200_fused_add_rms_norm_static_fp8_quant);
  m.impl("rms_norm_dynamic_per_token_quant", &b200_rms_norm_dynamic_per_token_quant);
  m.impl("rms_norm_nvfp4_quant", &b200_rms_norm_nvfp4_quant);
  m.impl("qkv_proj_norm_rope_cache_", &b200_qkv_proj_norm_rope_cache);
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
