// head_norm_rope.cu -- per-head Q/K RMSNorm + half-split RoPE, optionally
// fused with the paged KV-cache store, for B200 (sm_100a); C-ABI entry points.
//
// Reference behaviour (paths in the reference project):
//   sm120_rmsnorm/reference.py:27-49   the math: norm in fp32, round to the
//                                      activation dtype, times weight, round
//                                      again, RoPE in fp32, round
//   csrc/rmsnorm_kernels.cu:539-609    fused_qk_rms_norm_rope_cuda
//   csrc/rmsnorm_kernels.cu:611-709    fused_qk_rms_norm_rope_kv_cuda, whose
//                                      KV store (:425-435) copies rotated K
//                                      and V into slot `slot_mapping[t]` and
//                                      skips negative slots
//
// Work unit: one 128-wide head of one token. Eight lanes own a head; lane j
// holds elements [8j, 8j+8) and [64+8j, 64+8j+8), which are exactly each
// other's RoPE partners, so the rotation needs no data exchange and the only
// cross-lane traffic is a three-step shuffle for the sum of squares. For
// 16-bit types each half is one 16-byte load per lane. A warp carries four
// heads; heads of one token are adjacent, so the 512-byte cos/sin row is
// fetched from HBM once and then served from L1. Units are flattened over
// (token, head) on a 1-D grid: no limit on the token count.
//
// Out-of-range indices: a token whose position is outside [0, rope_positions)
// is left untouched (the reference kernel would read out of bounds); a slot
// outside [0, cache_slots) stores nothing (the reference skips slot < 0 only).
#include <algorithm>
#include <type_traits>

#include "device_utils.cuh"
#include "runtime.h"

namespace sm120n {
namespace {

constexpr int kHeadDim = 128;
constexpr int kHalf = kHeadDim / 2;
constexpr int kLanesPerHead = 8;
constexpr int kElemsPerHalf = kHalf / kLanesPerHead;  // 8 per lane per half
constexpr int kHeadsPerWarp = kWarpSize / kLanesPerHead;

template <typename T>
struct HeadArgs {
  T* query;
  T* key;
  const T* value;  // KV variant only
  const T* query_weight;
  const T* key_weight;
  const int64_t* positions;
  const float* cos_sin;
  T* key_cache;    // KV variant only
  T* value_cache;  // KV variant only
  const int32_t* slots;  // KV variant only
  int64_t tokens;
  int query_heads;
  int key_heads;
  int64_t rope_positions;
  int64_t cache_slots;
  float epsilon;
};

// Eight consecutive elements as fp32: two 16-byte loads for fp32, one for
// 16-bit types; element at a time when kVector is false (unaligned buffers).
template <typename T, bool kVector>
__device__ __forceinline__ void load8(const T* p, float* f) {
  if constexpr (kVector) {
    using P = Pack<T>;
#pragma unroll
    for (int i = 0; i < kElemsPerHalf / P::kElems; ++i) P::to_f32(load16(p + i * P::kElems), f + i * P::kElems);
  } else {
#pragma unroll
    for (int i = 0; i < kElemsPerHalf; ++i) f[i] = Scalar<T>::load(p + i);
  }
}

// Raw copy of eight elements (bit-exact V store).
template <typename T, bool kVector>
struct Raw8 {
  static constexpr int kWords = kVector ? (kElemsPerHalf * sizeof(T) / 16) : kElemsPerHalf;
  using Word = typename std::conditional<kVector, uint4, T>::type;
  Word w[kWords];
  __device__ __forceinline__ void load(const T* p) {
#pragma unroll
    for (int i = 0; i < kWords; ++i) w[i] = reinterpret_cast<const Word*>(p)[i];
  }
  __device__ __forceinline__ void store(T* p) const {
#pragma unroll
    for (int i = 0; i < kWords; ++i) reinterpret_cast<Word*>(p)[i] = w[i];
  }
};

// Eight fp32 values rounded to T and stored; `bits` keeps the stored
// encoding so the KV-cache copy is the identical bit pattern.
template <typename T, bool kVector>
__device__ __forceinline__ void store8(T* p, const float* f) {
  if constexpr (kVector) {
    using P = Pack<T>;
#pragma unroll
    for (int i = 0; i < kElemsPerHalf / P::kElems; ++i) store16(p + i * P::kElems, P::from_f32(f + i * P::kElems));
  } else {
#pragma unroll
    for (int i = 0; i < kElemsPerHalf; ++i) Scalar<T>::store(p + i, f[i]);
  }
}

__device__ __forceinline__ void load8_f32(const float* p, float* f, bool vector) {
  if (vector) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = a.x; f[1] = a.y; f[2] = a.z; f[3] = a.w;
    f[4] = b.x; f[5] = b.y; f[6] = b.z; f[7] = b.w;
  } else {
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = p[i];
  }
}

template <typename T, bool kStoreKV, bool kVector>
__global__ void __launch_bounds__(256) head_norm_rope_kernel(HeadArgs<T> a) {
  using S = Scalar<T>;
  wait_for_upstream_grid();
  release_downstream_grid();
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int part = lane % kLanesPerHead;       // position of this lane in its head
  const int head_in_warp = lane / kLanesPerHead;
  const int lo = part * kElemsPerHalf;         // first-half elements [lo, lo + 8)
  const int hi = kHalf + lo;                   // partners            [hi, hi + 8)
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) / kWarpSize;
  const int64_t warps = (static_cast<int64_t>(gridDim.x) * blockDim.x) / kWarpSize;
  const int heads = a.query_heads + a.key_heads;
  const int64_t units = a.tokens * heads;

  float qw_lo[kElemsPerHalf], qw_hi[kElemsPerHalf], kw_lo[kElemsPerHalf], kw_hi[kElemsPerHalf];
  load8<T, kVector>(a.query_weight + lo, qw_lo);
  load8<T, kVector>(a.query_weight + hi, qw_hi);
  load8<T, kVector>(a.key_weight + lo, kw_lo);
  load8<T, kVector>(a.key_weight + hi, kw_hi);

  for (int64_t first = warp * kHeadsPerWarp; first < units; first += warps * kHeadsPerWarp) {
    const int64_t unit = first + head_in_warp;
    const bool active = unit < units;
    const int64_t token = active ? unit / heads : 0;
    const int h = active ? static_cast<int>(unit - token * heads) : 0;
    const bool is_query = h < a.query_heads;
    const int kv_head = h - a.query_heads;
    T* head = is_query ? a.query + (token * a.query_heads + h) * kHeadDim
                       : a.key + (token * a.key_heads + kv_head) * kHeadDim;

    float x_lo[kElemsPerHalf], x_hi[kElemsPerHalf];
    int64_t position = -1;
    int64_t slot = -1;
    Raw8<T, kVector> v_lo, v_hi;
    if (active) {
      load8<T, kVector>(head + lo, x_lo);
      load8<T, kVector>(head + hi, x_hi);
      position = a.positions[token];
      if constexpr (kStoreKV) {
        if (!is_query) {
          slot = a.slots[token];
          if (slot >= 0 && slot < a.cache_slots) {
            const T* vh = a.value + (token * a.key_heads + kv_head) * kHeadDim;
            v_lo.load(vh + lo);
            v_hi.load(vh + hi);
          } else {
            slot = -1;
          }
        }
      }
    } else {
#pragma unroll
      for (int i = 0; i < kElemsPerHalf; ++i) x_lo[i] = x_hi[i] = 0.0f;
    }

    float sum_sq = accumulate_squares(0.0f, x_lo, kElemsPerHalf);
    sum_sq = accumulate_squares(sum_sq, x_hi, kElemsPerHalf);
    sum_sq = group_allreduce_sum<kLanesPerHead>(sum_sq);
    if (!active || position < 0 || position >= a.rope_positions) continue;
    const float inv = inverse_rms(sum_sq, static_cast<float>(kHeadDim), a.epsilon);

    // n = round(round(x * inv) * w): RMSNorm rounded to the activation dtype,
    // then the weight multiply in that dtype (reference.py:38-41).
    float n_lo[kElemsPerHalf], n_hi[kElemsPerHalf];
#pragma unroll
    for (int i = 0; i < kElemsPerHalf; ++i) {
      const float w_lo = is_query ? qw_lo[i] : kw_lo[i];
      const float w_hi = is_query ? qw_hi[i] : kw_hi[i];
      n_lo[i] = S::round(__fmul_rn(S::round(__fmul_rn(x_lo[i], inv)), w_lo));
      n_hi[i] = S::round(__fmul_rn(S::round(__fmul_rn(x_hi[i], inv)), w_hi));
    }

    float c[kElemsPerHalf], s[kElemsPerHalf];
    const float* row = a.cos_sin + position * kHeadDim;
    load8_f32(row + lo, c, kVector);
    load8_f32(row + hi, s, kVector);
    float y_lo[kElemsPerHalf], y_hi[kElemsPerHalf];
#pragma unroll
    for (int i = 0; i < kElemsPerHalf; ++i) {
      y_lo[i] = __fsub_rn(__fmul_rn(n_lo[i], c[i]), __fmul_rn(n_hi[i], s[i]));
      y_hi[i] = __fadd_rn(__fmul_rn(n_hi[i], c[i]), __fmul_rn(n_lo[i], s[i]));
    }
    store8<T, kVector>(head + lo, y_lo);
    store8<T, kVector>(head + hi, y_hi);
    if constexpr (kStoreKV) {
      if (slot >= 0) {
        T* kc = a.key_cache + (slot * a.key_heads + kv_head) * kHeadDim;
        T* vc = a.value_cache + (slot * a.key_heads + kv_head) * kHeadDim;
        store8<T, kVector>(kc + lo, y_lo);  // same rounding -> same bits as K
        store8<T, kVector>(kc + hi, y_hi);
        v_lo.store(vc + lo);
        v_hi.store(vc + hi);
      }
    }
  }
}

// threads_per_block == 0 selects the B200 default: up to 256 threads and a
// persistent grid capped at what is resident on the device.
template <typename T, bool kStoreKV>
int run_heads(const HeadArgs<T>& a, int threads_per_block, cudaStream_t stream) {
  const bool vector = aligned16(a.query) && aligned16(a.key) && aligned16(a.query_weight) &&
                      aligned16(a.key_weight) && aligned16(a.cos_sin) &&
                      (!kStoreKV || (aligned16(a.value) && aligned16(a.key_cache) &&
                                     aligned16(a.value_cache)));
  auto kernel = vector ? head_norm_rope_kernel<T, kStoreKV, true>
                       : head_norm_rope_kernel<T, kStoreKV, false>;
  const int64_t units = a.tokens * (a.query_heads + a.key_heads);
  const int64_t warps_needed = (units + kHeadsPerWarp - 1) / kHeadsPerWarp;
  int64_t threads = threads_per_block;
  int64_t blocks;
  if (threads == 0) {
    threads = std::min<int64_t>(256, warps_needed * kWarpSize);
    blocks = (warps_needed * kWarpSize + threads - 1) / threads;
    DeviceInfo dev;
    int rc = current_device_info(&dev);
    if (rc != SM120N_OK) return rc;
    int resident = 1;
    rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), static_cast<int>(threads), 0,
                           &resident);
    if (rc != SM120N_OK) return rc;
    blocks = std::min<int64_t>(blocks, static_cast<int64_t>(dev.sm_count) * resident);
  } else {
    blocks = (warps_needed * kWarpSize + threads - 1) / threads;
    blocks = std::min<int64_t>(blocks, int64_t{1} << 30);
  }
  return launch(kernel, dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1))),
                dim3(static_cast<unsigned>(threads)), 0, stream, a);
}

template <bool kStoreKV>
int run_heads_typed(int dtype, void* query, void* key, const void* value,
                    const void* query_weight, const void* key_weight, const int64_t* positions,
                    const float* cos_sin, void* key_cache, void* value_cache,
                    const int32_t* slots, int64_t tokens, int64_t query_heads,
                    int64_t key_heads, int64_t rope_positions, int64_t cache_slots,
                    float epsilon, int threads_per_block, cudaStream_t stream) {
  auto make = [&](auto* tag) {
    using T = std::remove_pointer_t<decltype(tag)>;
    return HeadArgs<T>{static_cast<T*>(query), static_cast<T*>(key),
                       static_cast<const T*>(value), static_cast<const T*>(query_weight),
                       static_cast<const T*>(key_weight), positions, cos_sin,
                       static_cast<T*>(key_cache), static_cast<T*>(value_cache), slots, tokens,
                       static_cast<int>(query_heads), static_cast<int>(key_heads),
                       rope_positions, cache_slots, epsilon};
  };
  switch (dtype) {
    case SM120N_F32:
      return run_heads<float, kStoreKV>(make(static_cast<float*>(nullptr)), threads_per_block, stream);
    case SM120N_F16:
      return run_heads<__half, kStoreKV>(make(static_cast<__half*>(nullptr)), threads_per_block, stream);
    default:
      return run_heads<__nv_bfloat16, kStoreKV>(make(static_cast<__nv_bfloat16*>(nullptr)),
                                                threads_per_block, stream);
  }
}

int check_heads(int64_t tokens, int64_t query_heads, int64_t key_heads, int64_t head_dim,
                int64_t rope_positions, int dtype, const char* head_dim_message) {
  if (dtype_size(dtype) == 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "supported dtypes are float16, bfloat16, and float32");
  }
  if (head_dim != kHeadDim) return fail(SM120N_ERR_UNSUPPORTED, "%s", head_dim_message);
  if (tokens < 0 || query_heads < 0 || key_heads < 0 || rope_positions < 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "tokens, head counts and rope_positions must be non-negative");
  }
  if (query_heads + key_heads > (1 << 20)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "at most 2^20 heads per token are supported");
  }
  if (tokens > (int64_t{1} << 40) / std::max<int64_t>(1, query_heads + key_heads)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "too many tokens");
  }
  return SM120N_OK;
}

}  // namespace
}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_fused_qk_rms_norm_rope(void* query, void* key, const void* query_weight,
                                             const void* key_weight, const int64_t* positions,
                                             const float* cos_sin_cache, int64_t tokens,
                                             int64_t query_heads, int64_t key_heads,
                                             int64_t head_dim, int64_t rope_positions, int dtype,
                                             float epsilon, int version, void* stream) {
  clear_error();
  int rc = check_heads(tokens, query_heads, key_heads, head_dim, rope_positions, dtype,
                       "fused QK Norm+RoPE requires head_dim=128");
  if (rc != SM120N_OK) return rc;
  if (version != 1 && version != 2) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "QK Norm+RoPE version must be 1 or 2");
  }
  if (tokens == 0 || query_heads + key_heads == 0) return SM120N_OK;
  if (!query || !key || !query_weight || !key_weight || !positions || !cos_sin_cache) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "tensor pointers must be non-null");
  }
  // version 2: B200 default launch; version 1: two warps per thread block.
  return run_heads_typed<false>(dtype, query, key, nullptr, query_weight, key_weight, positions,
                                cos_sin_cache, nullptr, nullptr, nullptr, tokens, query_heads,
                                key_heads, rope_positions, 0, epsilon, version == 1 ? 64 : 0,
                                static_cast<cudaStream_t>(stream));
}

extern "C" int sm120n_fused_qk_rms_norm_rope_kv(
    void* query, void* key, const void* value, const void* query_weight, const void* key_weight,
    const int64_t* positions, const float* cos_sin_cache, void* key_cache, void* value_cache,
    const int32_t* slot_mapping, int64_t tokens, int64_t query_heads, int64_t key_heads,
    int64_t head_dim, int64_t rope_positions, int64_t cache_slots, int dtype, float epsilon,
    int version, void* stream) {
  clear_error();
  int rc = check_heads(tokens, query_heads, key_heads, head_dim, rope_positions, dtype,
                       "fused QK Norm+RoPE+KV requires head_dim=128");
  if (rc != SM120N_OK) return rc;
  if (version != 1 && version != 4) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "QK Norm+RoPE+KV version must be 1 or 4 warps per block");
  }
  if (cache_slots < 0) return fail(SM120N_ERR_INVALID_ARGUMENT, "cache_slots must be non-negative");
  if (tokens == 0 || query_heads + key_heads == 0) return SM120N_OK;
  if (!query || !key || !query_weight || !key_weight || !positions || !cos_sin_cache ||
      (key_heads > 0 && (!value || !slot_mapping || (cache_slots > 0 && (!key_cache || !value_cache))))) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "tensor pointers must be non-null");
  }
  // version 1: B200 default launch; version 4: four warps per thread block.
  return run_heads_typed<true>(dtype, query, key, value, query_weight, key_weight, positions,
                               cos_sin_cache, key_cache, value_cache, slot_mapping, tokens,
                               query_heads, key_heads, rope_positions, cache_slots, epsilon,
                               version == 4 ? 128 : 0, static_cast<cudaStream_t>(stream));
}
