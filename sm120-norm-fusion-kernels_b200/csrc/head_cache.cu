// head_cache.cu -- generalised per-head Q/K RMSNorm + RoPE + paged KV store
// for B200 (sm_100a); C-ABI entry point sm120n_qk_norm_rope_cache.
//
// Generalises the reference's fused_qk_rms_norm_rope_kv_cuda (reference
// project, csrc/rmsnorm_kernels.cu:611-709, math of sm120_rmsnorm/
// reference.py:27-49) along the axes an inference engine needs:
//   * head sizes 64, 128 and 256, and partial rotary (the first rotary_dim
//     elements rotated, the rest normalised only);
//   * half-split (NEOX) or interleaved rotation pairs;
//   * Q, K and V as strided token rows, e.g. views into one QKV projection
//     output, updated in place without a gather;
//   * paged caches of any block size and stride order (NHD, HND, or K and V
//     interleaved per block), stored in the activation dtype or as fp8 e4m3
//     with per-tensor scales.
//
// Work unit: one head of one token, owned by D/16 lanes (4, 8 or 16). Every
// lane holds two 8-element chunks (one 16-byte access each for 16-bit types):
//   NEOX, lane p < R/16:        chunks at 8p and R/2 + 8p -- rotation partners
//   INTERLEAVED, lane p < R/16: chunks at 16p and 16p + 8 -- pairs inside each
//   lane p >= R/16:             chunks at 16p and 16p + 8 -- passed through
// so the rotation never exchanges data between lanes, and both styles read
// cos/sin entries [8p, 8p + 8) of the position's row. The only cross-lane
// step is the butterfly over the sum of squares. Units are flattened over
// (token, head) on a persistent 1-D grid.
#include <cuda_fp8.h>

#include <algorithm>

#include "head_utils.cuh"
#include "runtime.h"

namespace sm120n {
namespace {

enum CacheKind : int { kNoCache = 0, kSameType = 1, kFp8 = 2 };

template <typename T>
struct CacheArgs {
  T* query;
  T* key;
  const T* value;
  int64_t query_stride;  // elements between consecutive tokens
  int64_t key_stride;
  int64_t value_stride;
  const T* query_weight;
  const T* key_weight;
  const int64_t* positions;
  const float* cos_sin;  // [rope_positions, rotary_dim]
  int64_t rope_positions;
  void* key_cache;
  void* value_cache;
  const int32_t* slots;
  int64_t block_stride;  // cache elements
  int64_t slot_stride;
  int64_t head_stride;
  uint32_t block_size;
  int64_t cache_slots;  // num_blocks * block_size
  const float* k_scale;
  const float* v_scale;
  int64_t tokens;
  int query_heads;
  int key_heads;
  int rotary_dim;
  int cache_kind;
  bool interleaved;
  float epsilon;
  HeadDivisor heads_div;
};

// Interleaved rotation of one chunk: pairs (2i, 2i+1) for i < 4 with cos/sin
// entries c[i], s[i]: y0 = x0*c - x1*s, y1 = x1*c + x0*s, every product and
// sum rounded on its own.
template <typename T>
__device__ __forceinline__ Half8<T> rotate_interleaved(const Half8<T>& n, const float* c,
                                                       const float* s) {
  float2 f[4], y[4];
  unpack_pairs<T>(n, f);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float x1s = __fmul_rn(f[i].y, s[i]);
    const float x0s = __fmul_rn(f[i].x, s[i]);
    y[i] = product_plus(f[i], make_float2(c[i], c[i]), make_float2(-x1s, x0s));
  }
  return pack_pairs<T>(y);
}

// Eight fp8 e4m3 bytes sat(x / scale) of a chunk, element 0 in the low byte.
template <typename T>
__device__ __forceinline__ uint2 chunk_to_fp8(const Half8<T>& h, float scale) {
  float2 f[4];
  unpack_pairs<T>(h, f);
  uint32_t b[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 q = make_float2(__fdiv_rn(f[i].x, scale), __fdiv_rn(f[i].y, scale));
    b[i] = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3));
  }
  return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
}

template <bool kVector>
__device__ __forceinline__ void store_fp8_chunk(uint8_t* p, uint2 v) {
  if constexpr (kVector) {
    *reinterpret_cast<uint2*>(p) = v;
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) p[i] = static_cast<uint8_t>(v.x >> (8 * i));
#pragma unroll
    for (int i = 0; i < 4; ++i) p[4 + i] = static_cast<uint8_t>(v.y >> (8 * i));
  }
}

// kFullNeox: rotary over the whole head with NEOX (half-split) pairs, the
// common case, with the rotary width and pairing fixed at compile time. With
// them known the compiler keeps the kernel within the five-blocks-per-SM
// register budget without the spills of the general form (same box, strided
// QKV views, bf16 NHD cache: the 32768-token 64/8 prefill 242.5 us against
// 262.4, decode B = 1024 32/8 6.95 against 7.74; fp8 cache 242.1 / 8.63
// against 262.4 / 9.26).
template <typename T, int D, int kCache, bool kVector, bool kFullNeox>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? 5 : 2) head_cache_kernel(CacheArgs<T> a) {
  constexpr int kLanes = D / (2 * kChunkElems);
  const int rotary = kFullNeox ? D : a.rotary_dim;
  constexpr int kHeadsPerWarp = kWarpSize / kLanes;
  {
    // Before waiting for the upstream grid, ask L2 for the Q / K / V rows of
    // the tokens in this block's first two passes (threads 0-4 and 5-9) and
    // their positions and slots.
    const uint32_t heads = static_cast<uint32_t>(a.query_heads + a.key_heads);
    const uint32_t units = static_cast<uint32_t>(a.tokens) * heads;
    const uint32_t per_block = (blockDim.x / kWarpSize) * kHeadsPerWarp;
    const uint32_t pass = threadIdx.x / 5;
    const uint32_t role = threadIdx.x - pass * 5;
    const uint64_t first_unit =
        (static_cast<uint64_t>(blockIdx.x) + static_cast<uint64_t>(pass) * gridDim.x) * per_block;
    if (pass < 2 && first_unit < units) {
      const uint32_t first = static_cast<uint32_t>(first_unit);
      const uint32_t last = min(units, first + per_block) - 1;
      const uint32_t t0 = divide(a.heads_div, first);
      const uint32_t t1 = divide(a.heads_div, last);
      if (kVector && role < 3) {
        const int count_heads = role == 0 ? a.query_heads : a.key_heads;
        const T* base = role == 0 ? a.query : role == 1 ? a.key : a.value;
        const int64_t stride = role == 0 ? a.query_stride
                             : role == 1 ? a.key_stride : a.value_stride;
        if (count_heads > 0 && (role < 2 || kCache != kNoCache)) {
          for (uint32_t t = t0; t <= t1; ++t) {
            prefetch_l2(base + static_cast<int64_t>(t) * stride,
                        static_cast<uint32_t>(count_heads) * D * sizeof(T));
          }
        }
      } else if (role == 3) {
        prefetch_l2_line(a.positions + t0);
      } else if (role == 4 && kCache != kNoCache) {
        prefetch_l2_line(a.slots + t0);
      }
    }
    // The cos/sin rows of the first and last token of those two passes, from
    // four lanes of the block's last warp, as in head_norm_rope_kernel: the
    // position is read before the wait only to form an L2 request (bounds-
    // checked; a stale value wastes the request, nothing else). Rows are
    // 16-byte aligned on the vector path (rotary_dim is a multiple of 16).
    const uint32_t lane_in_last = threadIdx.x - kWarpSize * (blockDim.x / kWarpSize - 1);
    if (kVector && blockDim.x >= 2 * kWarpSize && lane_in_last < 4) {
      const uint64_t pass_unit = (static_cast<uint64_t>(blockIdx.x) +
                                  static_cast<uint64_t>(lane_in_last / 2) * gridDim.x) * per_block;
      if (pass_unit < units) {
        const uint32_t first = static_cast<uint32_t>(pass_unit);
        const uint32_t t0 = divide(a.heads_div, first);
        const uint32_t t = lane_in_last % 2 == 0 ? t0
                           : divide(a.heads_div, min(units, first + per_block) - 1);
        if (lane_in_last % 2 == 0 || t != t0) {
          const int64_t position = a.positions[t];
          if (position >= 0 && position < a.rope_positions) {
            prefetch_l2(a.cos_sin + position * rotary,
                        static_cast<uint32_t>(rotary) * sizeof(float));
          }
        }
      }
    }
  }
  wait_for_upstream_grid();
  release_downstream_grid();
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int part = lane % kLanes;
  const int head_in_warp = lane / kLanes;
  const bool rotates = kFullNeox || part < rotary / (2 * kChunkElems);
  const bool split = kFullNeox || (rotates && !a.interleaved);
  const int off_a = split ? part * kChunkElems : part * 2 * kChunkElems;
  const int off_b = split ? rotary / 2 + part * kChunkElems : off_a + kChunkElems;
  const int trig = part * kChunkElems;  // cos at [trig, trig + 8), sin R/2 further

  const uint32_t heads = static_cast<uint32_t>(a.query_heads + a.key_heads);
  const uint32_t units = static_cast<uint32_t>(a.tokens) * heads;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarpSize;
  const uint32_t warps = (gridDim.x * blockDim.x) / kWarpSize;

  float k_scale = 1.0f, v_scale = 1.0f;
  if constexpr (kCache == kFp8) {
    k_scale = *a.k_scale;
    v_scale = *a.v_scale;
  }

  for (uint32_t first = warp * kHeadsPerWarp; first < units; first += warps * kHeadsPerWarp) {
    const uint32_t unit = first + head_in_warp;
    const bool active = unit < units;
    const uint32_t token = active ? divide(a.heads_div, unit) : 0;
    const int h = active ? static_cast<int>(unit - token * heads) : 0;
    const bool is_query = h < a.query_heads;
    const int kv_head = h - a.query_heads;
    T* head = is_query ? a.query + static_cast<int64_t>(token) * a.query_stride +
                             static_cast<int64_t>(h) * D
                       : a.key + static_cast<int64_t>(token) * a.key_stride +
                             static_cast<int64_t>(kv_head) * D;
    Half8<T> x_a{}, x_b{}, v_a{}, v_b{};
    int64_t position = -1;
    int64_t slot = -1;
    if (active) {
      x_a = load_half<T, kVector>(head + off_a);
      x_b = load_half<T, kVector>(head + off_b);
      position = a.positions[token];
      if (kCache != kNoCache && !is_query) {
        slot = a.slots[token];
        // Same-type caches read V whatever the slot holds, so that no load
        // waits on the slot (B = 1024 decode, bf16 cache: 8.24 us against
        // 8.52); fp8 caches keep the V registers free until the slot is known
        // (read unconditionally, the general form spills and the 32768-token
        // prefill loses 1.5%; the whole-head NEOX form does not spill but its
        // prefill still loses 2.3%, 247.6 against 242.1 us, while its B = 1024
        // decode gains 1%). The store below checks the slot's range itself.
        if (kCache == kSameType || (slot >= 0 && slot < a.cache_slots)) {
          const T* vh = a.value + static_cast<int64_t>(token) * a.value_stride +
                        static_cast<int64_t>(kv_head) * D;
          v_a = load_half<T, kVector>(vh + off_a);
          v_b = load_half<T, kVector>(vh + off_b);
        } else {
          slot = -1;
        }
      }
    }
    const float2 acc = half_sum_squares<T>(x_b, half_sum_squares<T>(x_a, make_float2(0.f, 0.f)));
    const float total = group_allreduce_sum<kLanes>(__fadd_rn(acc.x, acc.y));  // before any exit
    if (!active || position < 0 || position >= a.rope_positions) continue;
    const float inv = head_inverse_rms<D>(make_float2(total, 0.0f), a.epsilon);
    // The weights (2 x head_dim elements) stay in L1; loading the selected
    // one per head keeps registers for the loads in flight.
    const T* weight = is_query ? a.query_weight : a.key_weight;
    const Half8<T> n_a = normalise_half<T>(x_a, load_half<T, kVector>(weight + off_a), inv);
    const Half8<T> n_b = normalise_half<T>(x_b, load_half<T, kVector>(weight + off_b), inv);
    Half8<T> y_a = n_a, y_b = n_b;
    if (rotates) {
      const float* row = a.cos_sin + position * rotary;
      float2 c[4], s[4];
      load8_pairs<kVector>(row + trig, c);
      load8_pairs<kVector>(row + rotary / 2 + trig, s);
      if (!kFullNeox && a.interleaved) {
        const float cf[8] = {c[0].x, c[0].y, c[1].x, c[1].y, c[2].x, c[2].y, c[3].x, c[3].y};
        const float sf[8] = {s[0].x, s[0].y, s[1].x, s[1].y, s[2].x, s[2].y, s[3].x, s[3].y};
        y_a = rotate_interleaved<T>(n_a, cf, sf);
        y_b = rotate_interleaved<T>(n_b, cf + 4, sf + 4);
      } else {
        rotate_half<T>(n_a, n_b, c, s, y_a, y_b);
      }
    }
    store_half<T, kVector>(head + off_a, y_a);
    store_half<T, kVector>(head + off_b, y_b);
    // (query heads keep slot = -1; every slot outside the cache stores nothing)
    if (kCache != kNoCache && slot >= 0 && slot < a.cache_slots) {
      const uint32_t block = static_cast<uint32_t>(slot) / a.block_size;
      const uint32_t offset = static_cast<uint32_t>(slot) - block * a.block_size;
      const int64_t base = static_cast<int64_t>(block) * a.block_stride +
                           static_cast<int64_t>(offset) * a.slot_stride +
                           static_cast<int64_t>(kv_head) * a.head_stride;
      if constexpr (kCache == kSameType) {
        T* kc = static_cast<T*>(a.key_cache) + base;
        T* vc = static_cast<T*>(a.value_cache) + base;
        store_half<T, kVector>(kc + off_a, y_a);  // same bits as K
        store_half<T, kVector>(kc + off_b, y_b);
        store_half<T, kVector>(vc + off_a, v_a);
        store_half<T, kVector>(vc + off_b, v_b);
      } else {
        uint8_t* kc = static_cast<uint8_t*>(a.key_cache) + base;
        uint8_t* vc = static_cast<uint8_t*>(a.value_cache) + base;
        store_fp8_chunk<kVector>(kc + off_a, chunk_to_fp8<T>(y_a, k_scale));
        store_fp8_chunk<kVector>(kc + off_b, chunk_to_fp8<T>(y_b, k_scale));
        store_fp8_chunk<kVector>(vc + off_a, chunk_to_fp8<T>(v_a, v_scale));
        store_fp8_chunk<kVector>(vc + off_b, chunk_to_fp8<T>(v_b, v_scale));
      }
    }
  }
}

bool aligned_to(const void* p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

template <typename T, int D, int kCache>
int run_cache(CacheArgs<T> a, cudaStream_t stream) {
  const int64_t cache_elem = a.cache_kind == kFp8 ? 1 : sizeof(T);
  // 16-byte activation accesses; 16-byte (same type) or 8-byte (fp8) stores
  // of cache chunks.
  const uintptr_t cache_align = a.cache_kind == kFp8 ? 8 : 16;
  const bool vector =
      aligned16(a.query) && aligned16(a.key) && aligned16(a.query_weight) &&
      aligned16(a.key_weight) && aligned16(a.cos_sin) &&
      (a.query_stride * sizeof(T)) % 16 == 0 && (a.key_stride * sizeof(T)) % 16 == 0 &&
      (a.cache_kind == kNoCache ||
       (aligned16(a.value) && (a.value_stride * sizeof(T)) % 16 == 0 &&
        aligned_to(a.key_cache, cache_align) && aligned_to(a.value_cache, cache_align) &&
        (a.block_stride * cache_elem) % cache_align == 0 &&
        (a.slot_stride * cache_elem) % cache_align == 0 &&
        (a.head_stride * cache_elem) % cache_align == 0));
  const bool full_neox = a.rotary_dim == D && !a.interleaved;
  auto kernel = !vector    ? head_cache_kernel<T, D, kCache, false, false>
                : full_neox ? head_cache_kernel<T, D, kCache, true, true>
                            : head_cache_kernel<T, D, kCache, true, false>;
  constexpr int64_t kHeadsPerWarp = kWarpSize / (D / (2 * kChunkElems));
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  const int64_t heads = a.query_heads + a.key_heads;
  a.heads_div = make_head_divisor(static_cast<uint32_t>(heads));
  // tokens * heads < 2^31 per launch (32-bit unit indices); larger calls are
  // consecutive launches on the stream.
  const int64_t max_tokens = ((int64_t{1} << 31) - 1) / heads;
  const int64_t all_tokens = a.tokens;
  for (int64_t done = 0; done < all_tokens; done += max_tokens) {
    CacheArgs<T> c = a;
    c.tokens = std::min(max_tokens, all_tokens - done);
    c.query = a.query + done * a.query_stride;
    c.key = a.key + done * a.key_stride;
    c.positions = a.positions + done;
    if (a.cache_kind != kNoCache && a.key_heads > 0) {
      c.value = a.value + done * a.value_stride;
      c.slots = a.slots + done;
    }
    const int64_t warps_needed = (c.tokens * heads + kHeadsPerWarp - 1) / kHeadsPerWarp;
    const int64_t threads = std::min<int64_t>(256, warps_needed * kWarpSize);
    int resident = 1;
    rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), static_cast<int>(threads), 0,
                           &resident);
    if (rc != SM120N_OK) return rc;
    const int64_t blocks =
        std::min<int64_t>((warps_needed * kWarpSize + threads - 1) / threads,
                          static_cast<int64_t>(dev.sm_count) * resident);
    rc = launch(kernel, dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1))),
                dim3(static_cast<unsigned>(threads)), 0, stream, c);
    if (rc != SM120N_OK) return rc;
  }
  return SM120N_OK;
}

template <typename T, int D>
int run_cache_kind(const CacheArgs<T>& a, cudaStream_t stream) {
  switch (a.cache_kind) {
    case kNoCache: return run_cache<T, D, kNoCache>(a, stream);
    case kSameType: return run_cache<T, D, kSameType>(a, stream);
    default: return run_cache<T, D, kFp8>(a, stream);
  }
}

template <typename T>
int run_cache_typed(const sm120n_qk_cache_args& in, int cache_kind, cudaStream_t stream) {
  CacheArgs<T> a{};
  a.query = static_cast<T*>(in.query);
  a.key = static_cast<T*>(in.key);
  a.value = static_cast<const T*>(in.value);
  a.query_stride = in.query_token_stride;
  a.key_stride = in.key_token_stride;
  a.value_stride = in.value_token_stride;
  a.query_weight = static_cast<const T*>(in.query_weight);
  a.key_weight = static_cast<const T*>(in.key_weight);
  a.positions = in.positions;
  a.cos_sin = in.cos_sin_cache;
  a.rope_positions = in.rope_positions;
  a.key_cache = in.key_cache;
  a.value_cache = in.value_cache;
  a.slots = in.slot_mapping;
  a.block_stride = in.cache_block_stride;
  a.slot_stride = in.cache_slot_stride;
  a.head_stride = in.cache_head_stride;
  a.block_size = static_cast<uint32_t>(std::max<int64_t>(in.block_size, 1));
  a.cache_slots = cache_kind == kNoCache ? 0 : in.num_blocks * in.block_size;
  a.k_scale = in.k_scale;
  a.v_scale = in.v_scale;
  a.tokens = in.tokens;
  a.query_heads = static_cast<int>(in.query_heads);
  a.key_heads = static_cast<int>(in.key_heads);
  a.rotary_dim = static_cast<int>(in.rotary_dim);
  a.cache_kind = cache_kind;
  a.interleaved = in.rope_style == SM120N_ROPE_INTERLEAVED;
  a.epsilon = in.epsilon;
  switch (in.head_dim) {
    case 64: return run_cache_kind<T, 64>(a, stream);
    case 128: return run_cache_kind<T, 128>(a, stream);
    default: return run_cache_kind<T, 256>(a, stream);
  }
}

int check_cache_args(const sm120n_qk_cache_args* a, int* cache_kind) {
  if (a == nullptr) return fail(SM120N_ERR_INVALID_ARGUMENT, "args must be non-null");
  if (a->struct_size != sizeof(sm120n_qk_cache_args)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "struct_size %u does not match this library's sm120n_qk_cache_args (%zu)",
                a->struct_size, sizeof(sm120n_qk_cache_args));
  }
  if (dtype_size(a->dtype) == 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "supported dtypes are float16, bfloat16, and float32");
  }
  if (a->head_dim != 64 && a->head_dim != 128 && a->head_dim != 256) {
    return fail(SM120N_ERR_UNSUPPORTED, "head_dim must be 64, 128 or 256 (got %lld)",
                static_cast<long long>(a->head_dim));
  }
  if (a->rotary_dim < 16 || a->rotary_dim > a->head_dim || a->rotary_dim % 16 != 0) {
    return fail(SM120N_ERR_UNSUPPORTED,
                "rotary_dim must be a multiple of 16 in [16, head_dim] (got %lld)",
                static_cast<long long>(a->rotary_dim));
  }
  if (a->rope_style != SM120N_ROPE_NEOX && a->rope_style != SM120N_ROPE_INTERLEAVED) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "unknown rope_style %d", a->rope_style);
  }
  if (a->cache_dtype != SM120N_CACHE_AUTO && a->cache_dtype != SM120N_CACHE_FP8_E4M3) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "unknown cache_dtype %d", a->cache_dtype);
  }
  if (a->tokens < 0 || a->query_heads < 0 || a->key_heads < 0 || a->rope_positions < 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "tokens, head counts and rope_positions must be non-negative");
  }
  const int64_t heads = a->query_heads + a->key_heads;
  if (heads > (1 << 20)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "at most 2^20 heads per token are supported");
  }
  if (a->tokens > (int64_t{1} << 40) / std::max<int64_t>(1, heads)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "too many tokens");
  }
  const bool store = a->key_cache != nullptr || a->value_cache != nullptr;
  *cache_kind = !store ? kNoCache : a->cache_dtype == SM120N_CACHE_FP8_E4M3 ? kFp8 : kSameType;
  if (a->tokens == 0 || heads == 0) return SM120N_OK;
  if (a->query_token_stride < a->query_heads * a->head_dim ||
      a->key_token_stride < a->key_heads * a->head_dim) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "token strides must cover heads * head_dim elements (rows may not overlap)");
  }
  if ((a->query_heads > 0 && !a->query) || (a->key_heads > 0 && !a->key) || !a->query_weight ||
      !a->key_weight || !a->positions || !a->cos_sin_cache) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "tensor pointers must be non-null");
  }
  if (store) {
    if (!a->key_cache || !a->value_cache) {
      return fail(SM120N_ERR_INVALID_ARGUMENT, "key_cache and value_cache go together");
    }
    if (a->key_heads > 0 && (!a->value || !a->slot_mapping)) {
      return fail(SM120N_ERR_INVALID_ARGUMENT, "a KV store needs value and slot_mapping");
    }
    if (a->value_token_stride < a->key_heads * a->head_dim) {
      return fail(SM120N_ERR_INVALID_ARGUMENT,
                  "token strides must cover heads * head_dim elements (rows may not overlap)");
    }
    if (a->num_blocks < 0 || a->block_size < 1 || a->block_size > INT32_MAX ||
        a->cache_block_stride < 0 || a->cache_slot_stride < 0 || a->cache_head_stride < 0) {
      return fail(SM120N_ERR_INVALID_ARGUMENT,
                  "cache geometry must have num_blocks >= 0, block_size >= 1 and "
                  "non-negative strides");
    }
    if (a->num_blocks > (int64_t{1} << 31) / a->block_size) {
      return fail(SM120N_ERR_INVALID_ARGUMENT, "num_blocks * block_size must be at most 2^31");
    }
    if (*cache_kind == kFp8 && (!a->k_scale || !a->v_scale)) {
      return fail(SM120N_ERR_INVALID_ARGUMENT, "fp8 caches need k_scale and v_scale");
    }
  }
  return SM120N_OK;
}

}  // namespace
}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_qk_norm_rope_cache(const sm120n_qk_cache_args* args, void* stream) {
  clear_error();
  int cache_kind = kNoCache;
  int rc = check_cache_args(args, &cache_kind);
  if (rc != SM120N_OK) return rc;
  if (args->tokens == 0 || args->query_heads + args->key_heads == 0) return SM120N_OK;
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (args->dtype) {
    case SM120N_F32: return run_cache_typed<float>(*args, cache_kind, s);
    case SM120N_F16: return run_cache_typed<__half>(*args, cache_kind, s);
    default: return run_cache_typed<__nv_bfloat16>(*args, cache_kind, s);
  }
}
