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

#include "head_utils.cuh"
#include "runtime.h"

namespace sm120n {
namespace {

constexpr int kHeadDim = 128;
constexpr int kHalf = kHeadDim / 2;
constexpr int kLanesPerHead = 8;
static_assert(kHalf / kLanesPerHead == kChunkElems, "one chunk per lane per half");
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
  // unit -> token division by heads = query_heads + key_heads, for unit
  // indices below 2^31
  HeadDivisor heads_div;
};

// One head of one token, between issuing its loads and finishing it.
template <typename T>
struct HeadJob {
  T* head;
  Half8<T> x_lo, x_hi, v_lo, v_hi;
  int64_t position;  // as loaded; checked in finish, so that no load waits on it
  int32_t slot;      // as loaded (KV variant, key heads)
  int kv_head;
  bool is_query;
  bool active;
};

// kHoistWeights: each lane keeps its chunks of both weights in registers for
// the whole launch (lowest latency: batch-1 decode); otherwise it loads the
// selected weight per head from L1, which frees 16 registers for a fifth
// resident block per SM and more loads in flight (measured on B200 for the
// 32768-token prefill: 244 us against 256 us).
template <typename T, bool kStoreKV, bool kVector, bool kHoistWeights>
__global__ void __launch_bounds__(256, sizeof(T) == 2 ? (kHoistWeights ? 4 : 5) : 2)
    head_norm_rope_kernel(HeadArgs<T> a) {
  {
    // Before waiting for the upstream grid, ask L2 for the heads of this
    // block's first two passes (threads 0-4 and 5-9) and their tokens'
    // position and slot (batch-1 decode: 1.86 us against 2.11 us; B = 1024,
    // where 540 of 740 blocks make a second pass: 7.36 against 7.87 us with
    // the first pass alone). Pass p of block b covers units
    // [(b + p * gridDim.x) * per_block, +per_block) for every block size (the
    // loop below walks warps in that order), so the request matches the
    // block's own pass; a grid that covers all units in one pass (versions 1
    // and 4, small calls) has no pass 1 and skips the request.
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
      const uint32_t count = divide(a.heads_div, last) - t0 + 1;
      if (!kVector) {
        // bulk prefetches need 16-byte-aligned rows
      } else if (role == 0 && a.query_heads > 0) {
        prefetch_l2(a.query + static_cast<int64_t>(t0) * a.query_heads * kHeadDim,
                    count * a.query_heads * kHeadDim * sizeof(T));
      } else if (role == 1 && a.key_heads > 0) {
        prefetch_l2(a.key + static_cast<int64_t>(t0) * a.key_heads * kHeadDim,
                    count * a.key_heads * kHeadDim * sizeof(T));
      } else if (role == 2 && kStoreKV && a.key_heads > 0) {
        prefetch_l2(a.value + static_cast<int64_t>(t0) * a.key_heads * kHeadDim,
                    count * a.key_heads * kHeadDim * sizeof(T));
      }
      if (role == 3) {
        prefetch_l2_line(a.positions + t0);
      } else if (role == 4 && kStoreKV) {
        prefetch_l2_line(a.slots + t0);
      }
    }
    // The cos/sin rows of the first and last token of those two passes, from
    // four lanes of the block's last warp (the first warp's lanes issue the
    // requests above). The position is read before the wait only to form an
    // L2 request: a stale value costs a wasted request, never a wrong result
    // (every load that uses data comes after the wait), and it is
    // bounds-checked before the address is formed. Without this the rows are
    // requested only after the position load that follows the wait: per call
    // in bench.py's graphs (same box) batch-1 decode 1.75-1.81 us against
    // 1.91-2.02, B = 64 2.02-2.05 against 2.35-2.37, B = 256 2.85-2.87
    // against 3.20-3.21, B = 1024 6.86-6.90 against 7.07-7.20; prefills and
    // the no-KV operator at T = 1..256 (positions already in L2) unchanged.
    // (The bulk request needs the 16-byte-aligned table of the vector path.)
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
            prefetch_l2(a.cos_sin + position * kHeadDim, kHeadDim * sizeof(float));
          }
        }
      }
    }
  }
  wait_for_upstream_grid();
  release_downstream_grid();
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int part = lane % kLanesPerHead;       // position of this lane in its head
  const int head_in_warp = lane / kLanesPerHead;
  const int lo = part * kChunkElems;         // first-half elements [lo, lo + 8)
  const int hi = kHalf + lo;                   // partners            [hi, hi + 8)
  // The host splits launches so that tokens * heads < 2^31: unit indices fit
  // in 32 bits and the token of a unit is one 32-bit division.
  const uint32_t heads = static_cast<uint32_t>(a.query_heads + a.key_heads);
  const uint32_t units = static_cast<uint32_t>(a.tokens) * heads;
  const uint32_t warp = (blockIdx.x * blockDim.x + threadIdx.x) / kWarpSize;
  const uint32_t warps = (gridDim.x * blockDim.x) / kWarpSize;

  Half8<T> qw_lo{}, qw_hi{}, kw_lo{}, kw_hi{};
  if constexpr (kHoistWeights) {
    qw_lo = load_half<T, kVector>(a.query_weight + lo);
    qw_hi = load_half<T, kVector>(a.query_weight + hi);
    kw_lo = load_half<T, kVector>(a.key_weight + lo);
    kw_hi = load_half<T, kVector>(a.key_weight + hi);
  }

  auto begin = [&](HeadJob<T>& job, uint32_t unit) {
    job.active = unit < units;
    const uint32_t token = job.active ? divide(a.heads_div, unit) : 0;
    const int h = job.active ? static_cast<int>(unit - token * heads) : 0;
    job.is_query = h < a.query_heads;
    job.kv_head = h - a.query_heads;
    job.head = job.is_query
                   ? a.query + (static_cast<int64_t>(token) * a.query_heads + h) * kHeadDim
                   : a.key + (static_cast<int64_t>(token) * a.key_heads + job.kv_head) * kHeadDim;
    job.position = -1;
    job.slot = -1;
    job.x_lo = Half8<T>{};
    job.x_hi = Half8<T>{};
    if (job.active) {
      job.x_lo = load_half<T, kVector>(job.head + lo);
      job.x_hi = load_half<T, kVector>(job.head + hi);
      job.position = a.positions[token];
      if constexpr (kStoreKV) {
        if (!job.is_query) {
          // V is read whatever the slot holds, so that no load waits on the slot
          job.slot = a.slots[token];
          const T* vh =
              a.value + (static_cast<int64_t>(token) * a.key_heads + job.kv_head) * kHeadDim;
          job.v_lo = load_half<T, kVector>(vh + lo);
          job.v_hi = load_half<T, kVector>(vh + hi);
        }
      }
    }
  };

  auto finish = [&](const HeadJob<T>& job) {
    float2 acc = half_sum_squares<T>(job.x_hi, half_sum_squares<T>(job.x_lo, make_float2(0.f, 0.f)));
    const float lane_sum = __fadd_rn(acc.x, acc.y);
    const float total = group_allreduce_sum<kLanesPerHead>(lane_sum);  // all lanes, before any exit
    if (!job.active || job.position < 0 || job.position >= a.rope_positions) return;
    const float inv = head_inverse_rms<kHeadDim>(make_float2(total, 0.0f), a.epsilon);
    Half8<T> w_lo, w_hi;
    if constexpr (kHoistWeights) {
      w_lo = select_half<T>(job.is_query, qw_lo, kw_lo);
      w_hi = select_half<T>(job.is_query, qw_hi, kw_hi);
    } else {
      const T* weight = job.is_query ? a.query_weight : a.key_weight;
      w_lo = load_half<T, kVector>(weight + lo);
      w_hi = load_half<T, kVector>(weight + hi);
    }
    const Half8<T> n_lo = normalise_half<T>(job.x_lo, w_lo, inv);
    const Half8<T> n_hi = normalise_half<T>(job.x_hi, w_hi, inv);
    float2 c[4], sn[4];
    load8_pairs<kVector>(a.cos_sin + job.position * kHeadDim + lo, c);
    load8_pairs<kVector>(a.cos_sin + job.position * kHeadDim + hi, sn);
    Half8<T> out_lo, out_hi;
    rotate_half<T>(n_lo, n_hi, c, sn, out_lo, out_hi);
    store_half<T, kVector>(job.head + lo, out_lo);
    store_half<T, kVector>(job.head + hi, out_hi);
    if constexpr (kStoreKV) {
      if (!job.is_query && job.slot >= 0 && job.slot < a.cache_slots) {
        const int64_t cache_head =
            (static_cast<int64_t>(job.slot) * a.key_heads + job.kv_head) * kHeadDim;
        store_half<T, kVector>(a.key_cache + cache_head + lo, out_lo);  // same bits as K
        store_half<T, kVector>(a.key_cache + cache_head + hi, out_hi);
        store_half<T, kVector>(a.value_cache + cache_head + lo, job.v_lo);
        store_half<T, kVector>(a.value_cache + cache_head + hi, job.v_hi);
      }
    }
  };

  for (uint32_t first = warp * kHeadsPerWarp; first < units; first += warps * kHeadsPerWarp) {
    HeadJob<T> job;
    begin(job, first + head_in_warp);
    finish(job);
  }
}

// threads_per_block == 0 selects the B200 default: up to 256 threads and a
// persistent grid capped at what is resident on the device.
template <typename T, bool kStoreKV>
int run_heads(HeadArgs<T> a, int threads_per_block, cudaStream_t stream) {
  const bool vector = aligned16(a.query) && aligned16(a.key) && aligned16(a.query_weight) &&
                      aligned16(a.key_weight) && aligned16(a.cos_sin) &&
                      (!kStoreKV || (aligned16(a.value) && aligned16(a.key_cache) &&
                                     aligned16(a.value_cache)));
  const int64_t heads = a.query_heads + a.key_heads;
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  // Below about 2048 heads per launch (decode batches up to ~64) the launch is
  // latency-bound and the hoisted-weight form is faster (batch-1 decode:
  // 2.37 us against 2.48 us); above, occupancy wins. Issuing the next four
  // heads' loads before finishing the current four (two jobs in flight per
  // warp) was measured too and lost: 4 blocks/SM make the 32768-token prefill
  // 267 us against 242 us, 3 blocks/SM 251 us.
  const bool hoist = a.tokens * (a.query_heads + a.key_heads) < 2048;
  auto kernel = vector ? (hoist ? head_norm_rope_kernel<T, kStoreKV, true, true>
                                : head_norm_rope_kernel<T, kStoreKV, true, false>)
                       : (hoist ? head_norm_rope_kernel<T, kStoreKV, false, true>
                                : head_norm_rope_kernel<T, kStoreKV, false, false>);
  const int64_t heads_per_warp = kHeadsPerWarp;
  // Keep tokens * heads below 2^31 per launch (the kernel indexes units in
  // 32 bits); larger calls become consecutive launches on the same stream.
  const int64_t max_tokens = ((int64_t{1} << 31) - 1) / heads;
  const int64_t all_tokens = a.tokens;
  a.heads_div = make_head_divisor(static_cast<uint32_t>(heads));
  for (int64_t done = 0; done < all_tokens; done += max_tokens) {
    HeadArgs<T> c = a;
    c.tokens = std::min(max_tokens, all_tokens - done);
    c.query = a.query + done * a.query_heads * kHeadDim;
    c.key = a.key + done * a.key_heads * kHeadDim;
    c.positions = a.positions + done;
    if constexpr (kStoreKV) {
      c.value = a.value + done * a.key_heads * kHeadDim;
      c.slots = a.slots + done;
    }
    const int64_t units = c.tokens * heads;
    const int64_t warps_needed = (units + heads_per_warp - 1) / heads_per_warp;
    int64_t threads = threads_per_block;
    int64_t blocks;
    if (threads == 0) {
      threads = std::min<int64_t>(256, warps_needed * kWarpSize);
      blocks = (warps_needed * kWarpSize + threads - 1) / threads;
      int resident = 1;
      rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), static_cast<int>(threads), 0,
                             &resident);
      if (rc != SM120N_OK) return rc;
      blocks = std::min<int64_t>(blocks, static_cast<int64_t>(dev.sm_count) * resident);
    } else {
      // At most 2^31 threads, so that the kernel's 32-bit warp index and
      // warp count cannot wrap; the kernel's loop takes any remaining units.
      blocks = std::min<int64_t>((warps_needed * kWarpSize + threads - 1) / threads,
                                 (int64_t{1} << 31) / threads);
    }
    rc = launch(kernel, dim3(static_cast<unsigned>(std::max<int64_t>(blocks, 1))),
                dim3(static_cast<unsigned>(threads)), 0, stream, c);
    if (rc != SM120N_OK) return rc;
  }
  return SM120N_OK;
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
