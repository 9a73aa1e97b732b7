// device_utils.cuh -- element packs, rounding and reductions shared by the
// B200 normalisation kernels.
//
// Numerics contract (matches the reference's PyTorch oracle on CPU, op by op):
//   * every fp32 product, sum and difference is rounded on its own: the
//     kernels use __fmul_rn / __fadd_rn / __fsub_rn, which the compiler never
//     contracts into an FMA;
//   * inv_rms = 1 / sqrt(sum_sq / n + eps) with correctly rounded divide and
//     square root (__fdiv_rn, __fsqrt_rn), which is how PyTorch's CPU rsqrt
//     and mean evaluate;
//   * fp32 -> bf16 / fp16 conversions round to nearest even.
// The only freedom left is the order of the fp32 sum of squares.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace sm120n {

constexpr int kWarpSize = 32;
constexpr unsigned kFullMask = 0xffffffffu;

// ---------------------------------------------------------------------------
// 16-byte packs. A pack holds kElems elements of T in a uint4; element e sits
// in word e / (4 / sizeof(T)), low half first (little endian).
// ---------------------------------------------------------------------------
template <typename T>
struct Pack;

template <>
struct Pack<float> {
  static constexpr int kElems = 4;
  __device__ __forceinline__ static void to_f32(const uint4& p, float* f) {
    f[0] = __uint_as_float(p.x);
    f[1] = __uint_as_float(p.y);
    f[2] = __uint_as_float(p.z);
    f[3] = __uint_as_float(p.w);
  }
  __device__ __forceinline__ static uint4 from_f32(const float* f) {
    return make_uint4(__float_as_uint(f[0]), __float_as_uint(f[1]),
                      __float_as_uint(f[2]), __float_as_uint(f[3]));
  }
};

template <>
struct Pack<__nv_bfloat16> {
  static constexpr int kElems = 8;
  // bf16 -> fp32 is a 16-bit shift: exact.
  __device__ __forceinline__ static void word_to_f32(uint32_t w, float& lo, float& hi) {
    lo = __uint_as_float(w << 16);
    hi = __uint_as_float(w & 0xffff0000u);
  }
  __device__ __forceinline__ static uint32_t f32_to_word(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);  // .x = lo, .y = hi
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static void to_f32(const uint4& p, float* f) {
    word_to_f32(p.x, f[0], f[1]);
    word_to_f32(p.y, f[2], f[3]);
    word_to_f32(p.z, f[4], f[5]);
    word_to_f32(p.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint4 from_f32(const float* f) {
    return make_uint4(f32_to_word(f[0], f[1]), f32_to_word(f[2], f[3]),
                      f32_to_word(f[4], f[5]), f32_to_word(f[6], f[7]));
  }
};

template <>
struct Pack<__half> {
  static constexpr int kElems = 8;
  __device__ __forceinline__ static void word_to_f32(uint32_t w, float& lo, float& hi) {
    __half2 h = *reinterpret_cast<__half2*>(&w);
    float2 f = __half22float2(h);
    lo = f.x;
    hi = f.y;
  }
  __device__ __forceinline__ static uint32_t f32_to_word(float lo, float hi) {
    __half2 h = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&h);
  }
  __device__ __forceinline__ static void to_f32(const uint4& p, float* f) {
    word_to_f32(p.x, f[0], f[1]);
    word_to_f32(p.y, f[2], f[3]);
    word_to_f32(p.z, f[4], f[5]);
    word_to_f32(p.w, f[6], f[7]);
  }
  __device__ __forceinline__ static uint4 from_f32(const float* f) {
    return make_uint4(f32_to_word(f[0], f[1]), f32_to_word(f[2], f[3]),
                      f32_to_word(f[4], f[5]), f32_to_word(f[6], f[7]));
  }
};

// A pack as element pairs (2i, 2i+1), the operand shape of the sm_100 packed
// fp32x2 instructions (__fadd2_rn / __fmul2_rn / __ffma2_rn: two IEEE
// round-to-nearest-even operations per instruction, each identical to the
// scalar one).
//
// Contraction: a packed product that feeds a packed sum was measured on B200
// to come out as one fused multiply-add (a single rounding), even with
// --fmad=false, unlike the scalar __fmul_rn / __fadd_rn, which are never
// merged. So the packed forms are used only where no sum consumes a product
// (products of products, sums of loaded values, deliberate FMAs), and every
// product-then-sum step uses the scalar intrinsics: product_plus().
__device__ __forceinline__ float2 product_plus(float2 a, float2 b, float2 c) {
  return make_float2(__fadd_rn(__fmul_rn(a.x, b.x), c.x), __fadd_rn(__fmul_rn(a.y, b.y), c.y));
}

template <typename T>
__device__ __forceinline__ void pack_to_pairs(const uint4& p, float2* f) {
  float g[Pack<T>::kElems];
  Pack<T>::to_f32(p, g);
#pragma unroll
  for (int i = 0; i < Pack<T>::kElems / 2; ++i) f[i] = make_float2(g[2 * i], g[2 * i + 1]);
}

template <typename T>
__device__ __forceinline__ uint4 pairs_to_pack(const float2* f) {
  float g[Pack<T>::kElems];
#pragma unroll
  for (int i = 0; i < Pack<T>::kElems / 2; ++i) {
    g[2 * i] = f[i].x;
    g[2 * i + 1] = f[i].y;
  }
  return Pack<T>::from_f32(g);
}

// Adds the squares of n pairs to a pair of accumulators. For 16-bit storage
// types x^2 is exact in fp32, so a packed FMA equals a rounded square followed
// by a rounded add; fp32 inputs round the square on its own.
template <typename T>
__device__ __forceinline__ float2 accumulate_square_pairs(float2 acc, const float2* f, int n) {
#pragma unroll
  for (int i = 0; i < n; ++i) {
    acc = sizeof(T) == 2 ? __ffma2_rn(f[i], f[i], acc) : product_plus(f[i], f[i], acc);
  }
  return acc;
}

// s = round(x + r) for one pack (kAdd; otherwise s = x), returned packed; its
// squares are added to `acc` (a pair of accumulators: even and odd elements).
// The rounded sum is what the reference squares.
template <typename T, bool kAdd>
__device__ __forceinline__ uint4 combine_pack(const uint4& x, const uint4& r, float2& acc) {
  constexpr int kPairs = Pack<T>::kElems / 2;
  float2 f[kPairs];
  pack_to_pairs<T>(x, f);
  uint4 s = x;
  if constexpr (kAdd) {
    float2 g[kPairs];
    pack_to_pairs<T>(r, g);
#pragma unroll
    for (int i = 0; i < kPairs; ++i) f[i] = __fadd2_rn(f[i], g[i]);
    s = pairs_to_pack<T>(f);
    pack_to_pairs<T>(s, f);
  }
  acc = accumulate_square_pairs<T>(acc, f, kPairs);
  return s;
}

// round(round32(s * inv) * w) for one pack: the RMSNorm output y.
template <typename T>
__device__ __forceinline__ uint4 normalise_pack(const uint4& s, const uint4& w, float inv) {
  constexpr int kPairs = Pack<T>::kElems / 2;
  const float2 inv2 = make_float2(inv, inv);
  float2 f[kPairs], g[kPairs];
  pack_to_pairs<T>(s, f);
  pack_to_pairs<T>(w, g);
#pragma unroll
  for (int i = 0; i < kPairs; ++i) f[i] = __fmul2_rn(__fmul2_rn(f[i], inv2), g[i]);
  return pairs_to_pack<T>(f);
}

// Scalar element access for the unaligned fallback kernels.
template <typename T>
struct Scalar;
template <>
struct Scalar<float> {
  __device__ __forceinline__ static float load(const float* p) { return *p; }
  __device__ __forceinline__ static void store(float* p, float v) { *p = v; }
  __device__ __forceinline__ static float round(float v) { return v; }
};
template <>
struct Scalar<__nv_bfloat16> {
  __device__ __forceinline__ static float load(const __nv_bfloat16* p) { return __bfloat162float(*p); }
  __device__ __forceinline__ static void store(__nv_bfloat16* p, float v) { *p = __float2bfloat16_rn(v); }
  __device__ __forceinline__ static float round(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
};
template <>
struct Scalar<__half> {
  __device__ __forceinline__ static float load(const __half* p) { return __half2float(*p); }
  __device__ __forceinline__ static void store(__half* p, float v) { *p = __float2half_rn(v); }
  __device__ __forceinline__ static float round(float v) { return __half2float(__float2half_rn(v)); }
};

// ---------------------------------------------------------------------------
// Global memory access, 16 bytes per thread per instruction.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint4 load16(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}
__device__ __forceinline__ void store16(void* p, const uint4& v) {
  *reinterpret_cast<uint4*>(p) = v;
}

// ---------------------------------------------------------------------------
// Reductions. The butterfly leaves the identical total in every lane of the
// group (fp32 addition is commutative, so both partners compute the same sum).
// ---------------------------------------------------------------------------
template <int kLanes>
__device__ __forceinline__ float group_allreduce_sum(float v) {
#pragma unroll
  for (int offset = kLanes / 2; offset > 0; offset >>= 1) {
    v = __fadd_rn(v, __shfl_xor_sync(kFullMask, v, offset));
  }
  return v;
}

// Block-wide sum with one barrier; `partial` is double buffered by `parity`
// so the next row's writes cannot race this row's reads.
__device__ __forceinline__ float block_allreduce_sum(float v, float (*partial)[kWarpSize],
                                                     int parity) {
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int warp = threadIdx.x / kWarpSize;
  const int warps = blockDim.x / kWarpSize;
  v = group_allreduce_sum<kWarpSize>(v);
  if (lane == 0) partial[parity][warp] = v;
  __syncthreads();
  float total = 0.0f;
  for (int i = 0; i < warps; ++i) total = __fadd_rn(total, partial[parity][i]);
  return total;
}

__device__ __forceinline__ float accumulate_squares(float acc, const float* f, int n) {
#pragma unroll
  for (int i = 0; i < n; ++i) acc = __fadd_rn(acc, __fmul_rn(f[i], f[i]));
  return acc;
}

// 1 / sqrt(sum_sq / n + eps), every step correctly rounded.
__device__ __forceinline__ float inverse_rms(float sum_sq, float n, float eps) {
  return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(sum_sq, n), eps)));
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch (sm_90+). griddepcontrol.wait returns once
// every grid this one depends on has completed and its memory is visible; it
// is a no-op when the kernel was launched without the PDL attribute. Every
// kernel calls it before its first global-memory access.
// ---------------------------------------------------------------------------
__device__ __forceinline__ void wait_for_upstream_grid() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}
__device__ __forceinline__ void release_downstream_grid() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// Bulk asynchronous copies (the TMA engine's untiled mode) into shared memory,
// completion tracked by an mbarrier's transaction count. The source is always
// this GPU's own global memory and each copy lands in the issuing CTA only.
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t shared_address(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbarrier_init(uint64_t* bar, uint32_t arrivals) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(shared_address(bar)),
               "r"(arrivals)
               : "memory");
}

// Makes mbarrier initialisation visible to the asynchronous proxy.
__device__ __forceinline__ void fence_mbarrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

// Orders this thread's earlier shared-memory accesses before later
// asynchronous-proxy accesses (a bulk copy refilling a consumed stage).
__device__ __forceinline__ void fence_async_shared() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// One arrival that also announces `bytes` of incoming transactions.
__device__ __forceinline__ void mbarrier_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(shared_address(bar)),
               "r"(bytes)
               : "memory");
}

// `bytes` (a multiple of 16) from 16-byte-aligned global memory into
// 16-byte-aligned shared memory; completes `bar`'s transactions.
__device__ __forceinline__ void bulk_load(void* smem_dst, const void* gmem_src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(shared_address(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(shared_address(bar))
      : "memory");
}

__device__ __forceinline__ bool mbarrier_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(shared_address(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// Every wait on asynchronous copies is bounded: after this many polls (each
// poll may suspend the thread for a short hardware-defined time, so the bound
// is tens of milliseconds or more, far beyond any real copy) the caller gets
// `false` and must record a fault and stop instead of spinning forever.
constexpr uint32_t kMaxBarrierPolls = 1u << 22;

__device__ __forceinline__ bool mbarrier_wait_bounded(uint64_t* bar, uint32_t parity) {
  for (uint32_t i = 0; i < kMaxBarrierPolls; ++i) {
    if (mbarrier_try_wait(bar, parity)) return true;
  }
  return false;
}

// Non-blocking test of the phase (no suspension, unlike try_wait).
__device__ __forceinline__ bool mbarrier_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t done;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(done)
      : "r"(shared_address(bar)), "r"(parity)
      : "memory");
  return done != 0;
}

// A wait for copies to land with the caller's poll limit (the host passes the
// process-wide limit, sm120n_set_wait_limit). At the default limit it is
// mbarrier_wait_bounded; a lowered limit polls without suspending, so a
// limit of a few polls gives up before any copy from memory can have landed
// (a test of the expiry path). Callers that give up must still drain their
// copies with mbarrier_wait_bounded before leaving.
__device__ __forceinline__ bool mbarrier_wait_limited(uint64_t* bar, uint32_t parity,
                                                      uint32_t polls) {
  if (polls >= kMaxBarrierPolls) return mbarrier_wait_bounded(bar, parity);
  for (uint32_t i = 0; i < polls; ++i) {
    if (mbarrier_test_wait(bar, parity)) return true;
  }
  return false;
}

// Asks L2 for `bytes` (a multiple of 16) at 16-byte-aligned global `p`; no
// data is returned and nothing waits for it. Kernels issue these for inputs
// before waiting for the upstream grid (programmatic dependent launch): a
// prefetch may precede that wait because L2 stays coherent with whatever the
// upstream grid writes, and every load that uses the data comes after it.
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// The same for the 128-byte line holding `p` (any alignment).
__device__ __forceinline__ void prefetch_l2_line(const void* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p) : "memory");
}

// Row kernels (arguments with input / residual / weight / rows / hidden, rows
// 16-byte aligned): before waiting for the upstream grid a block asks L2 for
// its first row of input and residual, and block 0 for the weight (one
// requester: a weight prefetch from every block measured slower on 1024-row
// calls). On the 48-call fused add + RMSNorm sweep: 110.7 us per step against
// 136.3 us without.
//
// prefetch_first_rows also asks for the block's second row (`next`, the row
// of its second pass), whose loads otherwise wait a full HBM round trip after
// the first pass: 1024 x 4096 bf16 (592 blocks, 432 of them with two rows)
// 7.15-7.27 us against 7.83-7.89, the sweep 110.4-110.6 us per step against
// 112.5-112.6.
template <typename T, bool kAdd, typename Args>
__device__ __forceinline__ void prefetch_first_rows(const Args& a, int64_t row, int64_t next) {
  if (threadIdx.x >= 5) return;
  const int64_t r = threadIdx.x < 3 ? row : next;
  if (r >= a.rows) return;
  const uint32_t bytes = static_cast<uint32_t>(a.hidden) * sizeof(T);
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) prefetch_l2(a.weight, bytes);
  } else if (threadIdx.x == 1 || threadIdx.x == 3) {
    prefetch_l2(a.input + r * a.hidden, bytes);
  } else if (kAdd) {
    prefetch_l2(a.residual + r * a.hidden, bytes);
  }
}

template <typename T, bool kAdd, typename Args>
__device__ __forceinline__ void prefetch_first_row(const Args& a, int64_t row) {
  if (threadIdx.x >= 3 || row >= a.rows) return;
  const uint32_t bytes = static_cast<uint32_t>(a.hidden) * sizeof(T);
  if (threadIdx.x == 0) {
    if (blockIdx.x == 0) prefetch_l2(a.weight, bytes);
  } else if (threadIdx.x == 1) {
    prefetch_l2(a.input + row * a.hidden, bytes);
  } else if (kAdd) {
    prefetch_l2(a.residual + row * a.hidden, bytes);
  }
}

__device__ __forceinline__ uint4 load16_shared(const void* p) {
  return *reinterpret_cast<const uint4*>(p);
}

}  // namespace sm120n
