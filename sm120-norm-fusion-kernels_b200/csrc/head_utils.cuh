// head_utils.cuh -- per-head building blocks shared by the Q/K RMSNorm + RoPE
// kernels: eight-element chunks of a head, their loads and stores, the
// per-head norm with the reference's double rounding, the half-split
// rotation, and the unit -> token division.
//
// Numerics (reference project, sm120_rmsnorm/reference.py:27-49): the norm
// is computed in fp32, rounded to the activation dtype, multiplied by the
// weight in that dtype (rounded again), and RoPE runs in fp32 with every
// product and sum rounded on its own before the final rounding.
#pragma once

#include "device_utils.cuh"

namespace sm120n {

constexpr int kChunkElems = 8;  // elements of a head one lane loads at a time

// Constants for dividing indices below 2^31 by d (1 <= d <= 2^20): with
// l = ceil(log2 d), m = ceil(2^(31+l) / d) satisfies 2^(31+l) <= m*d <=
// 2^(31+l) + 2^l, so floor(n*m / 2^(31+l)) = floor(n / d) (the round-up
// method for division by invariant integers).
struct HeadDivisor {
  uint32_t magic;
  int shift;
  bool pow2;
};

inline HeadDivisor make_head_divisor(uint32_t d) {
  HeadDivisor h{};
  int l = 0;
  while ((uint64_t{1} << l) < d) ++l;
  h.shift = l;
  h.pow2 = (d & (d - 1)) == 0;
  h.magic = h.pow2 ? 0u : static_cast<uint32_t>(((uint64_t{1} << (31 + l)) + d - 1) / d);
  return h;
}

__device__ __forceinline__ uint32_t divide(const HeadDivisor& h, uint32_t n) {
  return h.pow2 ? n >> h.shift : __umulhi(n, h.magic) >> (h.shift - 1);
}

// Eight elements of T as 32-bit words: four words (two elements each) for
// 16-bit types, eight for fp32. Loaded with 16-byte accesses when the buffers
// are aligned (kVector), element at a time otherwise.
template <typename T>
struct Half8 {
  static constexpr int kWords = kChunkElems * sizeof(T) / 4;
  uint32_t w[kWords];
};

template <typename T, bool kVector>
__device__ __forceinline__ Half8<T> load_half(const T* p) {
  Half8<T> h;
  if constexpr (kVector) {
#pragma unroll
    for (int i = 0; i < Half8<T>::kWords / 4; ++i) {
      const uint4 v = load16(p + i * (16 / sizeof(T)));
      h.w[4 * i] = v.x;
      h.w[4 * i + 1] = v.y;
      h.w[4 * i + 2] = v.z;
      h.w[4 * i + 3] = v.w;
    }
  } else if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i) h.w[i] = reinterpret_cast<const uint32_t*>(p)[i];
  } else {
    const uint16_t* q = reinterpret_cast<const uint16_t*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) h.w[i] = uint32_t(q[2 * i]) | (uint32_t(q[2 * i + 1]) << 16);
  }
  return h;
}

template <typename T, bool kVector>
__device__ __forceinline__ void store_half(T* p, const Half8<T>& h) {
  if constexpr (kVector) {
#pragma unroll
    for (int i = 0; i < Half8<T>::kWords / 4; ++i) {
      store16(p + i * (16 / sizeof(T)),
              make_uint4(h.w[4 * i], h.w[4 * i + 1], h.w[4 * i + 2], h.w[4 * i + 3]));
    }
  } else if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int i = 0; i < 8; ++i) reinterpret_cast<uint32_t*>(p)[i] = h.w[i];
  } else {
    uint16_t* q = reinterpret_cast<uint16_t*>(p);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      q[2 * i] = static_cast<uint16_t>(h.w[i] & 0xffffu);
      q[2 * i + 1] = static_cast<uint16_t>(h.w[i] >> 16);
    }
  }
}

// Elements (2i, 2i+1) of a half as float2 number i.
template <typename T>
__device__ __forceinline__ void unpack_pairs(const Half8<T>& h, float2* f) {
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (sizeof(T) == 4) {
      f[i] = make_float2(__uint_as_float(h.w[2 * i]), __uint_as_float(h.w[2 * i + 1]));
    } else {
      Pack<T>::word_to_f32(h.w[i], f[i].x, f[i].y);
    }
  }
}

template <typename T>
__device__ __forceinline__ Half8<T> pack_pairs(const float2* f) {
  Half8<T> h;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    if constexpr (sizeof(T) == 4) {
      h.w[2 * i] = __float_as_uint(f[i].x);
      h.w[2 * i + 1] = __float_as_uint(f[i].y);
    } else {
      h.w[i] = Pack<T>::f32_to_word(f[i].x, f[i].y);
    }
  }
  return h;
}

// Round-to-nearest-even product of two packed pairs. For bf16 and fp16 the
// fp32 product of two such values is exact, so this single rounding equals
// the oracle's round(round_fp32(n * w)).
template <typename T>
__device__ __forceinline__ uint32_t mul_pair_rn(uint32_t a, uint32_t b);
template <>
__device__ __forceinline__ uint32_t mul_pair_rn<__nv_bfloat16>(uint32_t a, uint32_t b) {
  __nv_bfloat162 r = __hmul2_rn(*reinterpret_cast<__nv_bfloat162*>(&a),
                                *reinterpret_cast<__nv_bfloat162*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}
template <>
__device__ __forceinline__ uint32_t mul_pair_rn<__half>(uint32_t a, uint32_t b) {
  __half2 r = __hmul2_rn(*reinterpret_cast<__half2*>(&a), *reinterpret_cast<__half2*>(&b));
  return *reinterpret_cast<uint32_t*>(&r);
}

// Sum of squares of a half into a pair of accumulators (even / odd
// elements). For 16-bit types x^2 is exact in fp32, so a packed FMA equals the
// oracle's rounded square followed by a rounded add; fp32 rounds the square
// on its own.
template <typename T>
__device__ __forceinline__ float2 half_sum_squares(const Half8<T>& h, float2 acc) {
  float2 f[4];
  unpack_pairs<T>(h, f);
  return accumulate_square_pairs<T>(acc, f, 4);
}

// n = round(round(x * inv) * w), the RMSNorm rounded to T and then weighted
// in T (reference.py:38-41).
template <typename T>
__device__ __forceinline__ Half8<T> normalise_half(const Half8<T>& x, const Half8<T>& w,
                                                   float inv) {
  const float2 inv2 = make_float2(inv, inv);
  float2 f[4];
  unpack_pairs<T>(x, f);
  if constexpr (sizeof(T) == 4) {
    float2 g[4];
    unpack_pairs<T>(w, g);
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = __fmul2_rn(__fmul2_rn(f[i], inv2), g[i]);
    return pack_pairs<T>(f);
  } else {
    Half8<T> n;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float2 t = __fmul2_rn(f[i], inv2);
      n.w[i] = mul_pair_rn<T>(Pack<T>::f32_to_word(t.x, t.y), w.w[i]);
    }
    return n;
  }
}

// Half-split rotation of one lane's pairs: lo = n_lo*c - n_hi*s,
// hi = n_hi*c + n_lo*s, each product and sum rounded on its own (the
// subtraction is an add of the negated product, exact under round to nearest
// even; product_plus keeps the first product out of a fused multiply-add).
template <typename T>
__device__ __forceinline__ void rotate_half(const Half8<T>& n_lo, const Half8<T>& n_hi,
                                            const float2* c, const float2* s,
                                            Half8<T>& out_lo, Half8<T>& out_hi) {
  float2 p[4], q[4], y_lo[4], y_hi[4];
  unpack_pairs<T>(n_lo, p);
  unpack_pairs<T>(n_hi, q);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 qs = make_float2(__fmul_rn(q[i].x, s[i].x), __fmul_rn(q[i].y, s[i].y));
    const float2 ps = make_float2(__fmul_rn(p[i].x, s[i].x), __fmul_rn(p[i].y, s[i].y));
    y_lo[i] = product_plus(p[i], c[i], make_float2(-qs.x, -qs.y));
    y_hi[i] = product_plus(q[i], c[i], ps);
  }
  out_lo = pack_pairs<T>(y_lo);
  out_hi = pack_pairs<T>(y_hi);
}

// 1 / sqrt(sum_sq / D + eps) for a power-of-two head size D: the mean is a
// multiply by an exact power of two; the reciprocal is correctly rounded, as
// a correctly rounded divide of 1 would be.
template <int D>
__device__ __forceinline__ float head_inverse_rms(float2 acc, float eps) {
  static_assert((D & (D - 1)) == 0, "head size must be a power of two");
  const float sum = __fadd_rn(acc.x, acc.y);
  return __frcp_rn(__fsqrt_rn(__fadd_rn(__fmul_rn(sum, 1.0f / D), eps)));
}

template <typename T>
__device__ __forceinline__ Half8<T> select_half(bool first, const Half8<T>& a, const Half8<T>& b) {
  Half8<T> r;
#pragma unroll
  for (int i = 0; i < Half8<T>::kWords; ++i) r.w[i] = first ? a.w[i] : b.w[i];
  return r;
}

// Eight consecutive fp32 values (cos or sin) as four pairs.
template <bool kVector>
__device__ __forceinline__ void load8_pairs(const float* p, float2* f) {
  if constexpr (kVector) {
    const float4 a = *reinterpret_cast<const float4*>(p);
    const float4 b = *reinterpret_cast<const float4*>(p + 4);
    f[0] = make_float2(a.x, a.y);
    f[1] = make_float2(a.z, a.w);
    f[2] = make_float2(b.x, b.y);
    f[3] = make_float2(b.z, b.w);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) f[i] = make_float2(p[2 * i], p[2 * i + 1]);
  }
}

}  // namespace sm120n
