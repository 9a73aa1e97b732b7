// norm_quant.cu -- RMSNorm (optionally after the residual add) with an fp8
// e4m3 output, for B200 (sm_100a); C-ABI entry point
// sm120n_rms_norm_fp8_quant.
//
// The normalised row y is the one sm120n_rms_norm / sm120n_fused_add_rms_norm
// produce (reference project, sm120_rmsnorm/reference.py:5-24: one rounding of
// s * inv_rms * w to the activation dtype); it is then quantised for an fp8
// GEMM instead of being stored:
//   static  q = sat(y * (1 / scale))
//   dynamic token_scale = max(min(max|y|, scale_ub) / 448, 1 / (448 * 512)),
//           q = sat(y * (1 / token_scale))
// sat() clamps to +-448 and rounds to the nearest e4m3fn value (ties to
// even), which is what the hardware conversion with saturation does.
//
// Kernels: one thread block per row with the row held in registers
// (16-byte loads, 8-byte fp8 stores for 16-bit inputs; rows up to 2048
// packs, i.e. 16384 bf16 elements), one barrier for the sum of squares and,
// for dynamic scales, one for the row maximum; a vectorised multi-pass kernel
// for wider rows; and a scalar multi-pass kernel for any other row.
#include <cuda_fp8.h>

#include <algorithm>

#include "device_utils.cuh"
#include "runtime.h"

namespace sm120n {
namespace {

constexpr float kFp8Max = 448.0f;
constexpr float kMinTokenScale = 1.0f / (448.0f * 512.0f);

template <typename T>
struct QuantArgs {
  const T* input;
  const T* residual;  // nullptr: plain RMSNorm
  const T* weight;
  T* residual_output;
  uint8_t* output;
  const float* scale;  // static scale, or nullptr for dynamic
  float* token_scales;
  const float* scale_ub;  // optional bound on the dynamic row maximum
  int64_t rows;
  int hidden;
  float epsilon;
};

__device__ __forceinline__ float block_allreduce(float v, float (*partial)[kWarpSize], int parity,
                                                 bool take_max) {
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int warp = threadIdx.x / kWarpSize;
  const int warps = blockDim.x / kWarpSize;
#pragma unroll
  for (int offset = kWarpSize / 2; offset > 0; offset >>= 1) {
    const float other = __shfl_xor_sync(kFullMask, v, offset);
    v = take_max ? fmaxf(v, other) : __fadd_rn(v, other);
  }
  if (lane == 0) partial[parity][warp] = v;
  __syncthreads();
  float total = 0.0f;  // the sum's identity; also the floor of an absolute maximum
  for (int i = 0; i < warps; ++i) {
    total = take_max ? fmaxf(total, partial[parity][i]) : __fadd_rn(total, partial[parity][i]);
  }
  return total;
}

// Quantised bytes of one pack of y (kElems values), element 0 lowest.
template <typename T>
__device__ __forceinline__ uint2 quantise_pack(const uint4& y, float inv_scale) {
  float f[Pack<T>::kElems];
  Pack<T>::to_f32(y, f);
  uint32_t b[4] = {0, 0, 0, 0};
#pragma unroll
  for (int i = 0; i < Pack<T>::kElems / 2; ++i) {
    const float2 q = make_float2(__fmul_rn(f[2 * i], inv_scale), __fmul_rn(f[2 * i + 1], inv_scale));
    b[i] = static_cast<uint32_t>(__nv_cvt_float2_to_fp8x2(q, __NV_SATFINITE, __NV_E4M3));
  }
  return make_uint2(b[0] | (b[1] << 16), b[2] | (b[3] << 16));
}

template <typename T>
__device__ __forceinline__ float pack_abs_max(const uint4& y, float m) {
  float f[Pack<T>::kElems];
  Pack<T>::to_f32(y, f);
#pragma unroll
  for (int i = 0; i < Pack<T>::kElems; ++i) m = fmaxf(m, fabsf(f[i]));
  return m;
}

template <typename T>
__device__ __forceinline__ void store_quantised(uint8_t* p, uint2 q) {
  if constexpr (Pack<T>::kElems == 8) {
    *reinterpret_cast<uint2*>(p) = q;
  } else {
    *reinterpret_cast<uint32_t*>(p) = q.x;
  }
}

__device__ __forceinline__ float token_scale(float peak, const float* scale_ub) {
  if (scale_ub != nullptr) peak = fminf(peak, *scale_ub);
  return fmaxf(__fdiv_rn(peak, kFp8Max), kMinTokenScale);
}

// kWeightsInRegisters: each thread keeps its weight packs in registers for the
// whole launch; otherwise it reads them from L1 per row, which frees the
// registers for more resident blocks (kMinBlocks per SM).
template <typename T, bool kAdd, bool kDynamic, int kPacksPerThread, int kMaxThreads,
          int kMinBlocks = 0, bool kWeightsInRegisters = true>
__global__ void __launch_bounds__(kMaxThreads, kMinBlocks) norm_quant_cta_kernel(QuantArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  __shared__ float peaks[2][kWarpSize];
  // as in row_norm_cta_kernel: no prefetch for the four-pack (prefill) forms
  if constexpr (kPacksPerThread < 4) {
    prefetch_first_rows<T, kAdd>(a, blockIdx.x, static_cast<int64_t>(blockIdx.x) + gridDim.x);
  }
  wait_for_upstream_grid();
  release_downstream_grid();
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);
  uint4 w[kPacksPerThread];
  if constexpr (kWeightsInRegisters) {
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) w[i] = load16(a.weight + static_cast<int64_t>(c) * E);
    }
  }
  float inv_scale = 0.0f;
  if constexpr (!kDynamic) inv_scale = __frcp_rn(*a.scale);

  int parity = 0;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.hidden;
    uint4 s[kPacksPerThread], r[kPacksPerThread];
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        s[i] = load16(a.input + base + static_cast<int64_t>(c) * E);
        if constexpr (kAdd) r[i] = load16(a.residual + base + static_cast<int64_t>(c) * E);
      }
    }
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        s[i] = combine_pack<T, kAdd>(s[i], r[i], acc);
        // stored before the reduction (every load of the row precedes it)
        if constexpr (kAdd) store16(a.residual_output + base + static_cast<int64_t>(c) * E, s[i]);
      }
    }
    const float inv =
        inverse_rms(block_allreduce(__fadd_rn(acc.x, acc.y), partial, parity, false), n, a.epsilon);
    float peak = 0.0f;
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        const uint4 wc =
            kWeightsInRegisters ? w[i] : load16(a.weight + static_cast<int64_t>(c) * E);
        s[i] = normalise_pack<T>(s[i], wc, inv);  // s now holds y
        if constexpr (kDynamic) peak = pack_abs_max<T>(s[i], peak);
      }
    }
    if constexpr (kDynamic) {
      const float scale = token_scale(block_allreduce(peak, peaks, parity, true), a.scale_ub);
      if (threadIdx.x == 0) a.token_scales[row] = scale;
      inv_scale = __frcp_rn(scale);
    }
    parity ^= 1;
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        store_quantised<T>(a.output + base + static_cast<int64_t>(c) * E,
                           quantise_pack<T>(s[i], inv_scale));
      }
    }
  }
}

// Wide 16-byte-aligned rows: packs in up to three passes (sum of squares and
// residual store; row maximum; quantisation). Later passes re-read exactly
// the packs this thread handled before, now resident in L2.
template <typename T, bool kAdd, bool kDynamic>
__global__ void __launch_bounds__(1024) norm_quant_wide_kernel(QuantArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  __shared__ float peaks[2][kWarpSize];
  wait_for_upstream_grid();
  release_downstream_grid();
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);
  float inv_scale = 0.0f;
  if constexpr (!kDynamic) inv_scale = __frcp_rn(*a.scale);
  const T* source = kAdd ? a.residual_output : a.input;
  int parity = 0;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.hidden;
    float2 acc = make_float2(0.0f, 0.0f);
    for (int c = threadIdx.x; c < packs; c += blockDim.x) {
      const int64_t off = base + static_cast<int64_t>(c) * E;
      uint4 r;
      if constexpr (kAdd) r = load16(a.residual + off);
      const uint4 s = combine_pack<T, kAdd>(load16(a.input + off), r, acc);
      if constexpr (kAdd) store16(a.residual_output + off, s);
    }
    const float inv =
        inverse_rms(block_allreduce(__fadd_rn(acc.x, acc.y), partial, parity, false), n, a.epsilon);
    auto y_at = [&](int c) {
      return normalise_pack<T>(load16(source + base + static_cast<int64_t>(c) * E),
                               load16(a.weight + static_cast<int64_t>(c) * E), inv);
    };
    if constexpr (kDynamic) {
      float peak = 0.0f;
      for (int c = threadIdx.x; c < packs; c += blockDim.x) peak = pack_abs_max<T>(y_at(c), peak);
      const float scale = token_scale(block_allreduce(peak, peaks, parity, true), a.scale_ub);
      if (threadIdx.x == 0) a.token_scales[row] = scale;
      inv_scale = __frcp_rn(scale);
    }
    parity ^= 1;
    for (int c = threadIdx.x; c < packs; c += blockDim.x) {
      store_quantised<T>(a.output + base + static_cast<int64_t>(c) * E,
                         quantise_pack<T>(y_at(c), inv_scale));
    }
  }
}

// Any row and alignment: element at a time, in up to three passes (sum of
// squares, row maximum, quantisation), each recomputing y from the stored sum.
template <typename T, bool kAdd, bool kDynamic>
__global__ void __launch_bounds__(256) norm_quant_scalar_kernel(QuantArgs<T> a) {
  using S = Scalar<T>;
  __shared__ float partial[2][kWarpSize];
  __shared__ float peaks[2][kWarpSize];
  wait_for_upstream_grid();
  release_downstream_grid();
  const float n = static_cast<float>(a.hidden);
  float inv_scale = 0.0f;
  if constexpr (!kDynamic) inv_scale = __frcp_rn(*a.scale);
  int parity = 0;
  const T* source = kAdd ? a.residual_output : a.input;
  for (int64_t row = blockIdx.x; row < a.rows; row += gridDim.x) {
    const int64_t base = row * a.hidden;
    float sum_sq = 0.0f;
    for (int c = threadIdx.x; c < a.hidden; c += blockDim.x) {
      float v = S::load(a.input + base + c);
      if constexpr (kAdd) {
        v = S::round(__fadd_rn(v, S::load(a.residual + base + c)));
        S::store(a.residual_output + base + c, v);
      }
      sum_sq = __fadd_rn(sum_sq, __fmul_rn(v, v));
    }
    const float inv = inverse_rms(block_allreduce(sum_sq, partial, parity, false), n, a.epsilon);
    auto y_at = [&](int c) {
      return S::round(__fmul_rn(__fmul_rn(S::load(source + base + c), inv), S::load(a.weight + c)));
    };
    if constexpr (kDynamic) {
      float peak = 0.0f;
      for (int c = threadIdx.x; c < a.hidden; c += blockDim.x) peak = fmaxf(peak, fabsf(y_at(c)));
      const float scale = token_scale(block_allreduce(peak, peaks, parity, true), a.scale_ub);
      if (threadIdx.x == 0) a.token_scales[row] = scale;
      inv_scale = __frcp_rn(scale);
    }
    parity ^= 1;
    for (int c = threadIdx.x; c < a.hidden; c += blockDim.x) {
      a.output[base + c] = static_cast<uint8_t>(
          __nv_cvt_float_to_fp8(__fmul_rn(y_at(c), inv_scale), __NV_SATFINITE, __NV_E4M3));
    }
  }
}

template <typename Kernel>
int grid_for(Kernel kernel, int threads, int64_t rows, int* grid) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  int resident = 1;
  rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), threads, 0, &resident);
  if (rc != SM120N_OK) return rc;
  *grid = static_cast<int>(
      std::max<int64_t>(1, std::min<int64_t>(rows, static_cast<int64_t>(dev.sm_count) * resident)));
  return SM120N_OK;
}

// `one_row_per_block`: a block per row, balanced by the block scheduler (the
// better shape for many wide rows, as for the plain row kernels); otherwise a
// persistent grid with a row loop.
template <typename T, bool kAdd, bool kDynamic, int kPPT, int kMaxThreads, int kMinBlocks = 0,
          bool kWeightsInRegisters = true>
int launch_quant_cta(const QuantArgs<T>& a, int packs, cudaStream_t stream,
                     bool one_row_per_block = false) {
  auto kernel =
      norm_quant_cta_kernel<T, kAdd, kDynamic, kPPT, kMaxThreads, kMinBlocks, kWeightsInRegisters>;
  const int threads = (((packs + kPPT - 1) / kPPT) + kWarpSize - 1) / kWarpSize * kWarpSize;
  int grid = 0;
  if (one_row_per_block && a.rows <= INT32_MAX) {
    grid = static_cast<int>(a.rows);
  } else {
    int rc = grid_for(kernel, threads, a.rows, &grid);
    if (rc != SM120N_OK) return rc;
  }
  return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
}

template <typename T, bool kAdd, bool kDynamic>
int run_quant(const QuantArgs<T>& a, cudaStream_t stream) {
  constexpr int E = Pack<T>::kElems;
  const int packs = a.hidden / E;
  const bool vectorisable = a.hidden % E == 0 && aligned16(a.input) && aligned16(a.weight) &&
                            (reinterpret_cast<uintptr_t>(a.output) % E) == 0 &&
                            (!kAdd || (aligned16(a.residual) && aligned16(a.residual_output)));
  // At most 512 threads per block, so a thread may hold its packs of x, r
  // and w in up to 128 registers without spilling.
  if (vectorisable && packs <= 4 * 512) {
    // Chosen from measurements on B200 (graphs of back-to-back calls on cold
    // data): rows wider than 512 packs with many rows run best as a
    // 256-thread block per row holding four packs per thread, reading the
    // weight from L1 per row so that more blocks fit on an SM: three per SM
    // with the residual add (four with dynamic scales), five without. Against the persistent grid of the
    // same blocks (three / four per SM), 65536 x 8192 bf16 with the add:
    // static 539 us against 575, dynamic 571 against 588; without it: static
    // 296 against 304, dynamic 342 against 380, fp16 static 285 against 316;
    // 2048 to 16384 rows and 5120- to 8192-wide rows gain 1-14% likewise
    // (the persistent grid with the weight in registers took 607 us with the
    // add). Narrower or fewer rows keep two packs per thread.
    DeviceInfo dev;
    int rc = current_device_info(&dev);
    if (rc != SM120N_OK) return rc;
    const bool many_rows = a.rows >= 8 * static_cast<int64_t>(dev.sm_count);
    if (packs <= 256) return launch_quant_cta<T, kAdd, kDynamic, 1, 256>(a, packs, stream);
    if (many_rows && packs > 512 && packs <= 1024) {
      if constexpr (kAdd && kDynamic) {
        // the row maximum's second barrier per row wants a fourth block per
        // SM (65536 x 8192 bf16 541 us against 571 at three)
        return launch_quant_cta<T, kAdd, kDynamic, 4, 256, 4, false>(a, packs, stream, true);
      } else if constexpr (kAdd) {
        return launch_quant_cta<T, kAdd, kDynamic, 4, 256, 3, false>(a, packs, stream, true);
      } else {
        return launch_quant_cta<T, kAdd, kDynamic, 4, 256, 5, false>(a, packs, stream, true);
      }
    }
    if (packs <= 1024) {
      const int threads = ((packs + 1) / 2 + kWarpSize - 1) / kWarpSize * kWarpSize;
      if constexpr (kDynamic) {
        // Dynamic scales add a second barrier per row (the row maximum).
        // Where the blocks holding the weight in registers cannot take every
        // row at once, reading it from L1 fits six blocks per SM instead of
        // four, and fewer blocks make a second pass (1024 x 4096 bf16 6.1 us
        // against 6.8 without the add, 7.8 against 7.9 with it; same sums).
        int grid = 0;
        rc = grid_for(norm_quant_cta_kernel<T, kAdd, kDynamic, 2, 512>, threads, a.rows, &grid);
        if (rc != SM120N_OK) return rc;
        if (threads <= 256 && a.rows > grid) {
          return launch_quant_cta<T, kAdd, kDynamic, 2, 256, 6, false>(a, packs, stream);
        }
      }
      return launch_quant_cta<T, kAdd, kDynamic, 2, 512>(a, packs, stream);
    }
    return launch_quant_cta<T, kAdd, kDynamic, 4, 512>(a, packs, stream);
  }
  int grid = 0;
  if (vectorisable) {
    auto kernel = norm_quant_wide_kernel<T, kAdd, kDynamic>;
    int rc = grid_for(kernel, 1024, a.rows, &grid);
    if (rc != SM120N_OK) return rc;
    return launch(kernel, dim3(grid), dim3(1024), 0, stream, a);
  }
  auto kernel = norm_quant_scalar_kernel<T, kAdd, kDynamic>;
  int rc = grid_for(kernel, 256, a.rows, &grid);
  if (rc != SM120N_OK) return rc;
  return launch(kernel, dim3(grid), dim3(256), 0, stream, a);
}

template <typename T>
int run_quant_typed(const void* input, const void* residual, const void* weight,
                    void* residual_output, void* output, const float* scale, float* token_scales,
                    const float* scale_ub, int64_t rows, int64_t hidden, float epsilon,
                    cudaStream_t stream) {
  QuantArgs<T> a{static_cast<const T*>(input), static_cast<const T*>(residual),
                 static_cast<const T*>(weight), static_cast<T*>(residual_output),
                 static_cast<uint8_t*>(output), scale, token_scales, scale_ub, rows,
                 static_cast<int>(hidden), epsilon};
  const bool add = residual != nullptr;
  const bool dynamic = scale == nullptr;
  if (add) {
    return dynamic ? run_quant<T, true, true>(a, stream) : run_quant<T, true, false>(a, stream);
  }
  return dynamic ? run_quant<T, false, true>(a, stream) : run_quant<T, false, false>(a, stream);
}

}  // namespace
}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_rms_norm_fp8_quant(const void* input, const void* residual,
                                         const void* weight, void* residual_output, void* output,
                                         const float* scale, float* token_scales,
                                         const float* scale_ub, int64_t rows, int64_t hidden_size,
                                         int dtype, float epsilon, void* stream) {
  clear_error();
  if (dtype_size(dtype) == 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "supported dtypes are float16, bfloat16, and float32");
  }
  if (rows < 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "rows must be non-negative (got %lld)",
                static_cast<long long>(rows));
  }
  if (hidden_size <= 0 || hidden_size > (int64_t{1} << 30)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "hidden_size must be in [1, 2^30] (got %lld)",
                static_cast<long long>(hidden_size));
  }
  if ((scale == nullptr) == (token_scales == nullptr)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "exactly one of scale (static) and token_scales (dynamic) must be given");
  }
  if (scale != nullptr && scale_ub != nullptr) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "scale_ub applies to dynamic scales only");
  }
  if ((residual == nullptr) != (residual_output == nullptr)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "residual and residual_output go together");
  }
  if (rows == 0) return SM120N_OK;
  if (!input || !weight || !output) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "input, weight and output must be non-null");
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  switch (dtype) {
    case SM120N_F32:
      return run_quant_typed<float>(input, residual, weight, residual_output, output, scale,
                                    token_scales, scale_ub, rows, hidden_size, epsilon, s);
    case SM120N_F16:
      return run_quant_typed<__half>(input, residual, weight, residual_output, output, scale,
                                     token_scales, scale_ub, rows, hidden_size, epsilon, s);
    default:
      return run_quant_typed<__nv_bfloat16>(input, residual, weight, residual_output, output,
                                            scale, token_scales, scale_ub, rows, hidden_size,
                                            epsilon, s);
  }
}
