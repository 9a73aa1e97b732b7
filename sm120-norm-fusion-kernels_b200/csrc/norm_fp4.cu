// norm_fp4.cu -- RMSNorm (optionally after the residual add) with an NVFP4
// output, for B200 (sm_100a); C-ABI entry point sm120n_rms_norm_fp4_quant.
//
// The normalised row y is the one sm120n_rms_norm / sm120n_fused_add_rms_norm
// produce (reference project, sm120_rmsnorm/reference.py:5-24); it is then
// quantised for a block-scaled fp4 GEMM instead of being stored. Per block of
// 16 consecutive elements of a row, with the caller's fp32 global scale g and
// every step one IEEE fp32 operation:
//   a = max |y|                         (exact)
//   s = e4m3(g * (a * c))               (c = 1/6 rounded to fp32; saturating,
//                                        nearest even)
//   r = s == 0 ? 0 : g / s              (IEEE division)
//   q = e2m1(y * r)                     (saturating at 6, nearest even)
// q is packed two per byte, element 2i in the low nibble; s is stored as one
// e4m3 byte per block, either row-major [rows, hidden / 16] or in the 128 x 4
// tiled layout that block-scaled tensor-core GEMMs read: rows padded to 128
// and blocks to 4, tile (rows / 128, blocks / 4) stored as [32][4][4] with
// byte offset ((m % 32) * 4 + (m % 128) / 32) * 4 + k % 4 inside the tile.
//
// Kernels: a block per row with the row held in registers (rows up to 2048
// 16-byte packs) and a vectorised two-pass kernel for wider rows. A 16-element
// block spans 2 packs of a 16-bit type (4 of fp32) held by adjacent lanes, so
// its maximum takes one (two) shuffles and no extra barrier. r takes one of
// 256 values (one per e4m3 code): the 256-thread many-row launch (a block
// per row) and the two-pass kernel divide once per code into a shared-memory
// table, one division per thread, so their per-block work has no division;
// the other launch shapes divide per 16-element block.
#include <cuda_fp4.h>
#include <cuda_fp8.h>

#include <algorithm>
#include <type_traits>

#include "device_utils.cuh"
#include "runtime.h"

namespace sm120n {
namespace {

constexpr int kBlockElems = 16;
constexpr float kOneSixth = 1.0f / 6.0f;  // rounded to fp32 at compile time

template <typename T>
struct Fp4Args {
  const T* input;
  const T* residual;  // nullptr: plain RMSNorm
  const T* weight;
  T* residual_output;
  uint8_t* output;        // [rows, hidden / 2]
  uint8_t* block_scales;  // e4m3, layout per `tiled`
  const float* global_scale;
  int64_t rows;
  int hidden;
  int scale_columns;  // hidden / 16, padded to 4 when tiled
  bool tiled;
  float epsilon;
};

// Byte offset of block `block`'s scale in row `row`, split into a part that
// depends on the row only and one that depends on the block only:
//   row-major  row * columns + block
//   tiled      tile (row / 128, block / 4) of 512 bytes, then
//              ((row % 32) * 4 + (row % 128) / 32) * 4 + block % 4 inside it
// (row and block are non-negative).
__device__ __forceinline__ int64_t scale_row_offset(int64_t row, int columns, bool tiled) {
  if (!tiled) return row * columns;
  const uint64_t m = static_cast<uint64_t>(row);
  return static_cast<int64_t>((m >> 7) * (static_cast<uint64_t>(columns) >> 2) * 512 +
                              (((m & 31) << 2) + ((m & 127) >> 5)) * 4);
}

__device__ __forceinline__ int64_t scale_block_offset(int block, bool tiled) {
  const uint32_t k = static_cast<uint32_t>(block);
  return tiled ? static_cast<int64_t>(k >> 2) * 512 + static_cast<int64_t>(k & 3u)
               : static_cast<int64_t>(k);
}

// r = g / s for the e4m3 code of s.
__device__ __forceinline__ float multiplier_of(uint8_t code, float g) {
  const __half_raw h = __nv_cvt_fp8_to_halfraw(static_cast<__nv_fp8_storage_t>(code), __NV_E4M3);
  const float s = __half2float(__half(h));
  return s == 0.0f ? 0.0f : __fdiv_rn(g, s);
}

// r = g / s for every e4m3 code s (0 for s = 0), one entry per thread,
// visible to the block after the caller's barrier.
__device__ __forceinline__ void fill_multipliers(float* table, float g) {
  for (int code = threadIdx.x; code < 256; code += blockDim.x) {
    table[code] = multiplier_of(static_cast<uint8_t>(code), g);
  }
}

// Block scale s (as an e4m3 byte) of a block whose largest magnitude is `peak`.
__device__ __forceinline__ uint8_t block_scale(float peak, float g) {
  return static_cast<uint8_t>(
      __nv_cvt_float_to_fp8(__fmul_rn(g, __fmul_rn(peak, kOneSixth)), __NV_SATFINITE, __NV_E4M3));
}

// e2m1 codes of one pack of y times r, two per byte (element 2i low), as the
// low Pack<T>::kElems / 2 bytes of the result.
template <typename T>
__device__ __forceinline__ uint32_t fp4_pack(const uint4& y, float r) {
  float2 f[Pack<T>::kElems / 2];
  pack_to_pairs<T>(y, f);
  const float2 r2 = make_float2(r, r);
  uint32_t b[Pack<T>::kElems / 2];
#pragma unroll
  for (int i = 0; i < Pack<T>::kElems / 2; ++i) {
    // packed product: each half rounds like __fmul_rn, and only the
    // conversion consumes it
    b[i] = __nv_cvt_float2_to_fp4x2(__fmul2_rn(f[i], r2), __NV_E2M1, cudaRoundNearest);
  }
  // byte i of the result is the low byte of b[i] (the bytes above the pack's
  // Pack<T>::kElems / 2 are not stored)
  const uint32_t low = __byte_perm(b[0], b[1], 0x0040);
  if constexpr (Pack<T>::kElems / 2 == 4) {
    return __byte_perm(low, __byte_perm(b[2], b[3], 0x0040), 0x5410);
  } else {
    return low;
  }
}

template <typename T>
__device__ __forceinline__ float pack_peak(const uint4& y) {
  if constexpr (sizeof(T) == 2) {
    // |y| and the largest by packed abs and max, both exact on the 16-bit
    // values
    using V2 = std::conditional_t<std::is_same_v<T, __half>, __half2, __nv_bfloat162>;
    auto magnitudes = [](uint32_t w) { return __habs2(*reinterpret_cast<const V2*>(&w)); };
    const V2 m = __hmax2(__hmax2(magnitudes(y.x), magnitudes(y.y)),
                         __hmax2(magnitudes(y.z), magnitudes(y.w)));
    float lo, hi;
    Pack<T>::word_to_f32(*reinterpret_cast<const uint32_t*>(&m), lo, hi);
    return fmaxf(lo, hi);
  } else {
    float f[Pack<T>::kElems];
    Pack<T>::to_f32(y, f);
    float m = 0.0f;
#pragma unroll
    for (int i = 0; i < Pack<T>::kElems; ++i) m = fmaxf(m, fabsf(f[i]));
    return m;
  }
}

// The largest magnitude of a 16-element block: packs of one block sit in
// kLanes adjacent lanes (pack index and lane agree modulo kLanes).
template <typename T>
__device__ __forceinline__ float block_peak(float m) {
  constexpr int kLanes = kBlockElems / Pack<T>::kElems;
#pragma unroll
  for (int offset = 1; offset < kLanes; offset <<= 1) {
    m = fmaxf(m, __shfl_xor_sync(kFullMask, m, offset));
  }
  return m;
}

template <typename T>
__device__ __forceinline__ void store_fp4(uint8_t* p, uint32_t v) {
  if constexpr (Pack<T>::kElems == 8) {
    *reinterpret_cast<uint32_t*>(p) = v;
  } else {
    *reinterpret_cast<uint16_t*>(p) = static_cast<uint16_t>(v);
  }
}

// Quantise one pack c of a row (y already normalised); every lane of the warp
// calls this (the shuffles need them all), `valid` marks real packs.
// `out_row`: the row's first output byte; `scale_row`: scale_row_offset of the
// row. `multipliers`: the per-code table, or nullptr to divide here.
template <typename T>
__device__ __forceinline__ void quantise_fp4_pack(const Fp4Args<T>& a, uint8_t* out_row,
                                                  int64_t scale_row, int c, bool valid,
                                                  const uint4& y, float g,
                                                  const float* multipliers) {
  constexpr int E = Pack<T>::kElems;
  constexpr int kLanes = kBlockElems / E;
  const float peak = block_peak<T>(valid ? pack_peak<T>(y) : 0.0f);
  if (!valid) return;
  const uint8_t code = block_scale(peak, g);
  const float r = multipliers != nullptr ? multipliers[code] : multiplier_of(code, g);
  store_fp4<T>(out_row + static_cast<uint32_t>(c) * (E / 2), fp4_pack<T>(y, r));
  if (c % kLanes == 0) {
    a.block_scales[scale_row + scale_block_offset(c / kLanes, a.tiled)] = code;
  }
}

// kMinBlocks: resident blocks per SM the register budget must allow (left to
// itself the compiler gives the four-pack, 256-thread shape 114 registers, 2
// blocks per SM, and the two-pack, 512-thread shape 80, 1 block per SM; both
// measured slower than the capped budgets).
// kWeightsInRegisters: each thread keeps its weight packs in registers for the
// whole launch; otherwise it reads them from L1 per row, which frees 16
// registers (the four-pack prefill shape then fits four blocks per SM).
template <typename T, bool kAdd, int kPacksPerThread, int kMaxThreads, int kMinBlocks,
          bool kTable, bool kWeightsInRegisters = true>
__global__ void __launch_bounds__(kMaxThreads, kMinBlocks) norm_fp4_cta_kernel(Fp4Args<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  __shared__ float multipliers[256];
  // every NVFP4 row is 16-byte aligned; the second row only below four packs
  if constexpr (kPacksPerThread < 4) {
    prefetch_first_rows<T, kAdd>(a, blockIdx.x, static_cast<int64_t>(blockIdx.x) + gridDim.x);
  } else {
    prefetch_first_row<T, kAdd>(a, blockIdx.x);
  }
  wait_for_upstream_grid();
  release_downstream_grid();
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);
  const float g = *a.global_scale;
  if constexpr (kTable) fill_multipliers(multipliers, g);  // read after the first barrier
  uint4 w[kPacksPerThread];
  if constexpr (kWeightsInRegisters) {
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) w[i] = load16(a.weight + static_cast<int64_t>(c) * E);
    }
  }
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
    const float inv = inverse_rms(block_allreduce_sum(__fadd_rn(acc.x, acc.y), partial, parity),
                                  n, a.epsilon);
    parity ^= 1;
    uint8_t* out_row = a.output + row * (a.hidden / 2);
    const int64_t scale_row = scale_row_offset(row, a.scale_columns, a.tiled);
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      const bool valid = c < packs;
      uint4 y = make_uint4(0, 0, 0, 0);
      if (valid) {
        y = normalise_pack<T>(
            s[i], kWeightsInRegisters ? w[i] : load16(a.weight + static_cast<int64_t>(c) * E),
            inv);
      }
      quantise_fp4_pack<T>(a, out_row, scale_row, c, valid, y, g, kTable ? multipliers : nullptr);
    }
  }
}

// Rows wider than the register kernel holds: pass 1 adds, stores the residual
// and sums squares; pass 2 re-reads the packs this thread handled (now in L2)
// and quantises them.
template <typename T, bool kAdd>
__global__ void __launch_bounds__(1024) norm_fp4_wide_kernel(Fp4Args<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  __shared__ float multipliers[256];
  prefetch_first_row<T, kAdd>(a, blockIdx.x);  // every NVFP4 row is 16-byte aligned
  wait_for_upstream_grid();
  release_downstream_grid();
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);
  const float g = *a.global_scale;
  fill_multipliers(multipliers, g);  // first read after the row's reduction barrier
  const T* source = kAdd ? a.residual_output : a.input;
  // every lane runs the same number of pass-2 iterations (the shuffles need
  // the whole warp); blockDim.x is a multiple of the warp size
  const int rounds = (packs + blockDim.x - 1) / blockDim.x;
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
    const float inv = inverse_rms(block_allreduce_sum(__fadd_rn(acc.x, acc.y), partial, parity),
                                  n, a.epsilon);
    parity ^= 1;
    uint8_t* out_row = a.output + row * (a.hidden / 2);
    const int64_t scale_row = scale_row_offset(row, a.scale_columns, a.tiled);
    for (int k = 0; k < rounds; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      const bool valid = c < packs;
      uint4 y = make_uint4(0, 0, 0, 0);
      if (valid) {
        y = normalise_pack<T>(load16(source + base + static_cast<int64_t>(c) * E),
                              load16(a.weight + static_cast<int64_t>(c) * E), inv);
      }
      quantise_fp4_pack<T>(a, out_row, scale_row, c, valid, y, g, multipliers);
    }
  }
}

template <typename Kernel>
int fp4_grid(Kernel kernel, int threads, int64_t rows, int* grid) {
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

template <typename T, bool kAdd, int kPPT, int kMaxThreads, int kMinBlocks = 1,
          bool kTable = false, bool kWeightsInRegisters = true>
int launch_fp4_cta(const Fp4Args<T>& a, int packs, cudaStream_t stream,
                   bool one_row_per_block = false) {
  auto kernel =
      norm_fp4_cta_kernel<T, kAdd, kPPT, kMaxThreads, kMinBlocks, kTable, kWeightsInRegisters>;
  const int threads = (((packs + kPPT - 1) / kPPT) + kWarpSize - 1) / kWarpSize * kWarpSize;
  int grid = 0;
  if (one_row_per_block && a.rows <= INT32_MAX) {
    grid = static_cast<int>(a.rows);
  } else {
    int rc = fp4_grid(kernel, threads, a.rows, &grid);
    if (rc != SM120N_OK) return rc;
  }
  return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
}

template <typename T, bool kAdd>
int run_fp4(const Fp4Args<T>& a, cudaStream_t stream) {
  constexpr int E = Pack<T>::kElems;
  const int packs = a.hidden / E;
  // The same launch shapes as the fp8 kernels of this family.
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  const bool many_rows = a.rows >= 8 * static_cast<int64_t>(dev.sm_count);
  if (packs <= 256) return launch_fp4_cta<T, kAdd, 1, 256>(a, packs, stream);
  if (many_rows && packs > 512 && packs <= 1024) {
    // A 256-thread block per row, the weight read from L1 per row: 60
    // registers and four blocks per SM instead of 80 and three (persistent
    // grids, bf16 65536 x 8192: 588 us against 643), then a block per row
    // instead of the persistent grid (65536 x 8192 with the add 538.5 us
    // against 568, fp16 32768 x 5120 183.5 against 198, 16384 x 8192 146
    // against 150; without the add 427 against 425). A block fills the
    // 256-entry multiplier table with one division per thread, no more than
    // dividing per 16-element block would cost. Bit-identical results.
    return launch_fp4_cta<T, kAdd, 4, 256, 4, true, false>(a, packs, stream, true);
  }
  if (packs <= 1024) return launch_fp4_cta<T, kAdd, 2, 512, 2>(a, packs, stream);
  if (packs <= 2048) return launch_fp4_cta<T, kAdd, 4, 512>(a, packs, stream);
  auto kernel = norm_fp4_wide_kernel<T, kAdd>;
  int grid = 0;
  rc = fp4_grid(kernel, 1024, a.rows, &grid);
  if (rc != SM120N_OK) return rc;
  return launch(kernel, dim3(grid), dim3(1024), 0, stream, a);
}

template <typename T>
int run_fp4_typed(const void* input, const void* residual, const void* weight,
                  void* residual_output, void* output, void* block_scales,
                  const float* global_scale, int64_t rows, int64_t hidden, float epsilon,
                  bool tiled, cudaStream_t stream) {
  const int blocks = static_cast<int>(hidden / kBlockElems);
  Fp4Args<T> a{static_cast<const T*>(input), static_cast<const T*>(residual),
               static_cast<const T*>(weight), static_cast<T*>(residual_output),
               static_cast<uint8_t*>(output), static_cast<uint8_t*>(block_scales), global_scale,
               rows, static_cast<int>(hidden), tiled ? (blocks + 3) / 4 * 4 : blocks, tiled,
               epsilon};
  return residual != nullptr ? run_fp4<T, true>(a, stream) : run_fp4<T, false>(a, stream);
}

}  // namespace
}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_rms_norm_fp4_quant(const void* input, const void* residual,
                                         const void* weight, void* residual_output, void* output,
                                         void* block_scales, const float* global_scale,
                                         int64_t rows, int64_t hidden_size, int dtype,
                                         float epsilon, int scale_layout, void* stream) {
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
  if (hidden_size % kBlockElems != 0) {
    return fail(SM120N_ERR_UNSUPPORTED,
                "NVFP4 needs hidden_size to be a multiple of 16 (got %lld)",
                static_cast<long long>(hidden_size));
  }
  if (scale_layout != SM120N_SCALES_ROW_MAJOR && scale_layout != SM120N_SCALES_TILED_128X4) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "unknown scale_layout %d", scale_layout);
  }
  if ((residual == nullptr) != (residual_output == nullptr)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "residual and residual_output go together");
  }
  if (rows == 0) return SM120N_OK;
  if (!input || !weight || !output || !block_scales || !global_scale) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "input, weight, output, block_scales and global_scale must be non-null");
  }
  const uintptr_t out_align = dtype == SM120N_F32 ? 2 : 4;
  if (!aligned16(input) || !aligned16(weight) || (residual && !aligned16(residual)) ||
      (residual_output && !aligned16(residual_output)) ||
      (reinterpret_cast<uintptr_t>(output) % out_align) != 0) {
    return fail(SM120N_ERR_UNSUPPORTED,
                "NVFP4 quantisation needs 16-byte-aligned input, residual and weight and a "
                "%d-byte-aligned output", static_cast<int>(out_align));
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  const bool tiled = scale_layout == SM120N_SCALES_TILED_128X4;
  switch (dtype) {
    case SM120N_F32:
      return run_fp4_typed<float>(input, residual, weight, residual_output, output, block_scales,
                                  global_scale, rows, hidden_size, epsilon, tiled, s);
    case SM120N_F16:
      return run_fp4_typed<__half>(input, residual, weight, residual_output, output,
                                   block_scales, global_scale, rows, hidden_size, epsilon, tiled,
                                   s);
    default:
      return run_fp4_typed<__nv_bfloat16>(input, residual, weight, residual_output, output,
                                          block_scales, global_scale, rows, hidden_size, epsilon,
                                          tiled, s);
  }
}
