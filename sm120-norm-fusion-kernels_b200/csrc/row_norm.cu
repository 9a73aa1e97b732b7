// row_norm.cu -- RMSNorm and residual-add + RMSNorm over [rows, hidden] for
// B200 (sm_100a), and their C-ABI entry points.
//
// Reference behaviour (paths in the reference project):
//   sm120_rmsnorm/reference.py:5-24         the math and its rounding order
//   csrc/rmsnorm_kernels.cu:472-524         rms_norm(_out)_cuda
//   csrc/rmsnorm_kernels.cu:526-537, 711-801 fused_add_rms_norm{,_out,_inplace}_cuda
//
// The path is HBM-bound (about 10 flops per element), so every kernel here is
// shaped around moving bytes: 16-byte loads and stores, each element read once
// and written once, the row held in registers across the reduction, weights
// loaded once per thread block, and persistent grids sized from the SM count
// and the measured occupancy. Kernel families:
//
//   warp   one warp per row, rows <= 32 * 8 packs (<= 4 KiB of bf16);
//          shuffle-only reduction, no block barrier (fused version 3).
//   cta    one thread block per row, rows <= 1024 packs (16 KiB of bf16),
//          1, 2 or 4 packs per thread; one barrier per row (double-buffered
//          partial sums). The default for every row up to 16 KiB.
//   staged a block per row, the row and the weight brought into shared memory
//          by the TMA engine (cp.async.bulk, mbarrier completion); with the
//          residual add 4-16 KiB rows in calls of 16-128 MiB, without it
//          8-16 KiB rows in calls of 16-32 MiB.
//   bulk   persistent blocks, rows staged through shared memory by the TMA
//          engine (cp.async.bulk, mbarrier completion); rows of 16-32 KiB.
//   wide   one thread block per row, any 16-byte-aligned row; two passes
//          (the second re-reads the row, which is then L2-resident).
//   scalar any row, any alignment; element at a time, two passes.
//
// In-place use (output == input, residual_output == residual) is safe in all
// families: each element is read before it is written and only by the thread
// that writes it, and no pointer is declared __restrict__.
#include <algorithm>
#include <type_traits>

#include "device_utils.cuh"
#include "runtime.h"

namespace sm120n {

// Bounded waits that expired in the pipelined kernels of this file since the
// last reset (see sm120n_get_device_faults). Zero in correct operation.
__device__ unsigned int g_expired_waits = 0;
static_assert(kDefaultWaitPolls == kMaxBarrierPolls, "host and device wait bounds agree");

namespace {

template <typename T>
struct RowArgs {
  const T* input;
  const T* residual;  // nullptr for plain RMSNorm
  const T* weight;
  T* output;
  T* residual_output;  // nullptr for plain RMSNorm
  int64_t rows;
  int hidden;
  float epsilon;
  uint32_t wait_polls;  // poll limit of waits on bulk copies (from the host's setting)
};

// ---- warp family -----------------------------------------------------------
template <typename T, bool kAdd, int kPacksPerLane>
__global__ void __launch_bounds__(256) row_norm_warp_kernel(RowArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  prefetch_first_row<T, kAdd>(a, static_cast<int64_t>(blockIdx.x) * (blockDim.x / kWarpSize));
  wait_for_upstream_grid();
  release_downstream_grid();
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int warps = blockDim.x / kWarpSize;
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);

  uint4 w[kPacksPerLane];
#pragma unroll
  for (int i = 0; i < kPacksPerLane; ++i) {
    const int c = lane + i * kWarpSize;
    if (c < packs) w[i] = load16(a.weight + static_cast<int64_t>(c) * E);
  }

  for (int64_t row = static_cast<int64_t>(blockIdx.x) * warps + threadIdx.x / kWarpSize;
       row < a.rows; row += static_cast<int64_t>(gridDim.x) * warps) {
    const int64_t base = row * a.hidden;
    uint4 s[kPacksPerLane], r[kPacksPerLane];
#pragma unroll
    for (int i = 0; i < kPacksPerLane; ++i) {
      const int c = lane + i * kWarpSize;
      if (c < packs) {
        s[i] = load16(a.input + base + static_cast<int64_t>(c) * E);
        if constexpr (kAdd) r[i] = load16(a.residual + base + static_cast<int64_t>(c) * E);
      }
    }
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < kPacksPerLane; ++i) {
      const int c = lane + i * kWarpSize;
      if (c < packs) {
        s[i] = combine_pack<T, kAdd>(s[i], r[i], acc);
        // stored before the reduction (every load of the row precedes it)
        if constexpr (kAdd) store16(a.residual_output + base + static_cast<int64_t>(c) * E, s[i]);
      }
    }
    const float sum_sq = group_allreduce_sum<kWarpSize>(__fadd_rn(acc.x, acc.y));
    const float inv = inverse_rms(sum_sq, n, a.epsilon);
#pragma unroll
    for (int i = 0; i < kPacksPerLane; ++i) {
      const int c = lane + i * kWarpSize;
      if (c < packs) {
        store16(a.output + base + static_cast<int64_t>(c) * E, normalise_pack<T>(s[i], w[i], inv));
      }
    }
  }
}

// ---- cta family --------------------------------------------------------------
// kWeightsInRegisters: each thread keeps its weight packs in registers for the
// whole launch; otherwise it reads them from L1 per row, which frees the
// registers for more resident blocks (kMinBlocks per SM).
template <typename T, bool kAdd, int kPacksPerThread, int kMaxThreads, int kMinBlocks = 0,
          bool kWeightsInRegisters = true>
__global__ void __launch_bounds__(kMaxThreads, kMinBlocks) row_norm_cta_kernel(RowArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  // Four packs per thread serve the many-row, bandwidth-bound calls, where the
  // prefetch measured neutral and its registers cost the third resident
  // block per SM (695 us against 619 us on 65536 x 8192): they go without it.
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
    // The updated residual is stored as soon as it is formed, so its write
    // traffic overlaps the block reduction (1024 x 4096 bf16: 7.9-8.0 us
    // against 8.5 us storing it after the reduction). Every load of the row
    // precedes it, so an in-place residual is safe.
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        s[i] = combine_pack<T, kAdd>(s[i], r[i], acc);
        if constexpr (kAdd) store16(a.residual_output + base + static_cast<int64_t>(c) * E, s[i]);
      }
    }
    const float inv = inverse_rms(block_allreduce_sum(__fadd_rn(acc.x, acc.y), partial, parity),
                                  n, a.epsilon);
    parity ^= 1;
#pragma unroll
    for (int i = 0; i < kPacksPerThread; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < packs) {
        const uint4 wc =
            kWeightsInRegisters ? w[i] : load16(a.weight + static_cast<int64_t>(c) * E);
        store16(a.output + base + static_cast<int64_t>(c) * E, normalise_pack<T>(s[i], wc, inv));
      }
    }
  }
}

// ---- wide family: any 16-byte-aligned row, two passes ------------------------
template <typename T, bool kAdd>
__global__ void __launch_bounds__(1024) row_norm_wide_kernel(RowArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  __shared__ float partial[2][kWarpSize];
  wait_for_upstream_grid();
  release_downstream_grid();
  const int packs = a.hidden / E;
  const float n = static_cast<float>(a.hidden);
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
    // Pass 2 re-reads exactly the packs this thread handled in pass 1.
    const T* source = kAdd ? a.residual_output : a.input;
    for (int c = threadIdx.x; c < packs; c += blockDim.x) {
      const int64_t off = base + static_cast<int64_t>(c) * E;
      const uint4 s = load16(source + off);
      store16(a.output + off, normalise_pack<T>(s, load16(a.weight + static_cast<int64_t>(c) * E), inv));
    }
  }
}

// ---- scalar family: any row, any alignment -----------------------------------
template <typename T, bool kAdd>
__global__ void __launch_bounds__(256) row_norm_scalar_kernel(RowArgs<T> a) {
  using S = Scalar<T>;
  __shared__ float partial[2][kWarpSize];
  wait_for_upstream_grid();
  release_downstream_grid();
  const float n = static_cast<float>(a.hidden);
  int parity = 0;
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
    const float inv = inverse_rms(block_allreduce_sum(sum_sq, partial, parity), n, a.epsilon);
    parity ^= 1;
    const T* source = kAdd ? a.residual_output : a.input;
    for (int c = threadIdx.x; c < a.hidden; c += blockDim.x) {
      const float v = S::load(source + base + c);
      S::store(a.output + base + c, __fmul_rn(__fmul_rn(v, inv), S::load(a.weight + c)));
    }
  }
}

// ---- bulk family: rows staged through shared memory by the TMA engine ------
// Persistent blocks; block b owns rows b, b + gridDim.x, ... and keeps up to
// `stages` of them in flight. Thread 0 streams a row's input (and residual)
// into a shared-memory stage with cp.async.bulk; the stage's mbarrier counts
// the arriving bytes. Every thread waits for the stage, reads its 16-byte
// packs from shared memory, and joins the block reduction; that barrier also
// proves the stage has been read, so thread 0 refills it with the row
// `stages` ahead before the outputs are computed and stored from registers.
// Memory-level parallelism therefore comes from the copy engine, not from
// registers held by waiting threads.
constexpr int kMaxStages = 8;

template <typename T, bool kAdd, int kPacksPerThread>
__global__ void __launch_bounds__(1024) row_norm_bulk_kernel(RowArgs<T> a, int stages) {
  constexpr int E = Pack<T>::kElems;
  extern __shared__ __align__(128) unsigned char stage_memory[];
  __shared__ __align__(8) uint64_t stage_full[kMaxStages];
  __shared__ float partial[2][kWarpSize];
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int warp = threadIdx.x / kWarpSize;
  const int warps = blockDim.x / kWarpSize;
  const int packs = a.hidden / E;
  const uint32_t row_bytes = static_cast<uint32_t>(a.hidden) * sizeof(T);
  const uint32_t stage_bytes = kAdd ? 2 * row_bytes : row_bytes;
  const int64_t first_row = blockIdx.x;
  const int64_t my_rows =
      first_row < a.rows ? (a.rows - first_row + gridDim.x - 1) / gridDim.x : 0;
  const float n = static_cast<float>(a.hidden);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) mbarrier_init(&stage_full[s], 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  wait_for_upstream_grid();
  release_downstream_grid();

  auto refill = [&](int64_t i) {  // thread 0 only
    const int s = static_cast<int>(i % stages);
    const int64_t row = first_row + i * gridDim.x;
    unsigned char* dst = stage_memory + static_cast<size_t>(s) * stage_bytes;
    mbarrier_arrive_expect_tx(&stage_full[s], stage_bytes);
    bulk_load(dst, a.input + row * a.hidden, row_bytes, &stage_full[s]);
    if constexpr (kAdd) bulk_load(dst + row_bytes, a.residual + row * a.hidden, row_bytes, &stage_full[s]);
  };
  if (threadIdx.x == 0) {
    for (int64_t i = 0; i < my_rows && i < stages; ++i) refill(i);
  }

  uint4 w[kPacksPerThread];
#pragma unroll
  for (int k = 0; k < kPacksPerThread; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < packs) w[k] = load16(a.weight + static_cast<int64_t>(c) * E);
  }

  for (int64_t i = 0; i < my_rows; ++i) {
    const int s = static_cast<int>(i % stages);
    const uint32_t phase = static_cast<uint32_t>((i / stages) & 1);
    const bool arrived = mbarrier_wait_limited(&stage_full[s], phase, a.wait_polls);
    const unsigned char* stage = stage_memory + static_cast<size_t>(s) * stage_bytes;
    uint4 v[kPacksPerThread];
    float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
    for (int k = 0; k < kPacksPerThread; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < packs) {
        uint4 r;
        if constexpr (kAdd) r = load16_shared(stage + row_bytes + static_cast<uint32_t>(c) * 16);
        v[k] = combine_pack<T, kAdd>(load16_shared(stage + static_cast<uint32_t>(c) * 16), r, acc);
      }
    }
    const float sum_sq = group_allreduce_sum<kWarpSize>(__fadd_rn(acc.x, acc.y));
    if (lane == 0) partial[i & 1][warp] = sum_sq;
    if (__syncthreads_or(!arrived)) {
      // A copy never completed within the bound: record it, give copies still
      // in flight a bounded chance to land, and leave this block's rows.
      if (threadIdx.x == 0) {
        atomicAdd(&g_expired_waits, 1u);
        for (int64_t j = i; j < my_rows && j < i + stages; ++j) {
          mbarrier_wait_bounded(&stage_full[j % stages], static_cast<uint32_t>((j / stages) & 1));
        }
      }
      __syncthreads();
      return;
    }
    if (threadIdx.x == 0 && i + stages < my_rows) {
      fence_async_shared();  // this stage's shared-memory reads before the refill
      refill(i + stages);
    }
    float total = 0.0f;
    for (int k = 0; k < warps; ++k) total = __fadd_rn(total, partial[i & 1][k]);
    const float inv = inverse_rms(total, n, a.epsilon);
    const int64_t base = (first_row + i * gridDim.x) * a.hidden;
#pragma unroll
    for (int k = 0; k < kPacksPerThread; ++k) {
      const int c = threadIdx.x + k * blockDim.x;
      if (c < packs) {
        const int64_t off = base + static_cast<int64_t>(c) * E;
        if constexpr (kAdd) store16(a.residual_output + off, v[k]);
        store16(a.output + off, normalise_pack<T>(v[k], w[k], inv));
      }
    }
  }
}

// ---- staged family: a block per row, the row brought in by the TMA engine ---
// For calls whose rows fit on the device in about one wave of these blocks.
// Right after the upstream wait thread 0 copies the block's input row,
// residual row and the weight into shared memory with bulk copies, so a
// launch's reads are all in flight at once and no block waits for a second
// pass; data in flight occupy shared memory instead of registers, which keeps
// 2048 / kMaxThreads blocks resident per SM (the persistent register kernel
// fits half as many). Packs are assigned to threads as in the cta family with
// the same block size, so results are bit-identical to it.
template <typename T, bool kAdd, int kPacksPerThread, int kMaxThreads>
__global__ void __launch_bounds__(kMaxThreads, 2048 / kMaxThreads)
    row_norm_staged_kernel(RowArgs<T> a) {
  constexpr int E = Pack<T>::kElems;
  extern __shared__ __align__(128) unsigned char staged[];  // input | residual | weight
  __shared__ __align__(8) uint64_t landed;
  __shared__ float partial[2][kWarpSize];
  const int64_t row = blockIdx.x;
  const int packs = a.hidden / E;
  const uint32_t row_bytes = static_cast<uint32_t>(a.hidden) * sizeof(T);
  unsigned char* input_s = staged;
  unsigned char* residual_s = staged + row_bytes;
  unsigned char* weight_s = staged + (kAdd ? 2 : 1) * row_bytes;
  prefetch_first_row<T, kAdd>(a, row);
  if (threadIdx.x == 0) {
    mbarrier_init(&landed, 1);
    fence_mbarrier_init();
  }
  __syncthreads();
  wait_for_upstream_grid();
  release_downstream_grid();
  const int64_t base = row * a.hidden;
  if (threadIdx.x == 0) {
    mbarrier_arrive_expect_tx(&landed, (kAdd ? 3 : 2) * row_bytes);
    bulk_load(input_s, a.input + base, row_bytes, &landed);
    if constexpr (kAdd) bulk_load(residual_s, a.residual + base, row_bytes, &landed);
    bulk_load(weight_s, a.weight, row_bytes, &landed);
  }
  const bool arrived = mbarrier_wait_limited(&landed, 0, a.wait_polls);
  if (__syncthreads_or(!arrived)) {
    // The copies did not land within the limit: record it, wait (with the
    // full bound) for them to finish before the block's shared memory is
    // released, and leave the row.
    if (threadIdx.x == 0) {
      atomicAdd(&g_expired_waits, 1u);
      mbarrier_wait_bounded(&landed, 0);
    }
    __syncthreads();
    return;
  }
  uint4 s[kPacksPerThread];
  float2 acc = make_float2(0.0f, 0.0f);
#pragma unroll
  for (int k = 0; k < kPacksPerThread; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < packs) {
      uint4 r;
      if constexpr (kAdd) r = load16_shared(residual_s + static_cast<uint32_t>(c) * 16);
      s[k] = combine_pack<T, kAdd>(load16_shared(input_s + static_cast<uint32_t>(c) * 16), r, acc);
      if constexpr (kAdd) store16(a.residual_output + base + static_cast<int64_t>(c) * E, s[k]);
    }
  }
  const float inv =
      inverse_rms(block_allreduce_sum(__fadd_rn(acc.x, acc.y), partial, 0), static_cast<float>(a.hidden),
                  a.epsilon);
#pragma unroll
  for (int k = 0; k < kPacksPerThread; ++k) {
    const int c = threadIdx.x + k * blockDim.x;
    if (c < packs) {
      store16(a.output + base + static_cast<int64_t>(c) * E,
              normalise_pack<T>(s[k], load16_shared(weight_s + static_cast<uint32_t>(c) * 16), inv));
    }
  }
}

// ---------------------------------------------------------------------------
// Host-side dispatch
// ---------------------------------------------------------------------------
enum class Family { kAuto, kWarp, kCta, kCtaOnePack, kWide, kBulk, kScalar, kStaged };

// Launch shape of the bulk family, or false when a row does not fit.
struct BulkPlan {
  int threads = 0;
  int stages = 0;
  size_t smem = 0;
};

inline bool plan_bulk(int64_t hidden, int elem_size, bool add, int packs_per_thread,
                      size_t block_smem, BulkPlan* plan) {
  const size_t row_bytes = static_cast<size_t>(hidden) * elem_size;
  const size_t stage_bytes = add ? 2 * row_bytes : row_bytes;
  const int64_t packs = row_bytes / 16;
  const int64_t threads = (packs + packs_per_thread - 1) / packs_per_thread;
  if (threads > 1024) return false;
  // About 96 KiB of rows in flight per block, between 2 and 8 stages.
  int stages = static_cast<int>(std::min<size_t>(kMaxStages, (96 * 1024) / stage_bytes));
  stages = std::max(stages, 2);
  const size_t static_smem = 1024;  // barriers and partial sums, rounded up
  while (stages > 2 && stages * stage_bytes + static_smem > block_smem) --stages;
  if (stages * stage_bytes + static_smem > block_smem) return false;
  plan->threads = static_cast<int>((threads + kWarpSize - 1) / kWarpSize * kWarpSize);
  plan->stages = stages;
  plan->smem = stages * stage_bytes;
  return true;
}

// A persistent grid: enough blocks for `units` (rows / rows-per-block) but no
// more than fit on the device at once.
template <typename Kernel>
int persistent_grid(Kernel kernel, int threads, int64_t blocks_needed, int* grid) {
  DeviceInfo dev;
  int rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  int resident = 1;
  rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), threads, 0, &resident);
  if (rc != SM120N_OK) return rc;
  const int64_t cap = static_cast<int64_t>(dev.sm_count) * resident;
  *grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(blocks_needed, cap)));
  return SM120N_OK;
}

template <typename T, bool kAdd, int kPacksPerLane>
int launch_warp(const RowArgs<T>& a, cudaStream_t stream) {
  constexpr int kWarpsPerBlock = 4;
  auto kernel = row_norm_warp_kernel<T, kAdd, kPacksPerLane>;
  const int threads = kWarpsPerBlock * kWarpSize;
  int grid = 0;
  int rc = persistent_grid(kernel, threads, (a.rows + kWarpsPerBlock - 1) / kWarpsPerBlock, &grid);
  if (rc != SM120N_OK) return rc;
  return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
}

// `one_row_per_block`: a block per row and let the block scheduler balance
// the waves (best for many rows: measured 620 us vs 682 us persistent on the
// 65536 x 8192 bf16 prefill); otherwise a persistent grid with a row loop.
template <typename T, bool kAdd, int kPacksPerThread, int kMaxThreads, int kMinBlocks = 0,
          bool kWeightsInRegisters = true>
int launch_cta(const RowArgs<T>& a, int threads, cudaStream_t stream,
               bool one_row_per_block = false) {
  auto kernel =
      row_norm_cta_kernel<T, kAdd, kPacksPerThread, kMaxThreads, kMinBlocks, kWeightsInRegisters>;
  int grid = 0;
  if (one_row_per_block && a.rows <= INT32_MAX) {
    grid = static_cast<int>(a.rows);
  } else {
    int rc = persistent_grid(kernel, threads, a.rows, &grid);
    if (rc != SM120N_OK) return rc;
  }
  return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
}

template <typename T, bool kAdd, int kPacksPerThread>
int launch_bulk(const RowArgs<T>& a, const BulkPlan& plan, cudaStream_t stream) {
  auto kernel = row_norm_bulk_kernel<T, kAdd, kPacksPerThread>;
  int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), plan.smem);
  if (rc != SM120N_OK) return rc;
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  int resident = 1;
  rc = max_resident_ctas(reinterpret_cast<const void*>(kernel), plan.threads, plan.smem, &resident);
  if (rc != SM120N_OK) return rc;
  const int64_t grid = std::max<int64_t>(
      1, std::min<int64_t>(a.rows, static_cast<int64_t>(dev.sm_count) * resident));
  return launch(kernel, dim3(static_cast<unsigned>(grid)), dim3(plan.threads), plan.smem, stream,
                a, plan.stages);
}

// A block per row (rows <= INT32_MAX), two packs per thread, the row staged
// in `smem` bytes of shared memory.
template <typename T, bool kAdd, int kMaxThreads>
int launch_staged(const RowArgs<T>& a, int threads, cudaStream_t stream) {
  auto kernel = row_norm_staged_kernel<T, kAdd, 2, kMaxThreads>;
  const size_t smem = static_cast<size_t>(kAdd ? 3 : 2) * a.hidden * sizeof(T);
  const int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
  if (rc != SM120N_OK) return rc;
  return launch(kernel, dim3(static_cast<unsigned>(a.rows)), dim3(threads), smem, stream, a);
}

inline int round_up_warps(int64_t threads) {
  return static_cast<int>((threads + kWarpSize - 1) / kWarpSize * kWarpSize);
}

template <typename T, bool kAdd>
int run_rows(const RowArgs<T>& a, Family family, cudaStream_t stream) {
  constexpr int E = Pack<T>::kElems;
  const bool vectorisable =
      a.hidden % E == 0 && aligned16(a.input) && aligned16(a.weight) && aligned16(a.output) &&
      (!kAdd || (aligned16(a.residual) && aligned16(a.residual_output)));
  const int packs = a.hidden / E;
  if (!vectorisable) family = Family::kScalar;

  bool many_rows = false;
  if (family == Family::kAuto) {
    // Chosen from measurements on B200 (back-to-back calls on cold data):
    //   rows <= 4 KiB          one block per row, one pack per thread (within
    //                          0.1-0.2 us of a same-size copy at <= 256 rows)
    //   4-16 KiB, many rows    one block per row, four packs per thread, a
    //                          block per row (>= the copy peak at 65536 rows)
    //   4-16 KiB otherwise     persistent blocks, two packs per thread
    //   16-32 KiB              rows staged through shared memory (bulk)
    //   wider                  two-pass block per row
    DeviceInfo dev;
    int rc = current_device_info(&dev);
    if (rc != SM120N_OK) return rc;
    many_rows = a.rows >= 8 * static_cast<int64_t>(dev.sm_count);
    const int64_t input_bytes = a.rows * static_cast<int64_t>(a.hidden) * sizeof(T);
    // Rows staged in shared memory, a block per row: with the residual add,
    // 4-16 KiB rows in calls of 16-128 MiB of input (bf16 2048 x 4096: 13.3
    // us against 13.8; 4096 x 4096: 24.6 against 25.6; 1024 x 8192: 13.3
    // against 14.4; 16384 x 2048: 47.0 against 50.7); without it only 8-16
    // KiB rows in calls of 16-32 MiB (1024 x 8192: 9.3 against 10.0; from
    // 32 MiB up the five-block register kernel wins: 4096 x 8192 28.7 us
    // against 32.8, 4096 x 4096 15.4 against 16.4; 4096 x 2048 8.0 against
    // 8.7). Below 16 MiB the register kernels win (1024 x 4096: 7.1 against
    // 7.3 us); far above, the four-pack kernel matches it (16384 x 8192: 162
    // us both).
    const bool staged = kAdd ? packs >= 256 && input_bytes <= (int64_t{128} << 20)
                             : packs >= 512 && input_bytes < (int64_t{32} << 20);
    if (staged && packs <= 1024 && input_bytes >= (int64_t{16} << 20)) {
      family = Family::kStaged;
    } else if (packs <= 256) {
      family = a.rows >= 1024 ? Family::kCta : Family::kCtaOnePack;
    } else if (packs <= 1024) {
      family = Family::kCta;
    } else if (packs <= 2048) {
      family = Family::kBulk;
    } else {
      family = Family::kWide;
    }
  }
  if (family == Family::kWarp && packs > 8 * kWarpSize) family = Family::kCta;
  if ((family == Family::kCta || family == Family::kCtaOnePack) && packs > 1024) {
    family = Family::kWide;
  }
  if (family == Family::kStaged && (packs > 1024 || a.rows > INT32_MAX)) family = Family::kCta;

  switch (family) {
    case Family::kWarp:
      if (packs <= 1 * kWarpSize) return launch_warp<T, kAdd, 1>(a, stream);
      if (packs <= 2 * kWarpSize) return launch_warp<T, kAdd, 2>(a, stream);
      if (packs <= 4 * kWarpSize) return launch_warp<T, kAdd, 4>(a, stream);
      return launch_warp<T, kAdd, 8>(a, stream);
    case Family::kCtaOnePack:
      return launch_cta<T, kAdd, 1, 1024>(a, round_up_warps(packs), stream);
    case Family::kCta: {
      if (many_rows && packs >= 512) {
        // The weight is read from L1 per row rather than held in registers,
        // which leaves room for more blocks per SM (bit-identical results).
        // Measured on one B200, graphs of back-to-back calls on cold data,
        // against the weight in registers: with the residual add at three
        // blocks per SM, 65536 x 8192 bf16 620 us (663), fp16 619 (661),
        // 16384 x 8192 bf16 163 (172; four blocks per SM: no gain); without it
        // at five, 65536 x 8192 bf16 314 us (479; four blocks per SM 329),
        // 16384 x 8192 86 (four: 90.5), 32768 x 5120 105 (four: 106.5).
        if constexpr (kAdd) {
          return launch_cta<T, kAdd, 4, 256, 3, false>(a, round_up_warps((packs + 3) / 4), stream,
                                                       true);
        } else {
          return launch_cta<T, kAdd, 4, 256, 5, false>(a, round_up_warps((packs + 3) / 4), stream,
                                                       true);
        }
      }
      // Two packs per thread: 32+ bytes of loads in flight per thread with a
      // modest register budget.
      const int threads = round_up_warps((packs + 1) / 2);
      if (threads <= 256) {
        // Where the grid of blocks holding the weight in registers cannot take
        // every row at once, the weight is read from L1 per row instead: six
        // 256-thread blocks fit per SM rather than four, so fewer blocks make
        // a second pass (1024 x 4096 bf16 7.0 us against 7.25, 768 x 4096 5.6
        // against 5.8; the same threads and packs, so the same sums). Where
        // every row fits, the registers win: the weight's load then sits on
        // each block's one critical path (512 x 4096 3.85 us against 4.3).
        int grid = 0;
        int rc = persistent_grid(row_norm_cta_kernel<T, kAdd, 2, 512>, threads, a.rows, &grid);
        if (rc != SM120N_OK) return rc;
        if (a.rows > grid) return launch_cta<T, kAdd, 2, 256, 6, false>(a, threads, stream);
      }
      return launch_cta<T, kAdd, 2, 512>(a, threads, stream);
    }
    case Family::kStaged: {
      const int threads = round_up_warps((packs + 1) / 2);
      if (threads <= 256) return launch_staged<T, kAdd, 256>(a, threads, stream);
      return launch_staged<T, kAdd, 512>(a, threads, stream);
    }
    case Family::kBulk: {
      size_t block_smem = 0;
      int rc = max_block_smem(&block_smem);
      if (rc != SM120N_OK) return rc;
      BulkPlan plan;
      if (plan_bulk(a.hidden, sizeof(T), kAdd, 2, block_smem, &plan)) {
        return launch_bulk<T, kAdd, 2>(a, plan, stream);
      }
      if (plan_bulk(a.hidden, sizeof(T), kAdd, 4, block_smem, &plan)) {
        return launch_bulk<T, kAdd, 4>(a, plan, stream);
      }
      family = Family::kWide;  // rows too wide to stage: two-pass kernel
      [[fallthrough]];
    }
    case Family::kWide: {
      auto kernel = row_norm_wide_kernel<T, kAdd>;
      const int threads = 1024;
      int grid = 0;
      int rc = persistent_grid(kernel, threads, a.rows, &grid);
      if (rc != SM120N_OK) return rc;
      return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
    }
    case Family::kScalar:
    default: {
      auto kernel = row_norm_scalar_kernel<T, kAdd>;
      const int threads = 256;
      int grid = 0;
      int rc = persistent_grid(kernel, threads, a.rows, &grid);
      if (rc != SM120N_OK) return rc;
      return launch(kernel, dim3(grid), dim3(threads), 0, stream, a);
    }
  }
}

template <bool kAdd>
int run_rows_typed(int dtype, const void* input, const void* residual, const void* weight,
                   void* output, void* residual_output, int64_t rows, int64_t hidden,
                   float epsilon, Family family, cudaStream_t stream) {
  switch (dtype) {
    case SM120N_F32: {
      RowArgs<float> a{static_cast<const float*>(input), static_cast<const float*>(residual),
                       static_cast<const float*>(weight), static_cast<float*>(output),
                       static_cast<float*>(residual_output), rows, static_cast<int>(hidden),
                       epsilon, wait_poll_limit()};
      return run_rows<float, kAdd>(a, family, stream);
    }
    case SM120N_F16: {
      RowArgs<__half> a{static_cast<const __half*>(input), static_cast<const __half*>(residual),
                        static_cast<const __half*>(weight), static_cast<__half*>(output),
                        static_cast<__half*>(residual_output), rows, static_cast<int>(hidden),
                        epsilon, wait_poll_limit()};
      return run_rows<__half, kAdd>(a, family, stream);
    }
    default: {
      using B = __nv_bfloat16;
      RowArgs<B> a{static_cast<const B*>(input), static_cast<const B*>(residual),
                   static_cast<const B*>(weight), static_cast<B*>(output),
                   static_cast<B*>(residual_output), rows, static_cast<int>(hidden), epsilon,
                   wait_poll_limit()};
      return run_rows<B, kAdd>(a, family, stream);
    }
  }
}

int check_rows(int64_t rows, int64_t hidden, int dtype) {
  if (dtype_size(dtype) == 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "supported dtypes are float16, bfloat16, and float32");
  }
  if (rows < 0) return fail(SM120N_ERR_INVALID_ARGUMENT, "rows must be non-negative (got %lld)",
                            static_cast<long long>(rows));
  if (hidden <= 0 || hidden > (int64_t{1} << 30)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "hidden_size must be in [1, 2^30] (got %lld)",
                static_cast<long long>(hidden));
  }
  return SM120N_OK;
}

}  // namespace
}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_rms_norm(const void* input, const void* weight, void* output, int64_t rows,
                               int64_t hidden_size, int dtype, float epsilon, int version,
                               void* stream) {
  clear_error();
  int rc = check_rows(rows, hidden_size, dtype);
  if (rc != SM120N_OK) return rc;
  if (version != 1 && version != 2) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "RMSNorm version must be 1 or 2");
  }
  if (rows == 0) return SM120N_OK;
  if (!input || !weight || !output) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "input, weight and output must be non-null");
  }
  const Family family = version == 1 ? Family::kCta : Family::kAuto;
  return run_rows_typed<false>(dtype, input, nullptr, weight, output, nullptr, rows, hidden_size,
                               epsilon, family, static_cast<cudaStream_t>(stream));
}

extern "C" int sm120n_fused_add_rms_norm(const void* input, const void* residual,
                                         const void* weight, void* output, void* residual_output,
                                         int64_t rows, int64_t hidden_size, int dtype,
                                         float epsilon, int version, void* stream) {
  clear_error();
  int rc = check_rows(rows, hidden_size, dtype);
  if (rc != SM120N_OK) return rc;
  if (version < 0 || version > 4 || version == 1) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "fused version must be 0 (auto), 2, 3, or 4");
  }
  if (version == 3 && hidden_size != 1024) {
    return fail(SM120N_ERR_UNSUPPORTED, "V3 is specialized for hidden_size=1024");
  }
  if (version == 4 && hidden_size != 1024) {
    return fail(SM120N_ERR_UNSUPPORTED, "V4 is specialized for hidden_size=1024");
  }
  if (rows == 0) return SM120N_OK;
  if (!input || !residual || !weight || !output || !residual_output) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "input, residual, weight, output and residual_output must be non-null");
  }
  Family family = Family::kAuto;
  switch (version) {
    case 2: family = Family::kCta; break;
    case 3: family = Family::kWarp; break;
    case 4: family = Family::kCtaOnePack; break;
    default: break;
  }
  return run_rows_typed<true>(dtype, input, residual, weight, output, residual_output, rows,
                              hidden_size, epsilon, family, static_cast<cudaStream_t>(stream));
}

extern "C" int sm120n_get_device_faults(uint32_t* out_count) {
  clear_error();
  if (out_count == nullptr) return fail(SM120N_ERR_INVALID_ARGUMENT, "out_count must be non-null");
  unsigned int value = 0;
  const cudaError_t err = cudaMemcpyFromSymbol(&value, g_expired_waits, sizeof value);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "reading the fault counter failed: %s", cudaGetErrorString(err));
  }
  unsigned int gemm = 0;
  const int rc = read_gemm_faults(&gemm);
  if (rc != SM120N_OK) return rc;
  *out_count = value + gemm;
  return SM120N_OK;
}

extern "C" int sm120n_reset_device_faults(void) {
  clear_error();
  const unsigned int zero = 0;
  const cudaError_t err = cudaMemcpyToSymbol(g_expired_waits, &zero, sizeof zero);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "resetting the fault counter failed: %s", cudaGetErrorString(err));
  }
  return reset_gemm_faults();
}
