// qkv_gemm.cu -- the QKV projection of an attention layer on the sm_100
// tensor cores with the Q/K RMSNorm + RoPE + paged KV store fused into its
// epilogue; C-ABI entry point sm120n_qkv_proj_norm_rope_cache.
//
//   qkv[t, :] = hidden[t, :] @ qkv_weight.T          (bf16 in, fp32 accumulate,
//                                                      rounded to bf16)
// then, per 128-wide head of qkv (Hq query, Hk key, Hk value heads), exactly
// what fused_qk_rms_norm_rope_kv does to a bf16 [T, H, 128] tensor (reference
// project, csrc/rmsnorm_kernels.cu:611-709; math of sm120_rmsnorm/
// reference.py:27-49): RMSNorm rounded twice, half-split RoPE, rotated K and
// V stored at slot_mapping[t] of a [slots, Hk, 128] cache.
//
// Tiling, one SM per tile: one thread block per 128-token x kTileN-column
// tile (one or two heads), four warps. The K dimension streams through
// kStages shared-memory stages of 128-row (A) and kTileN-row (B) x 64-element
// boxes, loaded by the TMA engine with 128-byte swizzling (thread 0 of warp 0)
// and consumed by tcgen05.mma.kind::f16 (M 128, N kTileN, K 16; issued by
// thread 0 of warp 1) into kTileN columns of tensor memory. tcgen05.commit
// releases each stage back to the loader and finally signals the epilogue.
//
// Tiling, two SMs per tile (larger token counts): a cluster of two CTAs per
// 256-token x 256-column tile, tcgen05.mma.cta_group::2 (M 256, N 256), each
// CTA staging half of A and half of B in three stages, two pairs resident per
// two SMs (qkv_gemm_pair_kernel below). Persistent pairs (the fused calls
// from about 512 tokens): one cluster per two SMs walks the 256 x 256 tiles
// with warp-specialised loader, tensor-core issuer and four epilogue warps,
// six stages and two TMEM accumulators, so that each tile's epilogue runs
// under the next tile's main loop (qkv_gemm_persistent_kernel). The host
// picks the form per call from a measured wave model.
//
// Epilogue: warp w reads TMEM lanes 32(w % 4) onwards, i.e. each thread owns one
// token row of the tile and, per head, all 128 accumulators of that row. It
// rounds them to bf16 (the GEMM output), sums squares in the order the
// stand-alone Q/K kernel uses (eight 16-element lane slices, pairwise
// butterfly), and then applies the same normalise / rotate helpers, so the
// result is bit-identical to this kernel's plain GEMM followed by
// fused_qk_rms_norm_rope_kv / qk_norm_rope_cache_ on its output.
//
// Every wait on an mbarrier is bounded; an expired wait increments a device
// counter (read with sm120n_get_device_faults), the block skips the rest of
// its work (waiting, again bounded, for its own asynchronous operations) and
// releases its tensor memory.
#include <cooperative_groups.h>
#include <cuda.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <map>
#include <mutex>

#include "head_utils.cuh"
#include "runtime.h"

namespace sm120n {

__device__ unsigned int g_gemm_expired_waits = 0;

namespace {

constexpr int kTileM = 128;
constexpr int kTileK = 64;    // 128 bytes of bf16: one swizzle row
constexpr int kMmaK = 16;
constexpr int kHead = 128;
constexpr uint32_t kABytes = kTileM * kTileK * 2;  // 16 KiB

// Launch shape: kTileN output columns (one or two heads) per block, kStages
// pipeline stages, kWarps warps (4 or 8; with 8 the epilogue splits the heads
// of a tile over two warp groups that read the same TMEM lanes).
template <int kTileN, int kStages, int kWarps>
struct Shape {
  static constexpr int kThreads = kWarps * kWarpSize;
  static constexpr uint32_t kBBytes = kTileN * kTileK * 2;
  static constexpr uint32_t kStageBytes = kABytes + kBBytes;
  static constexpr int kTmemColumns = kTileN;  // fp32 accumulator columns
  static constexpr int kHeads = kTileN / kHead;
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kStageBytes + 1024;
  // Instruction descriptor of tcgen05.mma.kind::f16: fp32 accumulator
  // (bit 4), bf16 A and B (bits 7 and 10), both K-major, N >> 3 at bit 17,
  // M >> 4 at bit 24.
  static constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                         (static_cast<uint32_t>(kTileN >> 3) << 17) |
                                         (static_cast<uint32_t>(kTileM >> 4) << 24);
};

struct GemmArgs {
  __nv_bfloat16* qkv;  // [tokens, N] output
  const __nv_bfloat16* query_weight;
  const __nv_bfloat16* key_weight;
  const int64_t* positions;
  const float* cos_sin;
  __nv_bfloat16* key_cache;
  __nv_bfloat16* value_cache;
  const int32_t* slots;
  int64_t tokens;
  int64_t rope_positions;
  int64_t cache_slots;
  int k_tiles;
  int query_heads;
  int key_heads;
  int n;  // (Hq + 2Hk) * 128
  float epsilon;
  int epilogue;  // 0: store the bf16 GEMM output only; 1: norm + RoPE + cache
};

// ---- PTX wrappers ----------------------------------------------------------
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const CUtensorMap* map, int x, int y,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(shared_address(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(shared_address(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   shared_address(slot)),
               "r"(columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void mma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                         uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   shared_address(bar))
               : "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane.
__device__ __forceinline__ void tmem_load32(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor of a K-major, 128-byte-swizzled tile whose
// rows are 128 bytes and whose 8-row groups are 1024 bytes apart (the layout
// the TMA engine writes for a 64-element bf16 box with SWIZZLE_128B): start
// address >> 4 in bits [0, 14), leading offset 1 (unused for this layout) in
// [16, 30), stride offset 1024 >> 4 in [32, 46), descriptor version 1 at
// bit 46, layout 2 (128-byte swizzle) in [61, 64).
__device__ __forceinline__ uint64_t smem_descriptor(const void* tile) {
  const uint64_t address = shared_address(tile);
  return ((address & 0x3FFFFull) >> 4) | (uint64_t{1} << 16) | (uint64_t{1024 >> 4} << 32) |
         (uint64_t{1} << 46) | (uint64_t{2} << 61);
}

__device__ __forceinline__ bool wait_or_record(uint64_t* bar, uint32_t parity) {
  if (mbarrier_wait_bounded(bar, parity)) return true;
  atomicAdd(&g_gemm_expired_waits, 1u);
  return false;
}

// bf16 pair word of two fp32 accumulators (round to nearest even).
__device__ __forceinline__ uint32_t round_pair(uint32_t lo, uint32_t hi) {
  return Pack<__nv_bfloat16>::f32_to_word(__uint_as_float(lo), __uint_as_float(hi));
}

// One 128-wide head of this thread's row, rounded to bf16: 64 words, word i
// holding elements 2i and 2i + 1.
__device__ __forceinline__ void load_head(uint32_t taddr, uint32_t* words) {
#pragma unroll
  for (int chunk = 0; chunk < 4; ++chunk) {
    uint32_t acc[32];
    tmem_load32(taddr + chunk * 32, acc);
#pragma unroll
    for (int i = 0; i < 16; ++i) words[chunk * 16 + i] = round_pair(acc[2 * i], acc[2 * i + 1]);
  }
}

__device__ __forceinline__ Half8<__nv_bfloat16> chunk_of(const uint32_t* words, int element) {
  Half8<__nv_bfloat16> h;
#pragma unroll
  for (int i = 0; i < 4; ++i) h.w[i] = words[element / 2 + i];
  return h;
}

__device__ __forceinline__ void put_chunk(uint32_t* words, int element,
                                          const Half8<__nv_bfloat16>& h) {
#pragma unroll
  for (int i = 0; i < 4; ++i) words[element / 2 + i] = h.w[i];
}

__device__ __forceinline__ void store_head(__nv_bfloat16* dst, const uint32_t* words) {
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    store16(dst + 8 * i, make_uint4(words[4 * i], words[4 * i + 1], words[4 * i + 2],
                                    words[4 * i + 3]));
  }
}

// Per-head RMSNorm + RoPE of one row in place, bit-identical to
// head_norm_rope_kernel: lane slice j of that kernel holds elements
// [8j, 8j + 8) and [64 + 8j, 64 + 8j + 8); its sum of squares is formed per
// slice (even / odd accumulators) and combined by the butterfly 4, 2, 1.
__device__ __forceinline__ void norm_rope_head(uint32_t* words, const __nv_bfloat16* weight,
                                               const float* cos_sin_row, float epsilon) {
  float slice[8];
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float2 acc = half_sum_squares<__nv_bfloat16>(
        chunk_of(words, 64 + 8 * j),
        half_sum_squares<__nv_bfloat16>(chunk_of(words, 8 * j), make_float2(0.f, 0.f)));
    slice[j] = __fadd_rn(acc.x, acc.y);
  }
  float t[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) t[j] = __fadd_rn(slice[j], slice[j + 4]);
  const float total = __fadd_rn(__fadd_rn(t[0], t[2]), __fadd_rn(t[1], t[3]));
  const float inv = head_inverse_rms<kHead>(make_float2(total, 0.0f), epsilon);
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const int lo = 8 * j, hi = 64 + 8 * j;
    const Half8<__nv_bfloat16> n_lo =
        normalise_half<__nv_bfloat16>(chunk_of(words, lo), load_half<__nv_bfloat16, true>(weight + lo), inv);
    const Half8<__nv_bfloat16> n_hi =
        normalise_half<__nv_bfloat16>(chunk_of(words, hi), load_half<__nv_bfloat16, true>(weight + hi), inv);
    float2 c[4], s[4];
    load8_pairs<true>(cos_sin_row + lo, c);
    load8_pairs<true>(cos_sin_row + hi, s);
    Half8<__nv_bfloat16> y_lo, y_hi;
    rotate_half<__nv_bfloat16>(n_lo, n_hi, c, s, y_lo, y_hi);
    put_chunk(words, lo, y_lo);
    put_chunk(words, hi, y_hi);
  }
}

// Epilogue of one 128-token slab of a tile: warp w reads TMEM lanes
// 32 * (w % 4) onwards (one token row per thread) and the heads hh of the tile
// with hh % (kWarps / 4) == w / 4; the accumulators of head hh sit in columns
// [128 hh, 128 hh + 128).
template <int kHeads, int kWarps>
__device__ __forceinline__ void store_slab(const GemmArgs& a, uint32_t tmem_base, int warp,
                                           int lane, int64_t first_row, int first_head) {
  const int lane_group = warp % 4;
  const int head_group = warp / 4;
  const int64_t row = first_row + lane_group * 32 + lane;
  const bool live = row < a.tokens;
  int64_t position = -1;
  int64_t slot = -1;
  if (live && a.epilogue) {
    position = a.positions[row];
    slot = a.slots != nullptr ? a.slots[row] : -1;
    if (slot >= a.cache_slots) slot = -1;
  }
  const bool rope = position >= 0 && position < a.rope_positions;
#pragma unroll 1
  for (int hh = head_group; hh < kHeads; hh += kWarps / 4) {
    uint32_t words[64];
    load_head(tmem_base + (static_cast<uint32_t>(lane_group * 32) << 16) + hh * kHead, words);
    if (!live) continue;  // after the warp-wide TMEM load
    const int head = first_head + hh;
    __nv_bfloat16* out = a.qkv + row * a.n + static_cast<int64_t>(head) * kHead;
    if (a.epilogue && rope && head < a.query_heads + a.key_heads) {
      const bool is_query = head < a.query_heads;
      norm_rope_head(words, is_query ? a.query_weight : a.key_weight,
                     a.cos_sin + position * kHead, a.epsilon);
    }
    store_head(out, words);
    if (a.epilogue && rope && slot >= 0 && head >= a.query_heads) {
      const bool is_key = head < a.query_heads + a.key_heads;
      const int kv_head = is_key ? head - a.query_heads : head - a.query_heads - a.key_heads;
      __nv_bfloat16* cache = is_key ? a.key_cache : a.value_cache;
      store_head(cache + (slot * a.key_heads + kv_head) * kHead, words);
    }
  }
}

template <int kTileN, int kStages, int kWarps>
__global__ void __launch_bounds__(kWarps * kWarpSize, 1)
    qkv_gemm_kernel(const __grid_constant__ CUtensorMap map_a,
                    const __grid_constant__ CUtensorMap map_b, GemmArgs a) {
  using S = Shape<kTileN, kStages, kWarps>;
  extern __shared__ unsigned char dynamic_smem[];
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ int aborted;
  // 128-byte swizzled tiles need 1024-byte-aligned stages
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~uintptr_t{1023});
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int n_tile = blockIdx.x;
  const int m_tile = blockIdx.y;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    mbarrier_init(&done, 1);
    aborted = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, S::kTmemColumns);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  wait_for_upstream_grid();
  release_downstream_grid();

  if (warp == 0 && lane == 0) {
    // loader
    for (int k = 0; k < a.k_tiles; ++k) {
      const int s = k % kStages;
      if (k >= kStages && !wait_or_record(&empty[s], ((k / kStages) - 1) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      if (atomicAdd(&aborted, 0)) break;
      unsigned char* stage = tiles + static_cast<size_t>(s) * S::kStageBytes;
      mbarrier_arrive_expect_tx(&full[s], S::kStageBytes);
      tma_load_2d(stage, &map_a, k * kTileK, m_tile * kTileM, &full[s]);
      tma_load_2d(stage + kABytes, &map_b, k * kTileK, n_tile * kTileN, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    // tensor-core issuer
    int k = 0;
    for (; k < a.k_tiles; ++k) {
      const int s = k % kStages;
      if (!wait_or_record(&full[s], (k / kStages) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      tc_fence_after();
      const unsigned char* stage = tiles + static_cast<size_t>(s) * S::kStageBytes;
      const uint64_t adesc = smem_descriptor(stage);
      const uint64_t bdesc = smem_descriptor(stage + kABytes);
#pragma unroll
      for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
        // advance 16 elements (32 bytes, 2 descriptor units) along K
        mma_bf16(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, S::kInstrDesc, (k | kk) != 0);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(&done);  // fires once every MMA issued above has completed
  }
  __syncwarp();

  const bool ready = wait_or_record(&done, 0);
  tc_fence_after();
  if (ready && !aborted) {
    store_slab<S::kHeads, kWarps>(a, tmem_base, warp, lane, static_cast<int64_t>(m_tile) * kTileM,
                                  n_tile * S::kHeads);
  }
  // release tensor memory once every warp is past its loads; after an expired
  // wait, first give in-flight tensor-core work a bounded chance to finish
  tc_fence_before();
  __syncthreads();
  if (warp == 0) {
    if (!ready) {
      if (lane == 0) mbarrier_wait_bounded(&done, 0);
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, S::kTmemColumns);
  }
}

// ---- 2-SM form: one CTA pair per 256-token x 256-column tile ----------------
//
// A cluster of two CTAs on neighbouring SMs computes a 256 x 256 tile with
// tcgen05.mma.cta_group::2 (M 256, N 256, K 16). CTA r of the pair stages
// tokens [128 r, 128 r + 128) of the tile (A) and weight rows
// [128 r, 128 r + 128) of its 256 columns (B); the instruction, issued by
// CTA 0, reads both CTAs' shared memory and leaves in each CTA's tensor
// memory its own 128 token rows x all 256 columns. Per 64-element K step an
// SM therefore loads 32 KiB instead of the 48 KiB of the one-SM 128 x 256
// tile, for the same tensor-core work.
//
// Both CTAs' TMA loads complete on CTA 0's stage barrier (which expects the
// pair's 64 KiB); CTA 0's commits arrive on the stage-free and done barriers
// of both CTAs. Each CTA runs the one-SM epilogue on its own 128 rows.
constexpr int kPairTileM = 2 * kTileM;  // tokens per pair
constexpr int kPairTileN = 256;         // output columns per pair (two heads)
constexpr uint32_t kPairStageBytes = 2 * kABytes;  // per CTA: 128 x 64 of A and of B

template <int kStages>
struct PairShape {
  static constexpr int kThreads = 4 * kWarpSize;
  static constexpr int kTmemColumns = kPairTileN;
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kPairStageBytes + 1024;
  static constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                         (static_cast<uint32_t>(kPairTileN >> 3) << 17) |
                                         (static_cast<uint32_t>(kPairTileM >> 4) << 24);
};

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// All threads of both CTAs of the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// Address, in the cluster's shared window, of the variable at `local` in CTA `rank`.
__device__ __forceinline__ uint32_t peer_shared_address(const void* local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(shared_address(local)), "r"(rank));
  return r;
}

// TMA tile load into this CTA's shared memory whose completion is counted on
// `bar`, a barrier of either CTA of the pair (cluster shared address).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int x, int y,
                                                 uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(shared_address(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t columns) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   shared_address(slot)),
               "r"(columns)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t columns) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(columns)
               : "memory");
}

__device__ __forceinline__ void mma_bf16_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc,
                                              uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives on the barrier at `bar`'s offset in both CTAs of the pair once all
// tensor-core work issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  const uint16_t both = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(shared_address(bar)),
      "h"(both)
      : "memory");
}

template <int kStages>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(4 * kWarpSize, kStages <= 3 ? 2 : 1)
    qkv_gemm_pair_kernel(const __grid_constant__ CUtensorMap map_a,
                         const __grid_constant__ CUtensorMap map_b, GemmArgs a) {
  using S = PairShape<kStages>;
  extern __shared__ unsigned char dynamic_smem[];
  __shared__ __align__(8) uint64_t full[kStages];   // used in CTA 0 only
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ int aborted;
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~uintptr_t{1023});
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x & (kWarpSize - 1);
  const uint32_t rank = cluster_rank();
  const int n_tile = blockIdx.x / 2;
  const int m_pair = blockIdx.y;
  const int64_t first_row = static_cast<int64_t>(m_pair) * kPairTileM + rank * kTileM;
  // A CTA whose rows all lie past the end loads the last token rows instead
  // (its results are never stored), so that no box starts out of range.
  const int a_row = static_cast<int>(std::min<int64_t>(first_row, a.tokens - 1));
  const int b_row = n_tile * kPairTileN + static_cast<int>(rank) * kTileM;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    mbarrier_init(&done, 1);
    aborted = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc_pair(&tmem_slot, S::kTmemColumns);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  wait_for_upstream_grid();
  release_downstream_grid();

  if (warp == 0 && lane == 0) {
    // loader (both CTAs): this CTA's halves of A and B, counted on CTA 0's barrier
    for (int k = 0; k < a.k_tiles; ++k) {
      const int s = k % kStages;
      if (k >= kStages && !wait_or_record(&empty[s], ((k / kStages) - 1) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      if (atomicAdd(&aborted, 0)) break;
      unsigned char* stage = tiles + static_cast<size_t>(s) * kPairStageBytes;
      if (rank == 0) mbarrier_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
      const uint32_t bar = peer_shared_address(&full[s], 0);
      tma_load_2d_pair(stage, &map_a, k * kTileK, a_row, bar);
      tma_load_2d_pair(stage + kABytes, &map_b, k * kTileK, b_row, bar);
    }
  } else if (warp == 1 && lane == 0 && rank == 0) {
    // tensor-core issuer (CTA 0)
    for (int k = 0; k < a.k_tiles; ++k) {
      const int s = k % kStages;
      if (!wait_or_record(&full[s], (k / kStages) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      tc_fence_after();
      const unsigned char* stage = tiles + static_cast<size_t>(s) * kPairStageBytes;
      const uint64_t adesc = smem_descriptor(stage);
      const uint64_t bdesc = smem_descriptor(stage + kABytes);
#pragma unroll
      for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
        mma_bf16_pair(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, S::kInstrDesc, (k | kk) != 0);
      }
      mma_commit_pair(&empty[s]);
    }
    mma_commit_pair(&done);  // both CTAs, once every MMA issued above has completed
  }
  __syncwarp();

  const bool ready = wait_or_record(&done, 0);
  tc_fence_after();
  if (ready && !aborted) {
    store_slab<kPairTileN / kHead, 4>(a, tmem_base, warp, lane, first_row,
                                      n_tile * (kPairTileN / kHead));
  }
  // Both CTAs past their TMEM loads (and, after an expired wait, a bounded
  // chance for the pair's tensor-core work to finish) before the pair's
  // tensor memory is released; no CTA leaves while the other may still
  // signal its barriers or read its shared memory.
  tc_fence_before();
  __syncthreads();
  if (warp == 0 && !ready) {
    if (lane == 0) mbarrier_wait_bounded(&done, 0);
    __syncwarp();
  }
  cluster_sync();
  if (warp == 0) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemColumns);
  }
}

// ---- persistent 2-SM form: warp-specialised, two accumulators ------------------
//
// One cluster of two CTAs per pair of SMs walks the 256-token x 256-column
// tiles tile = cluster, cluster + clusters, ... (column tiles fastest, so
// the clusters working at once share token rows and the weights stay in L2).
// Roles: warp 0 lane 0 loads (as in the pair kernel: this CTA's halves of A
// and B, counted on CTA 0's stage barrier), warp 1 lane 0 of CTA 0 issues
// the tcgen05.mma.cta_group::2 of every tile, warps 2-5 of both CTAs run the
// epilogue (warp w reads TMEM lanes 32 (w % 4) onwards). Tensor memory holds
// two 256-column accumulators: the tensor cores fill one while the epilogue
// warps drain the other, so a tile's epilogue overlaps the next tile's main
// loop inside the same CTA (the pair kernel overlaps them only across two
// resident pairs). Barriers: full / empty per stage as in the pair kernel;
// acc_full[b] (both CTAs) fires when the tile in accumulator b is complete;
// acc_empty[b] (CTA 0) counts the eight epilogue warps of the pair that have
// read accumulator b.
constexpr int kPersistentStages = 6;
constexpr int kEpilogueWarps = 4;
constexpr int kPersistentThreads = (2 + kEpilogueWarps) * kWarpSize;
constexpr int kAccumulators = 2;

template <int kStages>
struct PersistentShape {
  static constexpr int kTmemColumns = kAccumulators * kPairTileN;  // all 512 columns
  static constexpr size_t kSmem = static_cast<size_t>(kStages) * kPairStageBytes + 1024;
};

// One arrival on the barrier at `bar`'s offset in CTA `rank` of the cluster.
__device__ __forceinline__ void mbarrier_arrive_cluster(uint64_t* bar, uint32_t rank) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(
                   peer_shared_address(bar, rank))
               : "memory");
}

__device__ __forceinline__ bool flag_set(const int* flag) {
  return *reinterpret_cast<const volatile int*>(flag) != 0;
}

template <int kStages>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kPersistentThreads, 1)
    qkv_gemm_persistent_kernel(const __grid_constant__ CUtensorMap map_a,
                               const __grid_constant__ CUtensorMap map_b, GemmArgs a,
                               int column_tiles, int tiles) {
  using S = PersistentShape<kStages>;
  extern __shared__ unsigned char dynamic_smem[];
  __shared__ __align__(8) uint64_t full[kStages];  // used in CTA 0 only
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ __align__(8) uint64_t acc_full[kAccumulators];
  __shared__ __align__(8) uint64_t acc_empty[kAccumulators];  // used in CTA 0 only
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ int aborted;
  unsigned char* tiles_smem = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~uintptr_t{1023});
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x & (kWarpSize - 1);
  const uint32_t rank = cluster_rank();
  const int cluster = static_cast<int>(blockIdx.x / 2);
  const int clusters = static_cast<int>(gridDim.x / 2);

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    for (int b = 0; b < kAccumulators; ++b) {
      mbarrier_init(&acc_full[b], 1);
      mbarrier_init(&acc_empty[b], 2 * kEpilogueWarps);
    }
    mbarrier_init(&done, 1);
    aborted = 0;
    fence_mbarrier_init();
  }
  if (warp == 1) tmem_alloc_pair(&tmem_slot, S::kTmemColumns);
  tc_fence_before();
  cluster_sync();  // barriers of both CTAs initialised, the pair's TMEM allocated
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  wait_for_upstream_grid();
  release_downstream_grid();

  if (warp == 0) {
    if (lane == 0) {
      // loader (both CTAs)
      int step = 0;
      for (int tile = cluster; tile < tiles && !flag_set(&aborted); tile += clusters) {
        const int m_pair = tile / column_tiles;
        const int n_tile = tile - m_pair * column_tiles;
        const int64_t first_row = static_cast<int64_t>(m_pair) * kPairTileM + rank * kTileM;
        // rows past the end load the last token rows (never stored)
        const int a_row = static_cast<int>(std::min<int64_t>(first_row, a.tokens - 1));
        const int b_row = n_tile * kPairTileN + static_cast<int>(rank) * kTileM;
        for (int k = 0; k < a.k_tiles; ++k, ++step) {
          const int s = step % kStages;
          if (step >= kStages && !wait_or_record(&empty[s], ((step / kStages) - 1) & 1)) {
            atomicExch(&aborted, 1);
            break;
          }
          unsigned char* stage = tiles_smem + static_cast<size_t>(s) * kPairStageBytes;
          if (rank == 0) mbarrier_arrive_expect_tx(&full[s], 2 * kPairStageBytes);
          const uint32_t bar = peer_shared_address(&full[s], 0);
          tma_load_2d_pair(stage, &map_a, k * kTileK, a_row, bar);
          tma_load_2d_pair(stage + kABytes, &map_b, k * kTileK, b_row, bar);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      // tensor-core issuer (CTA 0)
      constexpr uint32_t kInstrDesc = PairShape<3>::kInstrDesc;
      int step = 0, local = 0;
      for (int tile = cluster; tile < tiles && !flag_set(&aborted); tile += clusters, ++local) {
        const int b = local % kAccumulators;
        if (local >= kAccumulators &&
            !wait_or_record(&acc_empty[b], ((local / kAccumulators) - 1) & 1)) {
          atomicExch(&aborted, 1);
          break;
        }
        tc_fence_after();
        const uint32_t accumulator = tmem_base + static_cast<uint32_t>(b * kPairTileN);
        bool ok = true;
        for (int k = 0; k < a.k_tiles; ++k, ++step) {
          const int s = step % kStages;
          if (!wait_or_record(&full[s], (step / kStages) & 1)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const unsigned char* stage = tiles_smem + static_cast<size_t>(s) * kPairStageBytes;
          const uint64_t adesc = smem_descriptor(stage);
          const uint64_t bdesc = smem_descriptor(stage + kABytes);
#pragma unroll
          for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
            mma_bf16_pair(accumulator, adesc + 2 * kk, bdesc + 2 * kk, kInstrDesc, (k | kk) != 0);
          }
          mma_commit_pair(&empty[s]);
        }
        if (!ok) {
          atomicExch(&aborted, 1);
          break;
        }
        mma_commit_pair(&acc_full[b]);  // both CTAs, once this tile's MMAs have completed
      }
      mma_commit_pair(&done);
    }
  } else {
    // epilogue (warps 2-5 of both CTAs)
    const int lane_group = warp % 4;
    int local = 0;
    for (int tile = cluster; tile < tiles; tile += clusters, ++local) {
      const int b = local % kAccumulators;
      if (!wait_or_record(&acc_full[b], (local / kAccumulators) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      tc_fence_after();
      const int m_pair = tile / column_tiles;
      const int n_tile = tile - m_pair * column_tiles;
      const int64_t first_row = static_cast<int64_t>(m_pair) * kPairTileM + rank * kTileM;
      store_slab<kPairTileN / kHead, 4>(a, tmem_base + static_cast<uint32_t>(b * kPairTileN),
                                        lane_group, lane, first_row,
                                        n_tile * (kPairTileN / kHead));
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbarrier_arrive_cluster(&acc_empty[b], 0);
    }
  }
  __syncwarp();

  // Teardown: every CTA waits (bounded) for the issuer's last commit, which
  // follows all of the pair's tensor-core work, so no arrival is still on
  // its way; then no CTA leaves while the other may still signal its
  // barriers, and the pair's TMEM is released.
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    if (lane == 0) mbarrier_wait_bounded(&done, 0);
    __syncwarp();
  }
  cluster_sync();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, S::kTmemColumns);
  }
}

// ---- Q/K epilogue of one head row on eight lanes -------------------------------
//
// For the kernels that finish a head row from a bf16 copy of it in shared
// memory: eight lanes per row, lane part p holding elements [8p, 8p + 8) and
// [64 + 8p, 64 + 8p + 8), with head_norm_rope_kernel's sum order, norm,
// rotation and KV store, so the result is that kernel's on the row. fetch_*
// are split so that a kernel can issue the loads early.
struct HeadRow {
  int64_t position = -1;
  int64_t slot = -1;
  bool live = false;
  bool rope = false;
  bool norm = false;
  float2 c[4], sn[4];
  Half8<__nv_bfloat16> nw_lo{}, nw_hi{};
};

__device__ __forceinline__ void head_row_fetch_token(HeadRow& r, const GemmArgs& a, bool live,
                                                     int64_t token) {
  r.live = live;
  if (live && a.epilogue) {
    r.position = a.positions[token];
    r.slot = a.slots != nullptr ? a.slots[token] : -1;
  }
}

__device__ __forceinline__ void head_row_fetch_tables(HeadRow& r, const GemmArgs& a, int head,
                                                      int part) {
  if (r.slot >= a.cache_slots) r.slot = -1;
  r.rope = r.position >= 0 && r.position < a.rope_positions;
  r.norm = r.live && a.epilogue && r.rope && head < a.query_heads + a.key_heads;
  if (r.norm) {
    const int lo = 8 * part;
    const int hi = kHead / 2 + lo;
    const __nv_bfloat16* nw = head < a.query_heads ? a.query_weight : a.key_weight;
    r.nw_lo = load_half<__nv_bfloat16, true>(nw + lo);
    r.nw_hi = load_half<__nv_bfloat16, true>(nw + hi);
    load8_pairs<true>(a.cos_sin + r.position * kHead + lo, r.c);
    load8_pairs<true>(a.cos_sin + r.position * kHead + hi, r.sn);
  }
}

// All eight lanes of every group must call (the sum of squares is a shuffle).
__device__ __forceinline__ void head_row_finish(const HeadRow& r, const GemmArgs& a, int head,
                                                int64_t token, int part,
                                                const __nv_bfloat16* row) {
  const int lo = 8 * part;
  const int hi = kHead / 2 + lo;
  Half8<__nv_bfloat16> x_lo{}, x_hi{};
  if (r.live) {
    x_lo = load_half<__nv_bfloat16, true>(row + lo);
    x_hi = load_half<__nv_bfloat16, true>(row + hi);
  }
  const float2 sq = half_sum_squares<__nv_bfloat16>(
      x_hi, half_sum_squares<__nv_bfloat16>(x_lo, make_float2(0.f, 0.f)));
  const float total = group_allreduce_sum<8>(__fadd_rn(sq.x, sq.y));
  Half8<__nv_bfloat16> y_lo = x_lo, y_hi = x_hi;
  if (r.norm) {
    const float inv = head_inverse_rms<kHead>(make_float2(total, 0.0f), a.epsilon);
    const Half8<__nv_bfloat16> n_lo = normalise_half<__nv_bfloat16>(x_lo, r.nw_lo, inv);
    const Half8<__nv_bfloat16> n_hi = normalise_half<__nv_bfloat16>(x_hi, r.nw_hi, inv);
    rotate_half<__nv_bfloat16>(n_lo, n_hi, r.c, r.sn, y_lo, y_hi);
  }
  if (r.live) {
    __nv_bfloat16* out = a.qkv + token * a.n + static_cast<int64_t>(head) * kHead;
    store_half<__nv_bfloat16, true>(out + lo, y_lo);
    store_half<__nv_bfloat16, true>(out + hi, y_hi);
    if (a.epilogue && r.rope && r.slot >= 0 && head >= a.query_heads) {
      const bool is_key = head < a.query_heads + a.key_heads;
      const int kv_head = is_key ? head - a.query_heads : head - a.query_heads - a.key_heads;
      __nv_bfloat16* cache =
          (is_key ? a.key_cache : a.value_cache) + (r.slot * a.key_heads + kv_head) * kHead;
      store_half<__nv_bfloat16, true>(cache + lo, y_lo);
      store_half<__nv_bfloat16, true>(cache + hi, y_hi);
    }
  }
}

// ---- split K for a few dozen tokens ----------------------------------------
//
// Up to 128 tokens give only one 128-token row of one-head tiles (N / 128
// blocks), each streaming its 128 weight rows through the whole K. Here a
// cluster of kSplits CTAs shares one such tile: CTA s runs the one-SM main
// loop (TMA, tcgen05.mma M128 N128 into 128 TMEM columns) over K tiles
// [s, s + 1) * K / kSplits, copies its fp32 partial tile from TMEM into its
// shared memory (rows padded to 132 floats: conflict-free 16-byte accesses),
// and after a cluster barrier CTA s sums rows [s, s + 1) * 128 / kSplits of
// the kSplits partials, in rank order, through distributed shared memory,
// rounds them to bf16 and runs the Q/K epilogue on eight lanes per row. Three
// stages keep two CTAs per SM (the partial tile and the reduced rows reuse
// the stage memory).
constexpr int kSplitRowFloats = kHead + 4;
constexpr uint32_t kSplitPartialBytes = kTileM * kSplitRowFloats * sizeof(float);

template <int kSplits, int kStages>
struct SplitShape {
  static constexpr int kThreads = 4 * kWarpSize;
  static constexpr uint32_t kStageBytes = 2 * kABytes;  // 128 x 64 of A and of B
  static constexpr int kRows = kTileM / kSplits;       // rows each CTA finishes
  // after the main loop the stage memory holds the fp32 partial tile and,
  // behind it, this CTA's reduced bf16 rows
  static constexpr size_t kAfterLoop = kSplitPartialBytes + kRows * kHead * 2;
  static constexpr size_t kSmem =
      (static_cast<size_t>(kStages) * kStageBytes > kAfterLoop
           ? static_cast<size_t>(kStages) * kStageBytes
           : kAfterLoop) + 1024;
  static constexpr uint32_t kInstrDesc = (1u << 4) | (1u << 7) | (1u << 10) |
                                         (static_cast<uint32_t>(kHead >> 3) << 17) |
                                         (static_cast<uint32_t>(kTileM >> 4) << 24);
  static_assert(kRows * 8 % kThreads == 0, "whole epilogue passes");
};

template <int kSplits, int kStages>
__global__ void __launch_bounds__(4 * kWarpSize, 2)
    qkv_gemm_splitk_kernel(const __grid_constant__ CUtensorMap map_a,
                           const __grid_constant__ CUtensorMap map_b, GemmArgs a) {
  namespace cg = cooperative_groups;
  using S = SplitShape<kSplits, kStages>;
  extern __shared__ unsigned char dynamic_smem[];
  __shared__ __align__(8) uint64_t full[kStages];
  __shared__ __align__(8) uint64_t empty[kStages];
  __shared__ __align__(8) uint64_t done;
  __shared__ uint32_t tmem_slot;
  __shared__ int aborted;
  __shared__ int cta_ok;  // this CTA's main loop completed; read by every CTA of the cluster
  unsigned char* tiles = reinterpret_cast<unsigned char*>(
      (reinterpret_cast<uintptr_t>(dynamic_smem) + 1023) & ~uintptr_t{1023});
  float* partial = reinterpret_cast<float*>(tiles);  // after the main loop
  auto rows = reinterpret_cast<__nv_bfloat16(*)[kHead]>(tiles + kSplitPartialBytes);
  cg::cluster_group cluster = cg::this_cluster();
  const int rank = static_cast<int>(cluster.block_rank());
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int n_tile = blockIdx.x / kSplits;  // = head
  const int m_tile = blockIdx.y;
  const int k_count = a.k_tiles / kSplits;
  const int k_first = rank * k_count;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbarrier_init(&full[s], 1);
      mbarrier_init(&empty[s], 1);
    }
    mbarrier_init(&done, 1);
    aborted = 0;
    fence_mbarrier_init();
  }
  if (warp == 0) tmem_alloc(&tmem_slot, kHead);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = tmem_slot;
  wait_for_upstream_grid();
  release_downstream_grid();

  if (warp == 0 && lane == 0) {
    for (int k = 0; k < k_count; ++k) {
      const int s = k % kStages;
      if (k >= kStages && !wait_or_record(&empty[s], ((k / kStages) - 1) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      if (atomicAdd(&aborted, 0)) break;
      unsigned char* stage = tiles + static_cast<size_t>(s) * S::kStageBytes;
      mbarrier_arrive_expect_tx(&full[s], S::kStageBytes);
      tma_load_2d(stage, &map_a, (k_first + k) * kTileK, m_tile * kTileM, &full[s]);
      tma_load_2d(stage + kABytes, &map_b, (k_first + k) * kTileK, n_tile * kHead, &full[s]);
    }
  } else if (warp == 1 && lane == 0) {
    for (int k = 0; k < k_count; ++k) {
      const int s = k % kStages;
      if (!wait_or_record(&full[s], (k / kStages) & 1)) {
        atomicExch(&aborted, 1);
        break;
      }
      tc_fence_after();
      const unsigned char* stage = tiles + static_cast<size_t>(s) * S::kStageBytes;
      const uint64_t adesc = smem_descriptor(stage);
      const uint64_t bdesc = smem_descriptor(stage + kABytes);
#pragma unroll
      for (int kk = 0; kk < kTileK / kMmaK; ++kk) {
        mma_bf16(tmem_base, adesc + 2 * kk, bdesc + 2 * kk, S::kInstrDesc, (k | kk) != 0);
      }
      mma_commit(&empty[s]);
    }
    mma_commit(&done);
  }
  __syncwarp();

  // the tokens this CTA finishes: rows rank * kRows .. + kRows of the tile
  constexpr int kPasses = S::kRows * 8 / S::kThreads;
  HeadRow job[kPasses];
#pragma unroll
  for (int p = 0; p < kPasses; ++p) {
    const int r = (p * S::kThreads + threadIdx.x) / 8;
    const int64_t t = static_cast<int64_t>(m_tile) * kTileM + rank * S::kRows + r;
    head_row_fetch_token(job[p], a, t < a.tokens, t);
  }

  // this CTA's fp32 partial tile into shared memory (stages are free: every
  // load was consumed by an MMA that has completed)
  const bool ready = wait_or_record(&done, 0);
  tc_fence_after();
  if (ready) {
    const int row = warp * kWarpSize + lane;
    float* dst = partial + row * kSplitRowFloats;
#pragma unroll 1
    for (int chunk = 0; chunk < kHead / 32; ++chunk) {
      uint32_t v[32];
      tmem_load32(tmem_base + (static_cast<uint32_t>(warp * kWarpSize) << 16) + chunk * 32, v);
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        reinterpret_cast<float4*>(dst + chunk * 32)[q] =
            make_float4(__uint_as_float(v[4 * q]), __uint_as_float(v[4 * q + 1]),
                        __uint_as_float(v[4 * q + 2]), __uint_as_float(v[4 * q + 3]));
      }
    }
  }
#pragma unroll
  for (int p = 0; p < kPasses; ++p) head_row_fetch_tables(job[p], a, n_tile, lane & 7);
  const int ok = __syncthreads_and(ready && !aborted);
  if (threadIdx.x == 0) cta_ok = ok;
  cluster.sync();  // every CTA's partial tile and verdict are in place

  // The rows are finished only if every CTA of the cluster completed its
  // slice: a CTA whose wait expired wrote no partial tile (its expiry is in
  // the fault counter), and its siblings must not sum what is in its place.
  bool cluster_ok = true;
#pragma unroll
  for (int s = 0; s < kSplits; ++s) cluster_ok = cluster_ok && *cluster.map_shared_rank(&cta_ok, s);

  // sum the partials of this CTA's rows in rank order
  for (int idx = threadIdx.x; cluster_ok && idx < S::kRows * kHead / 4; idx += S::kThreads) {
    const int r = idx / (kHead / 4);
    const int col = (idx - r * (kHead / 4)) * 4;
    const int offset = (rank * S::kRows + r) * kSplitRowFloats + col;
    float4 sum = *reinterpret_cast<const float4*>(cluster.map_shared_rank(partial + offset, 0));
#pragma unroll
    for (int s = 1; s < kSplits; ++s) {
      const float4 v = *reinterpret_cast<const float4*>(cluster.map_shared_rank(partial + offset, s));
      sum = make_float4(__fadd_rn(sum.x, v.x), __fadd_rn(sum.y, v.y), __fadd_rn(sum.z, v.z),
                        __fadd_rn(sum.w, v.w));
    }
    reinterpret_cast<uint32_t*>(&rows[r][col])[0] = Pack<__nv_bfloat16>::f32_to_word(sum.x, sum.y);
    reinterpret_cast<uint32_t*>(&rows[r][col])[1] = Pack<__nv_bfloat16>::f32_to_word(sum.z, sum.w);
  }
  __syncthreads();
  if (cluster_ok) {
#pragma unroll
    for (int p = 0; p < kPasses; ++p) {
      const int r = (p * S::kThreads + threadIdx.x) / 8;
      const int64_t t = static_cast<int64_t>(m_tile) * kTileM + rank * S::kRows + r;
      head_row_finish(job[p], a, n_tile, t, lane & 7, rows[r]);
    }
  }
  tc_fence_before();
  cluster.sync();  // no CTA leaves while another may still read its partial tile
  if (warp == 0) {
    if (!ready) {
      if (lane == 0) mbarrier_wait_bounded(&done, 0);
      __syncwarp();
    }
    tc_fence_after();
    tmem_dealloc(tmem_base, kHead);
  }
}

// ---- weight streaming for a few tokens -------------------------------------
//
// With at most kGemvMaxTokens tokens the projection only has to stream the
// weight matrix once (2 N K bytes), which the tensor-core tiles do at far
// below the HBM rate. Here a cluster of kGemvSplits CTAs owns one head (128
// weight rows) and CTA s reduces K slice s of all 128 rows for every token.
// Lane j = lane % 8 of lane group g = lane / 8 in warp w owns rows
// 16w + 4i + g (i = 0..3) and, in each of them, the 16-byte chunks at
// k = 64m + 8j of the slice (eight lanes cover 128 contiguous bytes). The
// chunks stream through a ring of kGemvRing phases in shared memory by
// cp.async (no registers held while in flight): phase m brings chunk m of
// each of the lane's four rows, the next phases are in flight while one is
// used. Each chunk is multiplied with the tokens' activations (bf16 in
// shared memory, read once per chunk for all four rows) in a fused
// multiply-add chain in element order, chunks in K order, and the eight
// lanes of a row combine by the butterfly 4, 2, 1. The slices' partial sums
// stay in each CTA's shared memory; after a cluster barrier CTA s sums, for
// its tokens (t % kGemvSplits == s), the partials of CTAs 0, 1, ... in that
// order through distributed shared memory, rounds to bf16 and runs the Q/K
// epilogue with eight lanes per head row exactly as head_norm_rope_kernel
// does. Every summation order is fixed, so the fused and the plain result of
// this path agree bit for bit with its own output followed by the Q/K kernel.
constexpr int kGemvSplits = 8;
constexpr int kGemvThreads = 256;  // 8 warps x 16 rows = one head
constexpr int kGemvMaxTokens = 4;
constexpr int kGemvMaxSlice = 1024;  // K / kGemvSplits, a multiple of 64
constexpr int kGemvRing = 4;         // phases in flight
// one phase: one 16-byte chunk of each of the thread's 4 rows
constexpr uint32_t kGemvPhaseBytes = 4 * 16 * kGemvThreads;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gmem_src) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(shared_address(smem_dst)),
               "l"(gmem_src)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() {
  asm volatile("cp.async.commit_group;" ::: "memory");
}
template <int kPending>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(kPending) : "memory");
}

template <int kTokens>
__global__ void __launch_bounds__(kGemvThreads, 3) qkv_gemv_kernel(const __nv_bfloat16* hidden,
                                                                  const __nv_bfloat16* weight,
                                                                  GemmArgs a, int hidden_size) {
  namespace cg = cooperative_groups;
  // dynamic: kGemvRing phases of kGemvPhaseBytes, then [kTokens][slice] bf16
  extern __shared__ uint4 gemv_dynamic[];
  __shared__ float partial[kTokens][kHead];
  __shared__ __align__(16) __nv_bfloat16 rows[kTokens][kHead];
  cg::cluster_group cluster = cg::this_cluster();
  const int split = static_cast<int>(cluster.block_rank());
  const int splits = static_cast<int>(cluster.num_blocks());
  const int head = blockIdx.y;
  const int warp = threadIdx.x / kWarpSize;
  const int lane = threadIdx.x & (kWarpSize - 1);
  const int g = lane >> 3;
  const int j = lane & 7;
  const int tokens = static_cast<int>(a.tokens);
  const int slice = hidden_size / splits;
  const int chunks = slice / 64;  // per lane and row
  const int64_t k0 = static_cast<int64_t>(split) * slice;
  unsigned char* ring = reinterpret_cast<unsigned char*>(gemv_dynamic);
  __nv_bfloat16* xs = reinterpret_cast<__nv_bfloat16*>(ring + kGemvRing * kGemvPhaseBytes);

  // Ask for this CTA's 128 weight-row slices in L2 at once (a prefetch
  // returns no data, so it may precede the wait for the upstream grid: L2
  // stays coherent with any write that grid makes).
  if (threadIdx.x < kHead) {
    const __nv_bfloat16* w_slice =
        weight + (static_cast<int64_t>(head) * kHead + threadIdx.x) * hidden_size + k0;
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(w_slice),
                 "r"(static_cast<uint32_t>(slice * sizeof(__nv_bfloat16)))
                 : "memory");
  }
  wait_for_upstream_grid();
  release_downstream_grid();

  // The epilogue's lanes (eight per head row this CTA finishes: tokens
  // t = split, split + splits, ...) fetch their token's position and slot
  // now and the cos/sin row and norm weights right after the main loop, so
  // that none of these loads is on the path after the cluster barrier.
  const int mine = tokens > split ? (tokens - split + splits - 1) / splits : 0;
  const bool epilogue_warp = warp * kWarpSize < mine * 8;
  const int er = threadIdx.x / 8;  // head row of an epilogue lane
  const int et = split + er * splits;
  HeadRow job;
  head_row_fetch_token(job, a, epilogue_warp && er < mine, et);

  // this thread's rows: 16 warp + 4 i + g; its chunk m of row i sits at
  // ring + (m % kGemvRing) * kGemvPhaseBytes + (i * kGemvThreads + threadIdx.x) * 16.
  // Every phase commits a group (an empty one past the last chunk), so
  // waiting for all but kGemvRing - 1 groups always means phase m has landed.
  const __nv_bfloat16* w_lane =
      weight + (static_cast<int64_t>(head) * kHead + 16 * warp + g) * hidden_size + k0 + 8 * j;
  auto issue = [&](int m) {
    if (m < chunks) {
      unsigned char* stage = ring + (m % kGemvRing) * kGemvPhaseBytes;
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        cp_async16(stage + (i * kGemvThreads + threadIdx.x) * 16,
                   w_lane + static_cast<int64_t>(4 * i) * hidden_size + 64 * m);
      }
    }
    cp_async_commit();
  };
#pragma unroll
  for (int m = 0; m < kGemvRing; ++m) issue(m);

  // this slice of every token's activations (zero past the last token)
  for (int i = threadIdx.x; i < kTokens * (slice / 8); i += kGemvThreads) {
    const int t = i / (slice / 8);
    const int c = (i - t * (slice / 8)) * 8;
    uint4 v = make_uint4(0, 0, 0, 0);
    if (t < tokens) v = load16(hidden + static_cast<int64_t>(t) * hidden_size + k0 + c);
    *reinterpret_cast<uint4*>(xs + t * slice + c) = v;
  }
  __syncthreads();

  float acc[4][kTokens];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int t = 0; t < kTokens; ++t) acc[i][t] = 0.0f;
  }
#pragma unroll 1
  for (int m = 0; m < chunks; ++m) {
    cp_async_wait<kGemvRing - 1>();
    const unsigned char* stage = ring + (m % kGemvRing) * kGemvPhaseBytes;
    float2 wf[4][4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 raw = *reinterpret_cast<const uint4*>(stage + (i * kGemvThreads + threadIdx.x) * 16);
      Half8<__nv_bfloat16> h;
      h.w[0] = raw.x; h.w[1] = raw.y; h.w[2] = raw.z; h.w[3] = raw.w;
      unpack_pairs<__nv_bfloat16>(h, wf[i]);
    }
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      const uint4 raw = *reinterpret_cast<const uint4*>(xs + t * slice + 64 * m + 8 * j);
      Half8<__nv_bfloat16> h;
      h.w[0] = raw.x; h.w[1] = raw.y; h.w[2] = raw.z; h.w[3] = raw.w;
      float2 xf[4];
      unpack_pairs<__nv_bfloat16>(h, xf);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        float v = acc[i][t];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          v = __fmaf_rn(wf[i][e].x, xf[e].x, v);
          v = __fmaf_rn(wf[i][e].y, xf[e].y, v);
        }
        acc[i][t] = v;
      }
    }
    // this thread alone reads and refills its slots of the stage
    issue(m + kGemvRing);
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
#pragma unroll
    for (int t = 0; t < kTokens; ++t) {
      const float total = group_allreduce_sum<8>(acc[i][t]);
      if (j == 0) partial[t][16 * warp + 4 * i + g] = total;
    }
  }
  head_row_fetch_tables(job, a, head, j);
  cluster.sync();  // every CTA's partial sums are in place

  // sum the splits' partials of each token this CTA finishes, in rank order
  for (int idx = threadIdx.x; idx < mine * kHead; idx += kGemvThreads) {
    const int r = idx / kHead;
    const int col = idx - r * kHead;
    const int t = split + r * splits;
    float sum = *cluster.map_shared_rank(&partial[t][col], 0);
    for (int s = 1; s < splits; ++s) sum = __fadd_rn(sum, *cluster.map_shared_rank(&partial[t][col], s));
    rows[r][col] = __float2bfloat16_rn(sum);
  }
  __syncthreads();

  // Q/K epilogue, eight lanes per head row (head_norm_rope_kernel's lane map)
  if (epilogue_warp) head_row_finish(job, a, head, et, j, rows[er < mine ? er : 0]);
  cluster.sync();  // no CTA leaves while another may still read its partial sums
}

// ---- host ----------------------------------------------------------------
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder(int* rc) {
  static std::once_flag once;
  static PFN_cuTensorMapEncodeTiled_v12000 encode = nullptr;
  static cudaError_t status = cudaSuccess;
  std::call_once(once, [] {
    cudaDriverEntryPointQueryResult query;
    status = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", reinterpret_cast<void**>(&encode),
                                     cudaEnableDefault, &query);
    if (status == cudaSuccess && query != cudaDriverEntryPointSuccess) status = cudaErrorNotSupported;
  });
  *rc = status == cudaSuccess && encode != nullptr
            ? SM120N_OK
            : fail(SM120N_ERR_CUDA, "cuTensorMapEncodeTiled is not available: %s",
                   cudaGetErrorString(status));
  return encode;
}

// Row-major [rows, cols] bf16 matrix as a TMA map with a 64 x box_rows box,
// 128-byte swizzle; rows past the end read as zeros.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  int rc = SM120N_OK;
  auto encode = tensor_map_encoder(&rc);
  if (rc != SM120N_OK) return rc;
  const cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  const cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols) * 2};
  const cuuint32_t box[2] = {static_cast<cuuint32_t>(kTileK), static_cast<cuuint32_t>(box_rows)};
  const cuuint32_t element_strides[2] = {1, 1};
  const CUresult r = encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                            strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                            CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    return fail(SM120N_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  }
  return SM120N_OK;
}

template <int kTileN, int kStages, int kWarps>
int launch_gemm(const CUtensorMap& map_a, const void* qkv_weight, int64_t n, int64_t hidden_size,
                const GemmArgs& a, int64_t tokens, cudaStream_t stream) {
  using S = Shape<kTileN, kStages, kWarps>;
  CUtensorMap map_b;
  int rc = make_map(&map_b, qkv_weight, n, hidden_size, kTileN);
  if (rc != SM120N_OK) return rc;
  auto kernel = qkv_gemm_kernel<kTileN, kStages, kWarps>;
  rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), S::kSmem);
  if (rc != SM120N_OK) return rc;
  const dim3 grid(static_cast<unsigned>(n / kTileN),
                  static_cast<unsigned>((tokens + kTileM - 1) / kTileM));
  return launch(kernel, grid, dim3(S::kThreads), S::kSmem, stream, map_a, map_b, a);
}

template <int kStages>
int launch_gemm_pair(const CUtensorMap& map_a, const void* qkv_weight, int64_t n,
                     int64_t hidden_size, const GemmArgs& a, int64_t tokens, cudaStream_t stream) {
  using S = PairShape<kStages>;
  CUtensorMap map_b;
  int rc = make_map(&map_b, qkv_weight, n, hidden_size, kTileM);
  if (rc != SM120N_OK) return rc;
  auto kernel = qkv_gemm_pair_kernel<kStages>;
  rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), S::kSmem);
  if (rc != SM120N_OK) return rc;
  const dim3 grid(static_cast<unsigned>(2 * (n / kPairTileN)),
                  static_cast<unsigned>((tokens + kPairTileM - 1) / kPairTileM));
  return launch(kernel, grid, dim3(S::kThreads), S::kSmem, stream, map_a, map_b, a);
}

// Clusters of qkv_gemm_persistent_kernel<kStages> resident at once on
// `device` (the current device; one CTA per SM), cached per device: the
// runtime's cluster occupancy, at most SMs / 2.
template <int kStages>
int persistent_clusters(int device, int sms, int* out) {
  static std::mutex mutex;
  static std::map<int, int> cache;
  std::lock_guard<std::mutex> lock(mutex);
  auto it = cache.find(device);
  if (it != cache.end()) {
    *out = it->second;
    return SM120N_OK;
  }
  using S = PersistentShape<kStages>;
  auto kernel = qkv_gemm_persistent_kernel<kStages>;
  int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), S::kSmem);
  if (rc != SM120N_OK) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(sms / 2 * 2));
  config.blockDim = dim3(kPersistentThreads);
  config.dynamicSmemBytes = S::kSmem;
  int clusters = 0;
  const cudaError_t err = cudaOccupancyMaxActiveClusters(&clusters, kernel, &config);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "querying the projection kernel's cluster occupancy failed: %s",
                cudaGetErrorString(err));
  }
  clusters = std::max(1, std::min(clusters, sms / 2));
  cache[device] = clusters;
  *out = clusters;
  return SM120N_OK;
}

template <int kStages>
int launch_gemm_persistent(const CUtensorMap& map_a, const void* qkv_weight, int64_t n,
                           int64_t hidden_size, const GemmArgs& a, int64_t tokens, int clusters,
                           cudaStream_t stream) {
  using S = PersistentShape<kStages>;
  CUtensorMap map_b;
  int rc = make_map(&map_b, qkv_weight, n, hidden_size, kTileM);
  if (rc != SM120N_OK) return rc;
  auto kernel = qkv_gemm_persistent_kernel<kStages>;
  rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), S::kSmem);
  if (rc != SM120N_OK) return rc;
  const int column_tiles = static_cast<int>(n / kPairTileN);
  const int64_t tiles = column_tiles * ((tokens + kPairTileM - 1) / kPairTileM);
  const int64_t grid_clusters = std::min<int64_t>(tiles, clusters);
  return launch(kernel, dim3(static_cast<unsigned>(2 * grid_clusters)), dim3(kPersistentThreads),
                S::kSmem, stream, map_a, map_b, a, column_tiles, static_cast<int>(tiles));
}

template <int kSplits, int kStages>
int launch_gemm_splitk(const CUtensorMap& map_a, const void* qkv_weight, int64_t n,
                       int64_t hidden_size, const GemmArgs& a, int64_t tokens, cudaStream_t stream) {
  using S = SplitShape<kSplits, kStages>;
  CUtensorMap map_b;
  int rc = make_map(&map_b, qkv_weight, n, hidden_size, kTileM);
  if (rc != SM120N_OK) return rc;
  auto kernel = qkv_gemm_splitk_kernel<kSplits, kStages>;
  rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), S::kSmem);
  if (rc != SM120N_OK) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(static_cast<unsigned>(kSplits * (n / kHead)),
                        static_cast<unsigned>((tokens + kTileM - 1) / kTileM));
  config.blockDim = dim3(S::kThreads);
  config.dynamicSmemBytes = S::kSmem;
  config.stream = stream;
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = kSplits;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  if (programmatic_launch_enabled()) {
    attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[1].val.programmaticStreamSerializationAllowed = 1;
    config.numAttrs = 2;
  }
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, map_a, map_b, a);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(err));
  }
  return SM120N_OK;
}

template <int kTokens>
int launch_gemv(const void* hidden, const void* qkv_weight, const GemmArgs& a, int64_t n,
                int64_t hidden_size, cudaStream_t stream) {
  auto kernel = qkv_gemv_kernel<kTokens>;
  const size_t smem = kGemvRing * kGemvPhaseBytes +
                      static_cast<size_t>(kTokens) * (hidden_size / kGemvSplits) * sizeof(__nv_bfloat16);
  int rc = allow_dynamic_smem(reinterpret_cast<const void*>(kernel), smem);
  if (rc != SM120N_OK) return rc;
  cudaLaunchConfig_t config = {};
  config.gridDim = dim3(kGemvSplits, static_cast<unsigned>(n / kHead));
  config.blockDim = dim3(kGemvThreads);
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[2];
  attribute[0].id = cudaLaunchAttributeClusterDimension;
  attribute[0].val.clusterDim.x = kGemvSplits;
  attribute[0].val.clusterDim.y = 1;
  attribute[0].val.clusterDim.z = 1;
  config.attrs = attribute;
  config.numAttrs = 1;
  if (programmatic_launch_enabled()) {
    attribute[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[1].val.programmaticStreamSerializationAllowed = 1;
    config.numAttrs = 2;
  }
  const cudaError_t err =
      cudaLaunchKernelEx(&config, kernel, static_cast<const __nv_bfloat16*>(hidden),
                         static_cast<const __nv_bfloat16*>(qkv_weight), a,
                         static_cast<int>(hidden_size));
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(err));
  }
  return SM120N_OK;
}

// CTA pairs of qkv_gemm_pair_kernel<kStages> resident at once on `device`
// (the current device), cached per device: SMs x blocks per SM / 2, blocks
// per SM limited by shared memory, registers and tensor memory (512
// columns). Computed from the kernel's resources because the runtime's
// cluster occupancy query reports one pair per two SMs for this kernel,
// while ncu's launch statistics show two blocks per SM (register and shared
// memory limits 2, 7.8 of 8 warps active).
template <int kStages>
int resident_pairs(int device, int* out) {
  static std::mutex mutex;
  static std::map<int, int> cache;
  {
    std::lock_guard<std::mutex> lock(mutex);
    auto it = cache.find(device);
    if (it != cache.end()) {
      *out = it->second;
      return SM120N_OK;
    }
  }
  using S = PairShape<kStages>;
  cudaFuncAttributes attributes;
  cudaError_t err = cudaFuncGetAttributes(&attributes, qkv_gemm_pair_kernel<kStages>);
  int sms = 0, smem_per_sm = 0, reserved = 0, regs_per_sm = 0;
  if (err == cudaSuccess) err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
  if (err == cudaSuccess) {
    err = cudaDeviceGetAttribute(&smem_per_sm, cudaDevAttrMaxSharedMemoryPerMultiprocessor, device);
  }
  if (err == cudaSuccess) {
    err = cudaDeviceGetAttribute(&reserved, cudaDevAttrReservedSharedMemoryPerBlock, device);
  }
  if (err == cudaSuccess) {
    err = cudaDeviceGetAttribute(&regs_per_sm, cudaDevAttrMaxRegistersPerMultiprocessor, device);
  }
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "querying the projection kernel's resources failed: %s",
                cudaGetErrorString(err));
  }
  const int64_t smem_per_block =
      static_cast<int64_t>(S::kSmem) + static_cast<int64_t>(attributes.sharedSizeBytes) + reserved;
  const int64_t regs_per_block = static_cast<int64_t>((attributes.numRegs + 7) / 8 * 8) * S::kThreads;
  const int64_t per_sm = std::max<int64_t>(
      1, std::min({static_cast<int64_t>(smem_per_sm) / smem_per_block,
                   static_cast<int64_t>(regs_per_sm) / regs_per_block,
                   static_cast<int64_t>(512 / S::kTmemColumns)}));
  const int pairs = static_cast<int>(std::max<int64_t>(1, sms * per_sm / 2));
  std::lock_guard<std::mutex> lock(mutex);
  cache[device] = pairs;
  *out = pairs;
  return SM120N_OK;
}

}  // namespace

int read_gemm_faults(unsigned int* value) {
  const cudaError_t err = cudaMemcpyFromSymbol(value, g_gemm_expired_waits, sizeof *value);
  return err == cudaSuccess ? SM120N_OK
                            : fail(SM120N_ERR_CUDA, "reading the fault counter failed: %s",
                                   cudaGetErrorString(err));
}

int reset_gemm_faults() {
  const unsigned int zero = 0;
  const cudaError_t err = cudaMemcpyToSymbol(g_gemm_expired_waits, &zero, sizeof zero);
  return err == cudaSuccess ? SM120N_OK
                            : fail(SM120N_ERR_CUDA, "resetting the fault counter failed: %s",
                                   cudaGetErrorString(err));
}

}  // namespace sm120n

using namespace sm120n;

extern "C" int sm120n_qkv_proj_norm_rope_cache(
    const void* hidden, const void* qkv_weight, void* qkv, int64_t tokens, int64_t hidden_size,
    int64_t query_heads, int64_t key_heads, const void* query_weight, const void* key_weight,
    const int64_t* positions, const float* cos_sin_cache, int64_t rope_positions,
    void* key_cache, void* value_cache, const int32_t* slot_mapping, int64_t cache_slots,
    float epsilon, int epilogue, void* stream) {
  clear_error();
  if (tokens < 0 || query_heads < 0 || key_heads < 0 || rope_positions < 0 || cache_slots < 0) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "sizes must be non-negative");
  }
  if (epilogue != 0 && epilogue != 1) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "epilogue must be 0 (GEMM only) or 1");
  }
  const int64_t heads = query_heads + 2 * key_heads;
  if (heads <= 0 || heads % 2 != 0 || heads > 4096) {
    return fail(SM120N_ERR_UNSUPPORTED,
                "the fused projection needs an even number of heads (query + 2 * key), "
                "at most 4096 (got %lld)", static_cast<long long>(heads));
  }
  if (hidden_size <= 0 || hidden_size % kTileK != 0 || hidden_size > (int64_t{1} << 20)) {
    return fail(SM120N_ERR_UNSUPPORTED,
                "hidden_size must be a positive multiple of 64 up to 2^20 (got %lld)",
                static_cast<long long>(hidden_size));
  }
  if (tokens > INT32_MAX - kTileM) return fail(SM120N_ERR_INVALID_ARGUMENT, "too many tokens");
  if (tokens == 0) return SM120N_OK;
  if (!hidden || !qkv_weight || !qkv) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "hidden, qkv_weight and qkv must be non-null");
  }
  if (epilogue && (!query_weight || !key_weight || !positions || !cos_sin_cache)) {
    return fail(SM120N_ERR_INVALID_ARGUMENT,
                "the norm epilogue needs query/key weights, positions and the cos/sin cache");
  }
  if (epilogue && key_heads > 0 && slot_mapping &&
      (cache_slots > 0 && (!key_cache || !value_cache))) {
    return fail(SM120N_ERR_INVALID_ARGUMENT, "a KV store needs key_cache and value_cache");
  }
  if (!aligned16(hidden) || !aligned16(qkv_weight) || !aligned16(qkv) ||
      (epilogue && (!aligned16(query_weight) || !aligned16(key_weight) ||
                    !aligned16(cos_sin_cache) || (key_cache && !aligned16(key_cache)) ||
                    (value_cache && !aligned16(value_cache))))) {
    return fail(SM120N_ERR_UNSUPPORTED, "the fused projection needs 16-byte-aligned buffers");
  }
  const int64_t n = heads * kHead;
  GemmArgs a{static_cast<__nv_bfloat16*>(qkv),
             static_cast<const __nv_bfloat16*>(query_weight),
             static_cast<const __nv_bfloat16*>(key_weight),
             positions,
             cos_sin_cache,
             static_cast<__nv_bfloat16*>(key_cache),
             static_cast<__nv_bfloat16*>(value_cache),
             epilogue ? slot_mapping : nullptr,
             tokens,
             rope_positions,
             (key_cache && value_cache) ? cache_slots : 0,
             static_cast<int>(hidden_size / kTileK),
             static_cast<int>(query_heads),
             static_cast<int>(key_heads),
             static_cast<int>(n),
             epsilon,
             epilogue};
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  // Up to four tokens stream the weights on the CUDA cores (2 N K bytes,
  // HBM-bound); hidden a multiple of 512 up to 8192 (eight slices of whole
  // 64-element chunks).
  if (tokens <= kGemvMaxTokens && hidden_size % (64 * kGemvSplits) == 0 &&
      hidden_size / kGemvSplits <= kGemvMaxSlice) {
    if (tokens == 1) return launch_gemv<1>(hidden, qkv_weight, a, n, hidden_size, st);
    if (tokens == 2) return launch_gemv<2>(hidden, qkv_weight, a, n, hidden_size, st);
    return launch_gemv<4>(hidden, qkv_weight, a, n, hidden_size, st);
  }
  CUtensorMap map_a;
  int rc = make_map(&map_a, hidden, tokens, hidden_size, kTileM);
  if (rc != SM120N_OK) return rc;
  // The launch form comes from a wave model measured on B200 (Qwen3-8B-shaped
  // projection, N = 6144, K = 4096, graphs of back-to-back calls), in ns:
  // with tiles resident at once on the device, a launch takes
  // ceil(tiles / resident) waves; one 64-element K step of a wave costs
  // about 470 ns for 128 x 128 tiles (one block per SM, six stages), 570 for
  // 128 x 256 tiles (one block per SM, four stages), 850 for 256 x 256 tiles
  // on CTA pairs (two pairs per two SMs, three stages) and, for one-head
  // tiles split along K over a cluster (two CTAs per SM), 380 (four ways)
  // and 450 (two ways) per step of the whole K; the Q/K epilogue adds 3.0,
  // 5.5, 15, 1.4 and 1.3 us per wave. The persistent pairs take
  // ceil(tiles / clusters) rounds of 420 ns per K step, plus 12 us (fill,
  // the cold weights, drain) and 3 us for the epilogue of the last tiles
  // (the others overlap the next tile's main loop). Splitting a last,
  // partial round into one-head units did not shorten it (1024 tokens:
  // 63.6 us either way; 4096: 169 against 165): a K step of a unit costs
  // about the same at N 128 as at N 256. The cheapest estimate wins: 5-128
  // tokens four-way split K (16-128 tokens: 24.6-25.4 us against 30.7-32.8
  // unsplit; eight ways 32.6-33.6 us), 129-384 two-way split K (256 tokens:
  // 32.7 us, 34.0 us with the Q/K epilogue, against 34.4 / 36.9 on one-head
  // tiles); above that, with the Q/K epilogue, the persistent pairs (512:
  // 45-47 us against 47 on two-head tiles; 2048: 92-100 against 125-130 on
  // pairs; 4096: 168-178 against 193-197; 32768: 1188-1231 against 1328;
  // 1024: 68-70 against 70-75 for one wave of pairs); the plain GEMM takes
  // two-head tiles at 512-768 tokens, pairs at 1024-1300 and at 4096 (one
  // wave of pairs against two rounds at 1024: 55-60 against 60-64 us), the
  // persistent pairs at 2048 and from 8192 tokens.
  DeviceInfo dev;
  rc = current_device_info(&dev);
  if (rc != SM120N_OK) return rc;
  int pairs = 1;
  rc = resident_pairs<3>(dev.device, &pairs);
  if (rc != SM120N_OK) return rc;
  const int64_t sms = dev.sm_count;
  int clusters = 1;
  rc = persistent_clusters<kPersistentStages>(dev.device, static_cast<int>(sms), &clusters);
  if (rc != SM120N_OK) return rc;
  const int64_t m128 = (tokens + kTileM - 1) / kTileM;
  const int64_t m256 = (tokens + kPairTileM - 1) / kPairTileM;
  const int64_t k_steps = hidden_size / kTileK;
  auto waves = [](int64_t tiles, int64_t slots) {
    return (tiles + slots - 1) / std::max<int64_t>(slots, 1);
  };
  struct Costs {
    int64_t one_head, two_heads, pair, persistent, split4, split2;
  };
  auto costs = [&](int64_t fused) {
    Costs c;
    c.one_head = waves(m128 * (n / 128), sms) * (470 * k_steps + 3000 * fused);
    c.two_heads = waves(m128 * (n / 256), sms) * (570 * k_steps + 5500 * fused);
    c.pair = waves(m256 * (n / kPairTileN), pairs) * (850 * k_steps + 15000 * fused);
    c.persistent = waves(m256 * (n / kPairTileN), clusters) * 420 * k_steps + 12000 + 3000 * fused;
    c.split4 = k_steps % 4 == 0
                   ? waves(m128 * (n / kHead) * 4, 2 * sms) * (380 * k_steps + 1400 * fused)
                   : INT64_MAX;
    c.split2 = k_steps % 2 == 0
                   ? waves(m128 * (n / kHead) * 2, 2 * sms) * (450 * k_steps + 1300 * fused)
                   : INT64_MAX;
    return c;
  };
  // The summation order -- K split four ways, two ways, or not at all --
  // follows from the plain GEMM's costs, so that a fused call rounds exactly
  // like the plain GEMM followed by the stand-alone Q/K kernel; the
  // epilogue's cost then picks among the unsplit forms, which all sum K in
  // the same order (16-element tensor-core steps, K ascending).
  const Costs plain = costs(0);
  const int64_t unsplit = std::min({plain.one_head, plain.two_heads, plain.pair, plain.persistent});
  if (plain.split4 < unsplit && plain.split4 <= plain.split2) {
    return launch_gemm_splitk<4, 3>(map_a, qkv_weight, n, hidden_size, a, tokens, st);
  }
  if (plain.split2 < unsplit) {
    return launch_gemm_splitk<2, 3>(map_a, qkv_weight, n, hidden_size, a, tokens, st);
  }
  const Costs c = epilogue ? costs(1) : plain;
  const int64_t best = std::min({c.one_head, c.two_heads, c.pair, c.persistent});
  if (c.persistent == best) {
    return launch_gemm_persistent<kPersistentStages>(map_a, qkv_weight, n, hidden_size, a, tokens,
                                                     clusters, st);
  }
  if (c.one_head == best) {
    return launch_gemm<128, 6, 4>(map_a, qkv_weight, n, hidden_size, a, tokens, st);
  }
  if (c.two_heads == best) {
    return launch_gemm<256, 4, 4>(map_a, qkv_weight, n, hidden_size, a, tokens, st);
  }
  return launch_gemm_pair<3>(map_a, qkv_weight, n, hidden_size, a, tokens, st);
}
