/*
 * sm120norm_b200.h -- C ABI of the B200 (sm_100a) fused normalisation kernels.
 *
 * Plain pointers, sizes and an opaque CUDA stream; no torch types. Every entry
 * point validates its scalar arguments, launches on the CURRENT CUDA device
 * (cudaSetDevice of the calling thread) on the given stream, never
 * synchronises, never allocates, and returns an sm120n_status. On failure a
 * human-readable message for the calling thread is available from
 * sm120n_last_error(); the messages reuse the reference's TORCH_CHECK texts
 * where the reference tests match them ("hidden_size=1024", "head_dim=128").
 *
 * Each function names the reference host launcher it replaces (paths are
 * relative to the reference project, FILWYZ/sm120-norm-fusion-kernels).
 *
 * Memory layout (all tensors dense, row-major, device memory):
 *   rows x hidden activations        element (i, j) at  base + i*hidden + j
 *   [tokens, heads, 128] Q / K / V   element (t, h, d) at base + (t*heads + h)*128 + d
 *   cos_sin_cache [rope_positions, 128] fp32: cos in [0, 64), sin in [64, 128)
 *   key/value cache [cache_slots, key_heads, 128]; a paged cache
 *   [blocks, block_size, key_heads, 128] is the same memory with
 *   slot = block * block_size + offset.
 *
 * Aliasing: output may equal input and residual_output may equal residual
 * (the in-place form). Any other overlap between buffers is undefined.
 *
 * The last four entry points (sm120n_qk_norm_rope_cache,
 * sm120n_rms_norm_fp8_quant, sm120n_rms_norm_fp4_quant,
 * sm120n_qkv_proj_norm_rope_cache) go beyond the reference's surface: they
 * serve an
 * inference engine around the same hot path (general head sizes and partial
 * rotary, Q/K/V as strided views of one QKV projection output, NHD / HND
 * paged caches, fp8 KV caches, RMSNorm feeding an fp8 or NVFP4 GEMM, the QKV
 * projection with the Q/K norm in its epilogue). Their math is
 * the reference's, generalised; each states its exact definition.
 */
#ifndef SM120NORM_B200_H_
#define SM120NORM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SM120N_ABI_VERSION 5

#if defined(__GNUC__)
#define SM120N_API __attribute__((visibility("default")))
#else
#define SM120N_API
#endif

/* Element type of activations, weights, outputs and KV caches. */
typedef enum sm120n_dtype {
  SM120N_F32 = 0,
  SM120N_F16 = 1,
  SM120N_BF16 = 2
} sm120n_dtype;

typedef enum sm120n_status {
  SM120N_OK = 0,
  SM120N_ERR_INVALID_ARGUMENT = 1, /* null pointer, bad size, bad dtype, bad version */
  SM120N_ERR_UNSUPPORTED = 2,      /* valid request this kernel family does not cover */
  SM120N_ERR_CUDA = 3              /* a CUDA runtime call or launch failed */
} sm120n_status;

/* Version of this ABI (SM120N_ABI_VERSION of the built library). */
SM120N_API int sm120n_abi_version(void);

/* Message describing the last failing call made by this thread ("" if none). */
SM120N_API const char* sm120n_last_error(void);

/* Static name of a status code. */
SM120N_API const char* sm120n_status_string(int status);

/*
 * Programmatic dependent launch: when enabled (the default), kernels are
 * launched with the programmatic-stream-serialisation attribute so their
 * launch overlaps the tail of the preceding kernel on the stream. Every kernel
 * waits for the preceding grid to complete before touching global memory, so
 * results do not depend on this switch. Process-wide.
 */
SM120N_API void sm120n_set_programmatic_launch(int enabled);
SM120N_API int sm120n_get_programmatic_launch(void);

/*
 * Number of bounded waits that expired in kernels on the current device since
 * the last sm120n_reset_device_faults(). Zero in correct operation; non-zero
 * means a pipelined kernel gave up waiting on its own asynchronous copies and
 * skipped the affected rows. Synchronises the current device.
 */
SM120N_API int sm120n_get_device_faults(uint32_t* out_count);
SM120N_API int sm120n_reset_device_faults(void);

/*
 * Diagnostic: the number of polls a kernel makes while waiting for its own
 * bulk copies (the row kernels that stage rows in shared memory) to land
 * before it gives up, records an expired wait in the fault counter and
 * leaves its rows unwritten. 0 restores the default (2^22 polls, far
 * beyond any real copy); values above it are clamped to it. Lowering it lets
 * a test make the bound expire without faulting or hanging anything: the
 * kernel still waits, with the full bound, for its copies to land before it
 * exits. Process-wide; no reference counterpart (the reference has no
 * asynchronous copies).
 */
SM120N_API void sm120n_set_wait_limit(uint32_t polls);
SM120N_API uint32_t sm120n_get_wait_limit(void);

/*
 * RMSNorm: output[i, :] = round(x[i, :] * (1 / sqrt(mean(x[i, :]^2) + eps)) * weight)
 * with fp32 accumulation. version 1 or 2 (2 = B200 shape dispatch).
 * Replaces rms_norm_out_cuda, csrc/rmsnorm_kernels.cu:482-524 (and
 * rms_norm_cuda :472-480, whose allocation stays with the caller).
 */
SM120N_API int sm120n_rms_norm(const void* input, const void* weight, void* output,
                    int64_t rows, int64_t hidden_size, int dtype,
                    float epsilon, int version, void* stream);

/*
 * Residual add + RMSNorm:
 *   residual_output = round(input + residual)
 *   output          = round(residual_output * inv_rms(residual_output) * weight)
 * version 0 (B200 shape dispatch), 2 (any hidden size), 3 or 4 (hidden_size
 * 1024 only; other sizes fail with "... hidden_size=1024").
 * In place: pass output == input and residual_output == residual.
 * Replaces fused_add_rms_norm_out_cuda, csrc/rmsnorm_kernels.cu:724-801,
 * fused_add_rms_norm_inplace_cuda :526-537 and fused_add_rms_norm_cuda
 * :711-722.
 */
SM120N_API int sm120n_fused_add_rms_norm(const void* input, const void* residual,
                              const void* weight, void* output,
                              void* residual_output, int64_t rows,
                              int64_t hidden_size, int dtype, float epsilon,
                              int version, void* stream);

/*
 * Per-head Q/K RMSNorm + half-split RoPE, in place on query and key:
 *   n = round(round(x * inv_rms(x)) * w)          (two roundings, as the
 *                                                   reference oracle does)
 *   y[i]    = round(n[i] * cos[i] - n[i+64] * sin[i])
 *   y[i+64] = round(n[i+64] * cos[i] + n[i] * sin[i]),  i < 64,
 *   cos/sin = cos_sin_cache[positions[t]].
 * head_dim must be 128. version 1 or 2. A token whose position lies outside
 * [0, rope_positions) is left unchanged.
 * Replaces fused_qk_rms_norm_rope_cuda, csrc/rmsnorm_kernels.cu:539-609.
 */
SM120N_API int sm120n_fused_qk_rms_norm_rope(void* query, void* key,
                                  const void* query_weight,
                                  const void* key_weight,
                                  const int64_t* positions,
                                  const float* cos_sin_cache, int64_t tokens,
                                  int64_t query_heads, int64_t key_heads,
                                  int64_t head_dim, int64_t rope_positions,
                                  int dtype, float epsilon, int version,
                                  void* stream);

/*
 * As sm120n_fused_qk_rms_norm_rope, plus the paged KV store: for each token
 * with 0 <= slot_mapping[t] < cache_slots,
 *   key_cache[slot, h, :]   = rotated key[t, h, :]   (bit-identical)
 *   value_cache[slot, h, :] = value[t, h, :]         (bit-identical).
 * Negative slots (padding) and slots >= cache_slots write nothing.
 * version 1 or 4 (warps per thread block).
 * Replaces fused_qk_rms_norm_rope_kv_cuda, csrc/rmsnorm_kernels.cu:611-709.
 */
SM120N_API int sm120n_fused_qk_rms_norm_rope_kv(
    void* query, void* key, const void* value, const void* query_weight,
    const void* key_weight, const int64_t* positions,
    const float* cos_sin_cache, void* key_cache, void* value_cache,
    const int32_t* slot_mapping, int64_t tokens, int64_t query_heads,
    int64_t key_heads, int64_t head_dim, int64_t rope_positions,
    int64_t cache_slots, int dtype, float epsilon, int version, void* stream);

/* ------------------------------------------------------------------------
 * Extensions (not in the reference's surface)
 * ------------------------------------------------------------------------ */

/* Pairing of rotated elements. NEOX: (i, i + rotary_dim/2), the reference's
 * half split. INTERLEAVED: (2i, 2i + 1). Both use cos/sin index i. */
typedef enum sm120n_rope_style {
  SM120N_ROPE_NEOX = 0,
  SM120N_ROPE_INTERLEAVED = 1
} sm120n_rope_style;

/* Element type of a KV cache: AUTO = the activation dtype (bit copies),
 * FP8_E4M3 = float8 e4m3fn, stored as sat(x / scale) rounded to nearest even,
 * saturating at +-448. */
typedef enum sm120n_cache_dtype {
  SM120N_CACHE_AUTO = 0,
  SM120N_CACHE_FP8_E4M3 = 1
} sm120n_cache_dtype;

/*
 * Arguments of sm120n_qk_norm_rope_cache. Sizes and strides in elements.
 *   query  [tokens, query_heads, head_dim], token t at query + t*query_token_stride,
 *          heads adjacent (stride head_dim); likewise key and value, so Q, K and
 *          V may be views into one [tokens, (Hq + 2*Hk) * head_dim] buffer.
 *   query_weight, key_weight [head_dim]; positions int64 [tokens];
 *   cos_sin_cache fp32 [rope_positions, rotary_dim] (cos | sin halves).
 *   key_cache / value_cache: NULL for no store. Slot s = slot_mapping[t] in
 *   [0, num_blocks * block_size) goes to block s / block_size, offset
 *   s % block_size; head h of that slot starts at
 *     block * cache_block_stride + offset * cache_slot_stride + h * cache_head_stride
 *   in both caches (NHD [blocks, block_size, Hk, D]: strides (block_size*Hk*D,
 *   Hk*D, D); HND [blocks, Hk, block_size, D]: (Hk*block_size*D, D,
 *   block_size*D)). Other slots write nothing.
 *   k_scale / v_scale: device fp32 scalars, required for FP8_E4M3 caches.
 */
typedef struct sm120n_qk_cache_args {
  uint32_t struct_size; /* sizeof(sm120n_qk_cache_args) */
  int32_t dtype;        /* sm120n_dtype of Q, K, V and the weights */
  int64_t tokens;
  int64_t query_heads;
  int64_t key_heads;
  int64_t head_dim;   /* 64, 128 or 256 */
  int64_t rotary_dim; /* multiple of 16 in [16, head_dim] */
  int32_t rope_style; /* sm120n_rope_style */
  int32_t cache_dtype; /* sm120n_cache_dtype */
  void* query;
  int64_t query_token_stride;
  void* key;
  int64_t key_token_stride;
  const void* value;
  int64_t value_token_stride;
  const void* query_weight;
  const void* key_weight;
  const int64_t* positions;
  const float* cos_sin_cache;
  int64_t rope_positions;
  void* key_cache;
  void* value_cache;
  const int32_t* slot_mapping;
  int64_t num_blocks;
  int64_t block_size;
  int64_t cache_block_stride;
  int64_t cache_slot_stride;
  int64_t cache_head_stride;
  const float* k_scale;
  const float* v_scale;
  float epsilon;
} sm120n_qk_cache_args;

/*
 * Generalised Q/K RMSNorm + RoPE + KV store, in place on query and key:
 *   n = round(round(x * inv_rms(x)) * w) over all head_dim elements,
 *   the first rotary_dim elements rotated in fp32 as in
 *   sm120n_fused_qk_rms_norm_rope (style chosen by rope_style), the rest
 *   passed through as n, everything rounded to the activation dtype;
 *   then, with caches, key_cache[slot, h] = rotated key (AUTO: bit copy),
 *   value_cache[slot, h] = value. With head_dim = rotary_dim = 128, NEOX,
 *   dense strides and an AUTO NHD cache this is bit-identical to
 *   sm120n_fused_qk_rms_norm_rope_kv. Tokens with positions outside
 *   [0, rope_positions) are left unchanged and store nothing.
 * Generalises csrc/rmsnorm_kernels.cu:611-709 (fused_qk_rms_norm_rope_kv_cuda),
 * whose checks :632-633 restrict it to head_dim 128 and a dense NHD cache.
 */
SM120N_API int sm120n_qk_norm_rope_cache(const sm120n_qk_cache_args* args, void* stream);

/*
 * RMSNorm (optionally after a residual add) with an fp8 e4m3fn output:
 *   s = residual ? round(input + residual) : input   (residual_output = s)
 *   y = round(s * inv_rms(s) * weight)                (sm120n_rms_norm's y)
 *   static  (scale != NULL):  q = sat(y * (1 / scale[0]))
 *   dynamic (scale == NULL):  a = max|y| of the row (min(a, scale_ub[0]) when
 *                             scale_ub != NULL); token_scales[row] =
 *                             max(a / 448, 1 / (448 * 512));
 *                             q = sat(y * (1 / token_scales[row]))
 *   sat(v): v clamped to [-448, 448] and rounded to the nearest e4m3fn value
 *   (ties to even); 1 / x is the correctly rounded fp32 reciprocal.
 * y follows the rounding sequence of sm120n_rms_norm / sm120n_fused_add_rms_norm
 * (only the order of the fp32 sum of squares may differ); y itself is not
 * written. output is [rows, hidden_size] bytes; residual_output may equal
 * residual.
 * No reference counterpart: the fp8 activation quantisation that follows
 * rms_norm_out_cuda (csrc/rmsnorm_kernels.cu:482-524) and
 * fused_add_rms_norm_out_cuda (:724-801) in an fp8 inference engine.
 */
SM120N_API int sm120n_rms_norm_fp8_quant(const void* input, const void* residual,
                              const void* weight, void* residual_output,
                              void* output, const float* scale,
                              float* token_scales, const float* scale_ub,
                              int64_t rows, int64_t hidden_size, int dtype,
                              float epsilon, void* stream);

/* Layout of NVFP4 block scales (one e4m3 byte per 16 elements of a row).
 * ROW_MAJOR: [rows, hidden / 16]. TILED_128X4: the layout block-scaled
 * tensor-core GEMMs read -- rows padded to a multiple of 128 and blocks to a
 * multiple of 4; the (row / 128, block / 4) tiles follow each other row of
 * tiles by row of tiles, and inside a 512-byte tile row m, block k sits at
 * ((m % 32) * 4 + (m % 128) / 32) * 4 + k % 4. The buffer then holds
 * round_up(rows, 128) * round_up(hidden / 16, 4) bytes; padding entries are
 * not written. */
typedef enum sm120n_scale_layout {
  SM120N_SCALES_ROW_MAJOR = 0,
  SM120N_SCALES_TILED_128X4 = 1
} sm120n_scale_layout;

/*
 * RMSNorm (optionally after a residual add) with an NVFP4 output for a
 * block-scaled fp4 GEMM. y is computed as in sm120n_rms_norm_fp8_quant; then
 * for every block of 16 consecutive elements of a row, with g = global_scale[0]
 * and each step one IEEE fp32 operation:
 *   a = max |y|;  s = e4m3(g * (a * c));  r = (s == 0) ? 0 : g / s;
 *   (c = 1/6 rounded to fp32)
 *   q = e2m1(y * r)   (e2m1 magnitudes 0, 0.5, 1, 1.5, 2, 3, 4, 6; both
 *                      conversions round to nearest even and saturate)
 * output: [rows, hidden / 2] bytes, element 2i in the low nibble;
 * block_scales: e4m3 bytes in `scale_layout` (sm120n_scale_layout).
 * hidden_size must be a multiple of 16; input, residual and weight 16-byte
 * aligned, output 4-byte aligned (2-byte for fp32). residual_output may equal
 * residual. No reference counterpart: the NVFP4 activation quantisation that
 * follows rms_norm_out_cuda (csrc/rmsnorm_kernels.cu:482-524) and
 * fused_add_rms_norm_out_cuda (:724-801) in an fp4 inference engine.
 */
SM120N_API int sm120n_rms_norm_fp4_quant(const void* input, const void* residual,
                              const void* weight, void* residual_output,
                              void* output, void* block_scales,
                              const float* global_scale, int64_t rows,
                              int64_t hidden_size, int dtype, float epsilon,
                              int scale_layout, void* stream);

/*
 * The QKV projection of an attention layer on the tensor cores, with the
 * Q/K RMSNorm + RoPE + KV store of sm120n_fused_qk_rms_norm_rope_kv fused into
 * its epilogue (bf16, head_dim 128, half-split RoPE over all 128 elements):
 *   qkv[t, :] = round_bf16(hidden[t, :] @ qkv_weight^T)   (fp32 accumulation)
 *   epilogue 1: then, on the [tokens, Hq + 2 * Hk, 128] view of qkv, exactly
 *   what sm120n_fused_qk_rms_norm_rope_kv does (in place on the Q and K heads,
 *   rotated K and V stored at slot_mapping[t] of the [cache_slots, Hk, 128]
 *   caches; pass null caches / slot_mapping for no store); epilogue 0: the
 *   plain GEMM.
 * hidden [tokens, hidden_size], qkv_weight [(Hq + 2Hk) * 128, hidden_size] and
 * qkv [tokens, (Hq + 2Hk) * 128] are dense row-major bf16, 16-byte aligned;
 * hidden_size a multiple of 64; Hq + 2Hk even. The result of epilogue 1 is
 * bit-identical to epilogue 0 followed by sm120n_fused_qk_rms_norm_rope_kv on
 * qkv.
 * Generalises the caller of csrc/rmsnorm_kernels.cu:611-709: the reference
 * runs that operator after a separate projection GEMM.
 */
SM120N_API int sm120n_qkv_proj_norm_rope_cache(
    const void* hidden, const void* qkv_weight, void* qkv, int64_t tokens,
    int64_t hidden_size, int64_t query_heads, int64_t key_heads,
    const void* query_weight, const void* key_weight, const int64_t* positions,
    const float* cos_sin_cache, int64_t rope_positions, void* key_cache,
    void* value_cache, const int32_t* slot_mapping, int64_t cache_slots,
    float epsilon, int epilogue, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* SM120NORM_B200_H_ */
