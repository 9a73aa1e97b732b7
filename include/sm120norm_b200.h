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
 */
#ifndef SM120NORM_B200_H_
#define SM120NORM_B200_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SM120N_ABI_VERSION 1

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

#ifdef __cplusplus
}
#endif

#endif /* SM120NORM_B200_H_ */
