// runtime.h -- host-side helpers behind the C ABI: error reporting, device
// properties and kernel launch.
#pragma once

#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <utility>

#include "sm120norm_b200.h"

namespace sm120n {

// Records a printf-style message for sm120n_last_error() on this thread and
// returns `status`.
int fail(int status, const char* fmt, ...) __attribute__((format(printf, 2, 3)));

// Clears this thread's message (start of every entry point).
void clear_error();

bool programmatic_launch_enabled();

// Polls a kernel makes while waiting for its own bulk copies to land before
// it records an expired wait (sm120n_set_wait_limit; kernels receive it as an
// argument). The default is far beyond any real copy.
constexpr uint32_t kDefaultWaitPolls = 1u << 22;
uint32_t wait_poll_limit();

struct DeviceInfo {
  int device = -1;
  int sm_count = 0;
};

// Properties of the calling thread's current device (cached per device).
int current_device_info(DeviceInfo* info);

// Resident thread blocks per SM for `kernel` at `threads` threads and `smem`
// dynamic shared bytes on the current device (cached).
int max_resident_ctas(const void* kernel, int threads, size_t smem, int* out);

// Allows `kernel` to use `bytes` of dynamic shared memory on the current
// device (cudaFuncAttributeMaxDynamicSharedMemorySize; cached).
int allow_dynamic_smem(const void* kernel, size_t bytes);

// Shared memory a block may use on the current device (opt-in maximum).
int max_block_smem(size_t* bytes);

// Launch `kernel` on `stream`, with the programmatic-stream-serialisation
// attribute when enabled.
template <typename... KernelArgs, typename... Args>
int launch(void (*kernel)(KernelArgs...), dim3 grid, dim3 block, size_t smem,
           cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t config = {};
  config.gridDim = grid;
  config.blockDim = block;
  config.dynamicSmemBytes = smem;
  config.stream = stream;
  cudaLaunchAttribute attribute[1];
  config.attrs = attribute;
  config.numAttrs = 0;
  if (programmatic_launch_enabled()) {
    attribute[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attribute[0].val.programmaticStreamSerializationAllowed = 1;
    config.numAttrs = 1;
  }
  const cudaError_t err = cudaLaunchKernelEx(&config, kernel, std::forward<Args>(args)...);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "kernel launch failed: %s", cudaGetErrorString(err));
  }
  return SM120N_OK;
}

// Expired-wait counter of the tensor-core projection kernel (qkv_gemm.cu),
// read / reset alongside the row kernels' counter.
int read_gemm_faults(unsigned int* value);
int reset_gemm_faults();

// Element size of an sm120n_dtype code, or 0 for an unknown code.
inline int dtype_size(int dtype) {
  switch (dtype) {
    case SM120N_F32: return 4;
    case SM120N_F16:
    case SM120N_BF16: return 2;
    default: return 0;
  }
}

inline bool aligned16(const void* p) {
  return (reinterpret_cast<uintptr_t>(p) & 15u) == 0;
}

}  // namespace sm120n
