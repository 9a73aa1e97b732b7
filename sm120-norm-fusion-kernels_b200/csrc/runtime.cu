// runtime.cu -- error state, device caches and process-wide switches of the
// C ABI (declared in include/sm120norm_b200.h and csrc/runtime.h).
#include <atomic>
#include <cstdarg>
#include <cstdio>
#include <mutex>
#include <string>
#include <tuple>
#include <map>

#include "runtime.h"

namespace sm120n {
namespace {

thread_local std::string g_last_error;
std::atomic<bool> g_programmatic_launch{true};
std::atomic<uint32_t> g_wait_polls{kDefaultWaitPolls};

constexpr int kMaxDevices = 64;
std::mutex g_cache_mutex;
int g_sm_count[kMaxDevices] = {0};
std::map<std::tuple<int, const void*, int, size_t>, int> g_occupancy;
std::map<std::pair<int, const void*>, size_t> g_smem_optin;
size_t g_block_smem[kMaxDevices] = {0};

}  // namespace

int fail(int status, const char* fmt, ...) {
  char buffer[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buffer, sizeof buffer, fmt, args);
  va_end(args);
  g_last_error = buffer;
  return status;
}

void clear_error() { g_last_error.clear(); }

bool programmatic_launch_enabled() { return g_programmatic_launch.load(std::memory_order_relaxed); }

uint32_t wait_poll_limit() { return g_wait_polls.load(std::memory_order_relaxed); }

int current_device_info(DeviceInfo* info) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(err));
  }
  if (device < 0 || device >= kMaxDevices) {
    return fail(SM120N_ERR_UNSUPPORTED, "device ordinal %d is out of range", device);
  }
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  if (g_sm_count[device] == 0) {
    int sms = 0;
    err = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device);
    if (err != cudaSuccess || sms <= 0) {
      return fail(SM120N_ERR_CUDA, "cannot query the SM count of device %d: %s", device,
                  cudaGetErrorString(err));
    }
    g_sm_count[device] = sms;
  }
  info->device = device;
  info->sm_count = g_sm_count[device];
  return SM120N_OK;
}

int max_resident_ctas(const void* kernel, int threads, size_t smem, int* out) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(err));
  }
  const auto key = std::make_tuple(device, kernel, threads, smem);
  {
    std::lock_guard<std::mutex> lock(g_cache_mutex);
    auto it = g_occupancy.find(key);
    if (it != g_occupancy.end()) {
      *out = it->second;
      return SM120N_OK;
    }
  }
  int ctas = 0;
  err = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&ctas, kernel, threads, smem);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "occupancy query failed: %s", cudaGetErrorString(err));
  }
  if (ctas < 1) ctas = 1;
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  g_occupancy[key] = ctas;
  *out = ctas;
  return SM120N_OK;
}

int allow_dynamic_smem(const void* kernel, size_t bytes) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(err));
  }
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  size_t& granted = g_smem_optin[std::make_pair(device, kernel)];
  if (granted >= bytes) return SM120N_OK;
  err = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(bytes));
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "cannot grant %zu bytes of shared memory: %s", bytes,
                cudaGetErrorString(err));
  }
  granted = bytes;
  return SM120N_OK;
}

int max_block_smem(size_t* bytes) {
  int device = 0;
  cudaError_t err = cudaGetDevice(&device);
  if (err != cudaSuccess) {
    return fail(SM120N_ERR_CUDA, "cudaGetDevice failed: %s", cudaGetErrorString(err));
  }
  if (device < 0 || device >= kMaxDevices) {
    return fail(SM120N_ERR_UNSUPPORTED, "device ordinal %d is out of range", device);
  }
  std::lock_guard<std::mutex> lock(g_cache_mutex);
  if (g_block_smem[device] == 0) {
    int value = 0;
    err = cudaDeviceGetAttribute(&value, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    if (err != cudaSuccess || value <= 0) {
      return fail(SM120N_ERR_CUDA, "cannot query shared memory per block: %s",
                  cudaGetErrorString(err));
    }
    g_block_smem[device] = static_cast<size_t>(value);
  }
  *bytes = g_block_smem[device];
  return SM120N_OK;
}

}  // namespace sm120n

extern "C" {

int sm120n_abi_version(void) { return SM120N_ABI_VERSION; }

const char* sm120n_last_error(void) { return sm120n::g_last_error.c_str(); }

const char* sm120n_status_string(int status) {
  switch (status) {
    case SM120N_OK: return "ok";
    case SM120N_ERR_INVALID_ARGUMENT: return "invalid argument";
    case SM120N_ERR_UNSUPPORTED: return "unsupported";
    case SM120N_ERR_CUDA: return "CUDA error";
    default: return "unknown status";
  }
}

void sm120n_set_programmatic_launch(int enabled) { sm120n::g_programmatic_launch.store(enabled != 0); }

int sm120n_get_programmatic_launch(void) { return sm120n::g_programmatic_launch.load() ? 1 : 0; }

void sm120n_set_wait_limit(uint32_t polls) {
  sm120n::g_wait_polls.store(polls == 0 || polls > sm120n::kDefaultWaitPolls
                                 ? sm120n::kDefaultWaitPolls
                                 : polls);
}

uint32_t sm120n_get_wait_limit(void) { return sm120n::g_wait_polls.load(); }

}  // extern "C"
