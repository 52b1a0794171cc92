// Status plumbing of the C ABI: error strings, the per-thread last CUDA error,
// per-device cached attributes and the device-side error word.
#include <atomic>
#include <cstdio>

#include "cf_common.cuh"

// Device-side error word. Kernels with bounded waits OR a DeviceError code
// into it and return instead of spinning forever; cf_device_status() reads and
// clears it.
__device__ unsigned g_cfb_device_error = 0u;

namespace cfb {
namespace {

thread_local int t_last_cuda_error = 0;

constexpr int kMaxDevices = 64;
std::atomic<int> g_sm_count[kMaxDevices];
std::atomic<unsigned *> g_error_word[kMaxDevices];

int current_device() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return -1;
  return dev;
}

}  // namespace

int record_cuda_error(cudaError_t err) {
  t_last_cuda_error = static_cast<int>(err);
  return CF_ERR_CUDA;
}

int sm_count() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return 148;
  int cached = g_sm_count[dev].load(std::memory_order_relaxed);
  if (cached > 0) return cached;
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) {
    n = 148;
  }
  g_sm_count[dev].store(n, std::memory_order_relaxed);
  return n;
}

unsigned *device_error_word() {
  const int dev = current_device();
  if (dev < 0 || dev >= kMaxDevices) return nullptr;
  unsigned *cached = g_error_word[dev].load(std::memory_order_acquire);
  if (cached != nullptr) return cached;
  void *addr = nullptr;
  if (cudaGetSymbolAddress(&addr, g_cfb_device_error) != cudaSuccess) return nullptr;
  g_error_word[dev].store(static_cast<unsigned *>(addr), std::memory_order_release);
  return static_cast<unsigned *>(addr);
}

}  // namespace cfb

extern "C" {

const char *cf_status_string(int status) {
  switch (status) {
    case CF_OK: return "ok";
    case CF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case CF_ERR_UNSUPPORTED: return "unsupported dtype, layout or shape";
    case CF_ERR_MISALIGNED: return "pointer misaligned for this kernel";
    case CF_ERR_CUDA: return "CUDA runtime error";
    case CF_ERR_DEVICE_TIMEOUT: return "a bounded device-side wait timed out";
    case CF_ERR_WORKSPACE: return "workspace missing or too small";
    case CF_ERR_NO_DEVICE: return "current device is not an sm_100 GPU";
    default: return "unknown status";
  }
}

int cf_last_cuda_error(void) { return cfb::t_last_cuda_error; }

int cf_device_status(void) {
  unsigned *word = cfb::device_error_word();
  if (word == nullptr) return cfb::record_cuda_error(cudaGetLastError());
  unsigned value = 0u;
  CFB_TRY_CUDA(cudaMemcpy(&value, word, sizeof(value), cudaMemcpyDeviceToHost));
  if (value == 0u) return CF_OK;
  const unsigned zero = 0u;
  CFB_TRY_CUDA(cudaMemcpy(word, &zero, sizeof(zero), cudaMemcpyHostToDevice));
  return CF_ERR_DEVICE_TIMEOUT;
}

const char *cf_build_info(void) {
  return "cudaforge_b200 0.1.0 sm_100a";
}

}  // extern "C"
