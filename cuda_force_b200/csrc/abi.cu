// Status plumbing of the C ABI: error strings, the per-thread last CUDA error,
// per-device cached attributes and the device-side error word.
#include <atomic>
#include <cstdio>

#include "cf_common.cuh"
#include "ptx.cuh"

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

// Test hook of the bounded-wait path: one warp waits on an mbarrier that
// nothing arrives on, with the same bounded wait the product kernels use, and
// records the expiry in the error word exactly as they do.
__global__ void expire_wait_kernel(uint64_t limit_ns, unsigned *error_word) {
  __shared__ __align__(8) uint64_t bar;
  if (threadIdx.x == 0) {
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbar_init();
  }
  __syncwarp();
  const bool ok = ptx::warp_wait(&bar, 0, limit_ns);
  if (!ok && threadIdx.x == 0) atomicOr(error_word, kDevErrTimeout);
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

int cf_debug_expire_wait(uint64_t limit_ns, cf_stream_t stream) {
  if (limit_ns < 1000000ull || limit_ns > 2000000000ull) return CF_ERR_INVALID_ARGUMENT;
  unsigned *word = cfb::device_error_word();
  if (word == nullptr) return cfb::record_cuda_error(cudaGetLastError());
  cfb::expire_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(limit_ns, word);
  CFB_TRY_CUDA(cudaGetLastError());
  return CF_OK;
}

const char *cf_build_info(void) {
  return "cudaforge_b200 0.1.0 sm_100a";
}

}  // extern "C"
