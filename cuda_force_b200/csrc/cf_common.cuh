// Shared host/device helpers for the sm_100a kernels: status plumbing, the
// device-side error word, and small launch utilities.
#pragma once

#include <cuda_runtime.h>

#include <atomic>
#include <cstdint>

#include "cudaforge_b200.h"

namespace cfb {

// Elements sharing one scale. Must equal QUANT_BLOCK_SIZE in
// cuda_force_b200/ops.py; tests/test_host.py parses both.
inline constexpr int kQuantBlockSize = 64;

inline constexpr int kWarp = 32;

// Device-side error word, one per device (file-scope __device__ variable in
// abi.cu). A kernel whose bounded wait runs out ORs a code in and returns.
enum DeviceError : unsigned {
  kDevErrNone = 0u,
  kDevErrTimeout = 1u,
};

// Sets the calling thread's last CUDA error and returns CF_ERR_CUDA.
int record_cuda_error(cudaError_t err);

// Checks the launch that was just issued. CF_OK or CF_ERR_CUDA.
inline int check_launch() {
  cudaError_t err = cudaGetLastError();
  return err == cudaSuccess ? CF_OK : record_cuda_error(err);
}

// Number of SMs of the current device (cached per device).
int sm_count();

// Address of the current device's error word (cached per device).
unsigned *device_error_word();

// Residual add and the RMS statistics of each row (norm.cu): residual_out =
// x + residual (when residual is given) and row_scale[r] = 1/sqrt(mean of the
// row's squares + eps), without writing a normalised row.
int residual_rms_stats(const void *x, const void *residual, void *residual_out, float *row_scale,
                       int64_t rows, int64_t cols, float eps, int dtype, cudaStream_t s);

inline bool aligned_to(const void *p, uintptr_t bytes) {
  return (reinterpret_cast<uintptr_t>(p) & (bytes - 1)) == 0;
}

}  // namespace cfb

#define CFB_TRY_CUDA(expr)                                   \
  do {                                                       \
    cudaError_t cfb_err_ = (expr);                           \
    if (cfb_err_ != cudaSuccess) return ::cfb::record_cuda_error(cfb_err_); \
  } while (0)

namespace cfb {

// Raises `Kernel`'s dynamic shared-memory limit once per device; the
// attribute lasts for the life of the CUDA context, so later launches skip the
// driver call (a context torn down by cudaDeviceReset would need it again).
template <auto Kernel>
int allow_dynamic_smem(size_t bytes) {
  static std::atomic<uint64_t> done{0};
  int dev = 0;
  CFB_TRY_CUDA(cudaGetDevice(&dev));
  if (dev < 0 || dev >= 64) return CF_ERR_UNSUPPORTED;
  const uint64_t bit = uint64_t{1} << dev;
  if (done.load(std::memory_order_acquire) & bit) return CF_OK;
  CFB_TRY_CUDA(cudaFuncSetAttribute(Kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(bytes)));
  done.fetch_or(bit, std::memory_order_release);
  return CF_OK;
}

}  // namespace cfb
