// Residual add + RMSNorm (and plain RMSNorm) for sm_100a.
//
// Semantics (reference python/cudaforge/ops.py:164-171 and :188-192,
// cpp/src/bindings.cpp:238-270; fp32 kernel cuda/src/fused_norm.cu:21-63):
//   summed = x + residual, rounded to the input dtype (one fp32 add, one
//            rounding: what the ATen add of two bf16/fp16 tensors gives);
//   out    = fl(summed * rsqrt(mean(summed^2) + eps) * weight), the product
//            and the mean in fp32, rounded once to the input dtype.
// With no residual the same kernel is the reference's plain rmsnorm.
//
// Design: HBM-bound (read x and residual once, write out and residual_out
// once; the weight row stays in L1/L2). One 256-thread CTA per row in a
// grid-stride loop over rows. Each thread keeps its 16-byte chunks of the
// rounded sum in registers between the reduction and the scaling pass, so the
// row is never read back (the reference re-reads residual_out). Rows longer
// than the register budget (more than 4 chunks per thread: 8192 16-bit or 4096
// fp32 elements) re-read their own residual_out chunks, still in L2, in the
// second pass; rows whose length or pointers do
// not allow 16-byte chunks take an element-wise form of the same kernel.
// Each thread reads an address before it writes it and no other thread
// touches it, so output may alias x and residual_out may alias residual.
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include "cf_common.cuh"

namespace cfb {
namespace {

constexpr int kNormThreads = 256;
constexpr int kNormWarps = kNormThreads / kWarp;
// 16-byte chunks per thread kept in registers: 4 is <= 80 registers (three or
// more CTAs per SM); 8 would need 130-150 and leave one CTA per SM.
constexpr int kMaxResident = 4;

template <typename T>
struct Elem;
template <>
struct Elem<float> {
  static __device__ __forceinline__ float load(const float *p) { return *p; }
  static __device__ __forceinline__ float round(float v) { return v; }
  static __device__ __forceinline__ void store(float *p, float v) { *p = v; }
};
template <>
struct Elem<__nv_bfloat16> {
  static __device__ __forceinline__ float load(const __nv_bfloat16 *p) {
    return __bfloat162float(*p);
  }
  static __device__ __forceinline__ float round(float v) {
    return __bfloat162float(__float2bfloat16_rn(v));
  }
  static __device__ __forceinline__ void store(__nv_bfloat16 *p, float v) {
    *p = __float2bfloat16_rn(v);
  }
};
template <>
struct Elem<__half> {
  static __device__ __forceinline__ float load(const __half *p) { return __half2float(*p); }
  static __device__ __forceinline__ float round(float v) {
    return __half2float(__float2half_rn(v));
  }
  static __device__ __forceinline__ void store(__half *p, float v) { *p = __float2half_rn(v); }
};

// A 16-byte chunk of T as floats, and back (round to nearest even).
template <typename T>
struct Chunk {
  static constexpr int kElems = 16 / sizeof(T);
  static __device__ __forceinline__ void unpack(const uint4 &v, float (&f)[kElems]) {
    const T *e = reinterpret_cast<const T *>(&v);
#pragma unroll
    for (int i = 0; i < kElems; ++i) f[i] = Elem<T>::load(e + i);
  }
  static __device__ __forceinline__ uint4 pack(const float (&f)[kElems]) {
    uint4 v;
    T *e = reinterpret_cast<T *>(&v);
#pragma unroll
    for (int i = 0; i < kElems; ++i) Elem<T>::store(e + i, f[i]);
    return v;
  }
};

// Weight values of chunk c (kElems of them) as floats; TW is T or float.
template <typename T, typename TW>
__device__ __forceinline__ void load_weight(const TW *w, int64_t c, float (&f)[Chunk<T>::kElems]) {
  constexpr int kE = Chunk<T>::kElems;
  const uint4 *src = reinterpret_cast<const uint4 *>(w + c * kE);
  constexpr int kVecs = kE * sizeof(TW) / 16;
#pragma unroll
  for (int v = 0; v < kVecs; ++v) {
    const uint4 raw = __ldg(src + v);
    const TW *e = reinterpret_cast<const TW *>(&raw);
#pragma unroll
    for (int i = 0; i < 16 / static_cast<int>(sizeof(TW)); ++i) {
      f[v * (16 / sizeof(TW)) + i] = Elem<TW>::load(e + i);
    }
  }
}

// Sum over the CTA; `buf` alternates between rows so one barrier per row
// suffices (a thread reaches the next write of the same buffer only after
// every thread has passed the following row's barrier, i.e. read this one).
__device__ __forceinline__ float block_sum(float v, float *buf) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int warp = threadIdx.x / kWarp;
  if ((threadIdx.x & (kWarp - 1)) == 0) buf[warp] = v;
  __syncthreads();
  float s = 0.0f;
#pragma unroll
  for (int i = 0; i < kNormWarps; ++i) s += buf[i];
  return s;
}

// 16-byte chunks. kV > 0: up to kV chunks per thread stay in registers
// (nchunks <= kV * kNormThreads); kV == 0: the second pass re-reads
// residual_out (or x when there is no residual).
template <typename T, typename TW, int kV>
__global__ void __launch_bounds__(kNormThreads)
    residual_rmsnorm_vec_kernel(const T *x, const T *residual, const TW *weight, T *out,
                                T *residual_out, int64_t rows, int64_t cols, float eps,
                                float *row_scale) {
  using C = Chunk<T>;
  constexpr int kE = C::kElems;
  __shared__ float red[2][kNormWarps];
  const int64_t nchunks = cols / kE;
  int parity = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, parity ^= 1) {
    const uint4 *xr = reinterpret_cast<const uint4 *>(x + row * cols);
    const uint4 *rr = residual ? reinterpret_cast<const uint4 *>(residual + row * cols) : nullptr;
    uint4 *sr = residual ? reinterpret_cast<uint4 *>(residual_out + row * cols) : nullptr;
    uint4 *orow = reinterpret_cast<uint4 *>(out + row * cols);
    float ss = 0.0f;
    constexpr int kKeep = kV > 0 ? kV : 1;
    uint4 keep[kKeep];
    if constexpr (kV > 0) {
      uint4 xa[kV], ra[kV];
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const int64_t c = threadIdx.x + static_cast<int64_t>(i) * kNormThreads;
        if (c < nchunks) {
          xa[i] = xr[c];
          if (rr) ra[i] = rr[c];
        }
      }
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const int64_t c = threadIdx.x + static_cast<int64_t>(i) * kNormThreads;
        if (c < nchunks) {
          float f[kE];
          C::unpack(xa[i], f);
          if (rr) {
            float g[kE];
            C::unpack(ra[i], g);
#pragma unroll
            for (int e = 0; e < kE; ++e) f[e] = Elem<T>::round(f[e] + g[e]);
            keep[i] = C::pack(f);
            sr[c] = keep[i];
          } else {
            keep[i] = xa[i];
          }
#pragma unroll
          for (int e = 0; e < kE; ++e) ss = fmaf(f[e], f[e], ss);
        }
      }
    } else {
      for (int64_t c = threadIdx.x; c < nchunks; c += kNormThreads) {
        float f[kE];
        C::unpack(xr[c], f);
        if (rr) {
          float g[kE];
          C::unpack(rr[c], g);
#pragma unroll
          for (int e = 0; e < kE; ++e) f[e] = Elem<T>::round(f[e] + g[e]);
          sr[c] = C::pack(f);
        }
#pragma unroll
        for (int e = 0; e < kE; ++e) ss = fmaf(f[e], f[e], ss);
      }
    }
    const float scale = rsqrtf(block_sum(ss, red[parity]) / static_cast<float>(cols) + eps);
    if (out == nullptr) {  // statistics only: the row's scale instead of the normalised row
      if (threadIdx.x == 0) row_scale[row] = scale;
      continue;
    }
    if constexpr (kV > 0) {
#pragma unroll
      for (int i = 0; i < kV; ++i) {
        const int64_t c = threadIdx.x + static_cast<int64_t>(i) * kNormThreads;
        if (c < nchunks) {
          float f[kE], w[kE];
          C::unpack(keep[i], f);
          load_weight<T, TW>(weight, c, w);
#pragma unroll
          for (int e = 0; e < kE; ++e) f[e] = f[e] * scale * w[e];
          orow[c] = C::pack(f);
        }
      }
    } else {
      const uint4 *back = rr ? sr : xr;
      for (int64_t c = threadIdx.x; c < nchunks; c += kNormThreads) {
        float f[kE], w[kE];
        C::unpack(back[c], f);
        load_weight<T, TW>(weight, c, w);
#pragma unroll
        for (int e = 0; e < kE; ++e) f[e] = f[e] * scale * w[e];
        orow[c] = C::pack(f);
      }
    }
  }
}

// Element-wise form for rows whose length or pointers rule out 16-byte chunks.
template <typename T, typename TW>
__global__ void __launch_bounds__(kNormThreads)
    residual_rmsnorm_scalar_kernel(const T *x, const T *residual, const TW *weight, T *out,
                                   T *residual_out, int64_t rows, int64_t cols, float eps,
                                   float *row_scale) {
  __shared__ float red[2][kNormWarps];
  int parity = 0;
  for (int64_t row = blockIdx.x; row < rows; row += gridDim.x, parity ^= 1) {
    const int64_t base = row * cols;
    float ss = 0.0f;
    for (int64_t c = threadIdx.x; c < cols; c += kNormThreads) {
      float v = Elem<T>::load(x + base + c);
      if (residual) {
        v = Elem<T>::round(v + Elem<T>::load(residual + base + c));
        Elem<T>::store(residual_out + base + c, v);
      }
      ss = fmaf(v, v, ss);
    }
    const float scale = rsqrtf(block_sum(ss, red[parity]) / static_cast<float>(cols) + eps);
    if (out == nullptr) {
      if (threadIdx.x == 0) row_scale[row] = scale;
      continue;
    }
    const T *back = residual ? residual_out : x;
    for (int64_t c = threadIdx.x; c < cols; c += kNormThreads) {
      const float v = Elem<T>::load(back + base + c);
      Elem<T>::store(out + base + c, v * scale * Elem<TW>::load(weight + c));
    }
  }
}

template <typename T, typename TW, int kV>
int launch_vec(const void *x, const void *r, const void *w, void *o, void *ro, int64_t rows,
               int64_t cols, float eps, float *rs, unsigned grid, cudaStream_t s) {
  residual_rmsnorm_vec_kernel<T, TW, kV><<<grid, kNormThreads, 0, s>>>(
      static_cast<const T *>(x), static_cast<const T *>(r), static_cast<const TW *>(w),
      static_cast<T *>(o), static_cast<T *>(ro), rows, cols, eps, rs);
  return check_launch();
}

template <typename T, typename TW>
int norm_dispatch(const void *x, const void *r, const void *w, void *o, void *ro, int64_t rows,
                  int64_t cols, float eps, cudaStream_t s, float *rs = nullptr) {
  const int64_t want = static_cast<int64_t>(sm_count()) * 8;
  const unsigned grid = static_cast<unsigned>(rows < want ? rows : want);
  constexpr int kE = Chunk<T>::kElems;
  const bool vec = cols % kE == 0 && aligned_to(x, 16) && (o == nullptr || aligned_to(o, 16)) &&
                   aligned_to(w, 16) && (r == nullptr || (aligned_to(r, 16) && aligned_to(ro, 16)));
  if (!vec) {
    residual_rmsnorm_scalar_kernel<T, TW><<<grid, kNormThreads, 0, s>>>(
        static_cast<const T *>(x), static_cast<const T *>(r), static_cast<const TW *>(w),
        static_cast<T *>(o), static_cast<T *>(ro), rows, cols, eps, rs);
    return check_launch();
  }
  const int64_t per_thread = (cols / kE + kNormThreads - 1) / kNormThreads;
  if (per_thread <= 1) return launch_vec<T, TW, 1>(x, r, w, o, ro, rows, cols, eps, rs, grid, s);
  if (per_thread <= 2) return launch_vec<T, TW, 2>(x, r, w, o, ro, rows, cols, eps, rs, grid, s);
  if (per_thread <= kMaxResident) {
    return launch_vec<T, TW, kMaxResident>(x, r, w, o, ro, rows, cols, eps, rs, grid, s);
  }
  return launch_vec<T, TW, 0>(x, r, w, o, ro, rows, cols, eps, rs, grid, s);
}

}  // namespace

int residual_rms_stats(const void *x, const void *residual, void *residual_out, float *row_scale,
                       int64_t rows, int64_t cols, float eps, int dtype, cudaStream_t s) {
  if (rows == 0 || cols == 0) return CF_OK;
  switch (dtype) {
    case CF_DTYPE_F32:
      return norm_dispatch<float, float>(x, residual, x, nullptr, residual_out, rows, cols, eps,
                                         s, row_scale);
    case CF_DTYPE_BF16:
      return norm_dispatch<__nv_bfloat16, __nv_bfloat16>(x, residual, x, nullptr, residual_out,
                                                         rows, cols, eps, s, row_scale);
    default:
      return norm_dispatch<__half, __half>(x, residual, x, nullptr, residual_out, rows, cols,
                                           eps, s, row_scale);
  }
}

}  // namespace cfb

extern "C" {

int cf_fused_residual_rmsnorm(const void *x, const void *residual, const void *weight,
                              int weight_dtype, void *output, void *residual_out, int64_t rows,
                              int64_t cols, float eps, int dtype, cf_stream_t stream) {
  if (rows < 0 || cols < 0) return CF_ERR_INVALID_ARGUMENT;
  if (rows == 0 || cols == 0) return CF_OK;
  if (x == nullptr || weight == nullptr || output == nullptr) return CF_ERR_INVALID_ARGUMENT;
  if ((residual == nullptr) != (residual_out == nullptr)) return CF_ERR_INVALID_ARGUMENT;
  if (dtype != CF_DTYPE_F32 && dtype != CF_DTYPE_BF16 && dtype != CF_DTYPE_F16) {
    return CF_ERR_UNSUPPORTED;
  }
  if (weight_dtype != dtype && weight_dtype != CF_DTYPE_F32) return CF_ERR_UNSUPPORTED;
  if (rows > (int64_t{1} << 40) / cols) return CF_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool wf = weight_dtype == CF_DTYPE_F32;
  switch (dtype) {
    case CF_DTYPE_F32:
      return cfb::norm_dispatch<float, float>(x, residual, weight, output, residual_out, rows,
                                              cols, eps, s);
    case CF_DTYPE_BF16:
      return wf ? cfb::norm_dispatch<__nv_bfloat16, float>(x, residual, weight, output,
                                                           residual_out, rows, cols, eps, s)
                : cfb::norm_dispatch<__nv_bfloat16, __nv_bfloat16>(x, residual, weight, output,
                                                                   residual_out, rows, cols,
                                                                   eps, s);
    default:
      return wf ? cfb::norm_dispatch<__half, float>(x, residual, weight, output, residual_out,
                                                    rows, cols, eps, s)
                : cfb::norm_dispatch<__half, __half>(x, residual, weight, output, residual_out,
                                                     rows, cols, eps, s);
  }
}

}  // extern "C"
