// Block-wise INT8 quantise / dequantise / fake-quantise for sm_100a.
//
// Semantics (reference python/cudaforge/ops.py:215-240 and
// cpp/src/bindings.cpp:298-329, kernels cuda/src/quantization.cu:18-76):
//   blocks of 64 consecutive elements of the flattened tensor;
//   scale = fl32(absmax / 127), replaced by 1 when not > 0 (zero, NaN, underflow);
//   code  = clamp(rint_half_even(fl32(x / scale)), -127, 127), NaN -> 0;
//   dequant = fl32(code * scale).
//
// Design (not a translation of the reference's one-thread-per-element kernel):
//   * main path (quantize_tma_kernel): a persistent grid streams 32 KB tiles
//     through a 5-stage shared-memory ring with bulk copies (TMA engine) and
//     writes codes and scales back with bulk stores; tails, misaligned tensors
//     and fake-quant use a register-streaming kernel whose lanes issue UNROLL
//     independent 16-byte loads before touching any of them;
//   * a 64-element block is spread over 16 lanes (f32) or 8 lanes (f16/bf16);
//     the absmax is a shuffle-xor max over those lanes of |x| bit patterns as
//     unsigned integers, which orders non-negative floats exactly and makes a
//     NaN win, the same propagation as torch.amax;
//   * codes: the exact quotient fl32(x / s) is only needed near a rounding
//     boundary. Each element is first multiplied by r = rn(1/s); when the
//     product is further than 2^-12 from a half-integer (true for all but ~1e-4
//     of elements) its rint equals rint(fl32(x/s)) — |t - x/s| < 2^-15.9 for
//     |x/s| <= 127 with s and r normal — otherwise the correctly rounded IEEE
//     division decides. Bit-exact, at a fraction of the divider's issue cost;
//   * codes are packed 4 or 8 per store; the register path writes them with
//     streaming stores (st.global.cs).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>

#include "cf_common.cuh"
#include "ptx.cuh"

namespace cfb {
namespace {

constexpr int kThreads = 256;

template <typename T>
struct VecTraits;
template <>
struct VecTraits<float> {
  static constexpr int kPerVec = 4;
};
template <>
struct VecTraits<__nv_bfloat16> {
  static constexpr int kPerVec = 8;
};
template <>
struct VecTraits<__half> {
  static constexpr int kPerVec = 8;
};

__device__ __forceinline__ uint4 ld_stream_v4(const void *p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

__device__ __forceinline__ unsigned ld_stream_u32(const void *p) {
  unsigned v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::256B.u32 %0, [%1];" : "=r"(v) : "l"(p));
  return v;
}

__device__ __forceinline__ void unpack(const uint4 &v, float (&f)[4]) {
  f[0] = __uint_as_float(v.x);
  f[1] = __uint_as_float(v.y);
  f[2] = __uint_as_float(v.z);
  f[3] = __uint_as_float(v.w);
}

__device__ __forceinline__ void unpack_bf16x2(unsigned w, float &lo, float &hi) {
  lo = __uint_as_float(w << 16);
  hi = __uint_as_float(w & 0xffff0000u);
}

__device__ __forceinline__ void unpack(const uint4 &v, float (&f)[8], __nv_bfloat16 *) {
  unpack_bf16x2(v.x, f[0], f[1]);
  unpack_bf16x2(v.y, f[2], f[3]);
  unpack_bf16x2(v.z, f[4], f[5]);
  unpack_bf16x2(v.w, f[6], f[7]);
}

__device__ __forceinline__ void unpack_h2(unsigned w, float &lo, float &hi) {
  __half2 h = *reinterpret_cast<__half2 *>(&w);
  float2 f = __half22float2(h);
  lo = f.x;
  hi = f.y;
}

__device__ __forceinline__ void unpack(const uint4 &v, float (&f)[8], __half *) {
  unpack_h2(v.x, f[0], f[1]);
  unpack_h2(v.y, f[2], f[3]);
  unpack_h2(v.z, f[4], f[5]);
  unpack_h2(v.w, f[6], f[7]);
}

template <typename T>
__device__ __forceinline__ float load_scalar(const T *p);
template <>
__device__ __forceinline__ float load_scalar<float>(const float *p) {
  return __ldg(p);
}
template <>
__device__ __forceinline__ float load_scalar<__nv_bfloat16>(const __nv_bfloat16 *p) {
  const unsigned short bits = __ldg(reinterpret_cast<const unsigned short *>(p));
  return __uint_as_float(static_cast<unsigned>(bits) << 16);
}
template <>
__device__ __forceinline__ float load_scalar<__half>(const __half *p) {
  return __half2float(__ldg(p));
}

// Block scale from the absmax bit pattern: fl32(absmax / 127), or 1 when that
// is not > 0. A NaN pattern (above 0x7f800000) gives NaN / 127 = NaN -> 1.
__device__ __forceinline__ float block_scale(unsigned absmax_bits) {
  const float s = __fdiv_rn(__uint_as_float(absmax_bits), 127.0f);
  return s > 0.0f ? s : 1.0f;
}

// Whether the reciprocal shortcut is valid for this scale (s and 1/s normal).
__device__ __forceinline__ bool fast_scale(float s) {
  return s >= 0x1p-126f && s <= 0x1p126f;
}

__device__ __forceinline__ int clamp_code(int v) { return min(max(v, -127), 127); }

// clamp(rint_half_even(fl32(x / s)), -127, 127), NaN -> 0 (cvt.rni of NaN is 0).
__device__ __forceinline__ int quantise_one(float x, float s, float r, bool fast) {
  if (fast) {
    const float t = __fmul_rn(x, r);
    const float n = rintf(t);
    // 0.5 - 2^-12: the product is at least 2^-12 away from a half-integer.
    if (fabsf(t - n) <= 0.499755859375f) return clamp_code(__float2int_rn(n));
  }
  return clamp_code(__float2int_rn(__fdiv_rn(x, s)));
}

__device__ __forceinline__ unsigned pack4(int a, int b, int c, int d) {
  return (static_cast<unsigned>(a) & 0xffu) | ((static_cast<unsigned>(b) & 0xffu) << 8) |
         ((static_cast<unsigned>(c) & 0xffu) << 16) | (static_cast<unsigned>(d) << 24);
}

// ---------------------------------------------------------------------------
// Quantisation core shared by every kernel.
// ---------------------------------------------------------------------------
// Per-block constants. `fast` selects the reciprocal path: the block holds no
// NaN/inf and both s and 1/s are normal, so |x * r| <= 127 * (1 + 2^-22) and
// no clamp is needed.
struct BlockParams {
  float s;
  float r;
  bool fast;
};

__device__ __forceinline__ BlockParams block_params(unsigned absmax_bits) {
  BlockParams b;
  b.s = block_scale(absmax_bits);
  b.r = __frcp_rn(b.s);
  b.fast = absmax_bits < 0x7f800000u && b.s >= 0x1p-126f && b.s <= 0x1p126f;
  return b;
}

// Codes of 4 elements of one block, packed little-endian into a word.
//
// Fast path: m = fma(x, r, 1.5 * 2^23) rounds the exact product x * r to the
// nearest integer (ties to even) in one instruction, leaving that integer in
// the low bits of m's bit pattern (so the code byte is read directly); d, the
// product's distance to that integer, is exact to 2^-24. When |d| is at most
// 0.5 - 2^-12 the rounding of fl32(x / s) agrees, because
// |x*r - x/s| <= 2^-17 and |fl32(x/s) - x/s| <= 2^-18 for |x/s| <= 127.
// Otherwise (a near tie, about one element in 4000) or off the fast path, the
// correctly rounded IEEE division decides.
__device__ __forceinline__ uint32_t quantise4(const float (&x)[4], const BlockParams &b) {
  constexpr float kRound = 12582912.0f;           // 1.5 * 2^23
  constexpr float kTieGuard = 0.499755859375f;    // 0.5 - 2^-12
  uint32_t mb[4];
  unsigned slow = b.fast ? 0u : 0xfu;
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float m = __fmaf_rn(x[e], b.r, kRound);
    const float d = __fmaf_rn(x[e], b.r, -(m - kRound));
    mb[e] = __float_as_uint(m);
    slow |= (fabsf(d) > kTieGuard ? 1u : 0u) << e;
  }
  if (slow != 0u) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      if (slow & (1u << e)) {
        mb[e] = static_cast<uint32_t>(clamp_code(__float2int_rn(__fdiv_rn(x[e], b.s))));
      }
    }
  }
  return __byte_perm(__byte_perm(mb[0], mb[1], 0x0040u), __byte_perm(mb[2], mb[3], 0x0040u),
                     0x5410u);
}

// Absolute-value bit pattern maximum of a lane's 16-byte vector, as float bits.
// Non-negative floats order like their bit patterns and NaN patterns sit above
// +inf, so the maximum propagates NaN exactly as torch.amax does.
__device__ __forceinline__ unsigned vec_absmax_bits(const uint4 &v, float *) {
  unsigned m = max(v.x & 0x7fffffffu, v.y & 0x7fffffffu);
  m = max(m, v.z & 0x7fffffffu);
  return max(m, v.w & 0x7fffffffu);
}
// bf16: max of the packed 16-bit magnitudes, two per instruction; the bf16
// pattern shifted left by 16 is the float pattern.
__device__ __forceinline__ unsigned vec_absmax_bits(const uint4 &v, __nv_bfloat16 *) {
  unsigned m = __vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu);
  m = __vmaxu2(m, v.z & 0x7fff7fffu);
  m = __vmaxu2(m, v.w & 0x7fff7fffu);
  return max(m << 16, m & 0xffff0000u);
}
// fp16: same packed maximum on the half patterns, then widened to float exactly.
__device__ __forceinline__ unsigned vec_absmax_bits(const uint4 &v, __half *) {
  unsigned m = __vmaxu2(v.x & 0x7fff7fffu, v.y & 0x7fff7fffu);
  m = __vmaxu2(m, v.z & 0x7fff7fffu);
  m = __vmaxu2(m, v.w & 0x7fff7fffu);
  const unsigned short h = static_cast<unsigned short>(max(m & 0xffffu, m >> 16));
  return __float_as_uint(__half2float(__ushort_as_half(h)));
}

// One lane's share of the warp-cooperative layout: a 16-byte vector of
// kPerVec elements, kLanesPerBlock lanes per 64-element block.
template <typename T>
struct LaneQuant {
  static constexpr int kPerVec = VecTraits<T>::kPerVec;
  static constexpr int kLanesPerBlock = kQuantBlockSize / kPerVec;
  static constexpr int kWords = kPerVec / 4;  // packed code words per lane

  static __device__ __forceinline__ void run(const uint4 &v, uint32_t (&codes)[kWords],
                                             float &scale) {
    unsigned m = vec_absmax_bits(v, static_cast<T *>(nullptr));
#pragma unroll
    for (int off = kLanesPerBlock / 2; off > 0; off >>= 1) {
      m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
    }
    const BlockParams b = block_params(m);
    float f[kPerVec];
    if constexpr (kPerVec == 4) {
      unpack(v, f);
    } else {
      unpack(v, f, static_cast<T *>(nullptr));
    }
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      const float x4[4] = {f[4 * w], f[4 * w + 1], f[4 * w + 2], f[4 * w + 3]};
      codes[w] = quantise4(x4, b);
    }
    scale = b.s;
  }
};

__device__ __forceinline__ float rcp_approx(float s) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(s));
  return r;
}

// Shared-memory layout of the TMA kernel: 4 lanes per 64-element block, 16
// elements (kChunks 16-byte chunks) per lane, 8 blocks per warp step.
//
// Lane 4b+i of a step owns chunks 4*((j + (b & 1)) % kChunks) + i (j = 0 ..
// kChunks-1) of block b. Within one load instruction j the 32 chunk indices
// then cover every residue mod 8 exactly four times, so the 16-byte shared
// loads are bank-conflict-free while each lane's chunks stay in one block.
template <typename T>
struct Quad {
  static constexpr int kPerChunk = 16 / static_cast<int>(sizeof(T));  // elements per chunk
  static constexpr int kChunks = 16 / kPerChunk;                       // chunks per lane
  static constexpr int kStepElems = 8 * kQuantBlockSize;               // 8 blocks per step

  static __device__ __forceinline__ int chunk_of(int lane, int j) {
    const int b = lane >> 2;
    return 4 * ((j + (b & 1)) % kChunks) + (lane & 3);
  }

  // Quantises one warp step: reads from `src` (the step's 512 elements),
  // writes codes to `codes` (512 bytes) and 8 scales to `scales`.
  static __device__ __forceinline__ void step(const uint8_t *src, uint8_t *codes, float *scales,
                                              int lane) {
    const int b = lane >> 2;
    uint4 v[kChunks];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int elem = b * kQuantBlockSize + chunk_of(lane, j) * kPerChunk;
      v[j] = *reinterpret_cast<const uint4 *>(src + elem * static_cast<int>(sizeof(T)));
    }
    unsigned m = 0u;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) m = max(m, vec_absmax_bits(v[j], static_cast<T *>(nullptr)));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const float s = block_scale(m);
    // 1 ulp reciprocal: |x*r - x/s| <= 127 * 2^-23 < 2^-15.9, far inside the guard.
    const bool fast = m < 0x7f800000u && s >= 0x1p-126f && s <= 0x1p126f;
    const float r = rcp_approx(s);

    constexpr float kRound = 12582912.0f;         // 1.5 * 2^23
    constexpr float kTieGuard = 0.499755859375f;  // 0.5 - 2^-12
    float f[16];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      float g[kPerChunk];
      if constexpr (kPerChunk == 4) {
        unpack(v[j], g);
      } else {
        unpack(v[j], g, static_cast<T *>(nullptr));
      }
#pragma unroll
      for (int e = 0; e < kPerChunk; ++e) f[j * kPerChunk + e] = g[e];
    }
    uint32_t mb[16];
    float worst = 0.0f;
#pragma unroll
    for (int e = 0; e < 16; ++e) {
      const float mm = __fmaf_rn(f[e], r, kRound);
      const float d = __fmaf_rn(f[e], r, -(mm - kRound));
      mb[e] = __float_as_uint(mm);
      worst = fmaxf(worst, fabsf(d));
    }
    if (!fast || !(worst <= kTieGuard)) {
#pragma unroll
      for (int e = 0; e < 16; ++e) {
        mb[e] = static_cast<uint32_t>(clamp_code(__float2int_rn(__fdiv_rn(f[e], s))));
      }
    }
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int e0 = j * kPerChunk;
      uint8_t *dst = codes + b * kQuantBlockSize + chunk_of(lane, j) * kPerChunk;
      const uint32_t w0 = __byte_perm(__byte_perm(mb[e0], mb[e0 + 1], 0x0040u),
                                      __byte_perm(mb[e0 + 2], mb[e0 + 3], 0x0040u), 0x5410u);
      if constexpr (kPerChunk == 4) {
        *reinterpret_cast<uint32_t *>(dst) = w0;
      } else {
        const uint32_t w1 = __byte_perm(__byte_perm(mb[e0 + 4], mb[e0 + 5], 0x0040u),
                                        __byte_perm(mb[e0 + 6], mb[e0 + 7], 0x0040u), 0x5410u);
        *reinterpret_cast<uint2 *>(dst) = make_uint2(w0, w1);
      }
    }
    if ((lane & 3) == 0) scales[b] = s;
  }
};

__device__ __forceinline__ float code_to_float(uint32_t word, int byte) {
  return static_cast<float>(static_cast<int8_t>((word >> (8 * byte)) & 0xffu));
}

__device__ __forceinline__ void st_stream_u32(void *p, unsigned v) {
  asm volatile("st.global.cs.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ void st_stream_v2(void *p, unsigned a, unsigned b) {
  asm volatile("st.global.cs.v2.u32 [%0], {%1,%2};" ::"l"(p), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ void st_stream_f32(float *p, float v) {
  asm volatile("st.global.cs.f32 [%0], %1;" ::"l"(p), "f"(v) : "memory");
}
__device__ __forceinline__ void st_stream_f4(float *p, float a, float b, float c, float d) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(a), "f"(b), "f"(c),
               "f"(d)
               : "memory");
}

// ---------------------------------------------------------------------------
// Vectorised quantiser: one "unit" = UNROLL warp-wide 16-byte loads.
// ---------------------------------------------------------------------------
template <typename T, int UNROLL>
struct QuantUnit {
  static constexpr int kPerVec = VecTraits<T>::kPerVec;          // elements per lane load
  static constexpr int kLanesPerBlock = kQuantBlockSize / kPerVec;  // 16 (f32) or 8
  static constexpr int kPerLoad = kWarp * kPerVec;                  // elements per warp load
  static constexpr int kElems = UNROLL * kPerLoad;                  // elements per unit

  // Processes elements [base, base + kElems) of one tensor. kFake selects the
  // fake-quant output (float) instead of codes + scales.
  template <bool kFake>
  static __device__ __forceinline__ void run(const T *__restrict__ in, int8_t *__restrict__ codes,
                                             float *__restrict__ scales,
                                             float *__restrict__ fake_out, int64_t base,
                                             int lane) {
    uint4 v[UNROLL];
#pragma unroll
    for (int j = 0; j < UNROLL; ++j) {
      v[j] = ld_stream_v4(in + base + static_cast<int64_t>(j) * kPerLoad + lane * kPerVec);
    }
#pragma unroll
    for (int j = 0; j < UNROLL; ++j) {
      uint32_t q[kPerVec / 4];
      float s;
      LaneQuant<T>::run(v[j], q, s);
      const int64_t e0 = base + static_cast<int64_t>(j) * kPerLoad + lane * kPerVec;
      if constexpr (kFake) {
#pragma unroll
        for (int w = 0; w < kPerVec / 4; ++w) {
          st_stream_f4(fake_out + e0 + 4 * w, __fmul_rn(code_to_float(q[w], 0), s),
                       __fmul_rn(code_to_float(q[w], 1), s), __fmul_rn(code_to_float(q[w], 2), s),
                       __fmul_rn(code_to_float(q[w], 3), s));
        }
      } else {
        if constexpr (kPerVec == 4) {
          st_stream_u32(codes + e0, q[0]);
        } else {
          st_stream_v2(codes + e0, q[0], q[1]);
        }
        if ((lane & (kLanesPerBlock - 1)) == 0) st_stream_f32(scales + e0 / kQuantBlockSize, s);
      }
    }
  }
};

template <typename T, int UNROLL, bool kFake>
__global__ void __launch_bounds__(kThreads)
    quantize_vec_kernel(const T *__restrict__ in, int8_t *__restrict__ codes,
                        float *__restrict__ scales, float *__restrict__ fake_out, int64_t nunits) {
  using U = QuantUnit<T, UNROLL>;
  const int lane = threadIdx.x & (kWarp - 1);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / kWarp);
  for (int64_t u = warp; u < nunits; u += nwarps) {
    U::template run<kFake>(in, codes, scales, fake_out, u * U::kElems, lane);
  }
}

// Scalar path: one warp per quantisation block, two elements per lane. Handles
// the ragged tail and any tensor whose pointers are not vector-aligned.
template <typename T, bool kFake>
__global__ void __launch_bounds__(kThreads)
    quantize_scalar_kernel(const T *__restrict__ in, int8_t *__restrict__ codes,
                           float *__restrict__ scales, float *__restrict__ fake_out,
                           int64_t first_block, int64_t end_block, int64_t count) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / kWarp);
  for (int64_t b = first_block + warp; b < end_block; b += nwarps) {
    const int64_t i0 = b * kQuantBlockSize + lane;
    const int64_t i1 = i0 + kWarp;
    const float x0 = i0 < count ? load_scalar<T>(in + i0) : 0.0f;
    const float x1 = i1 < count ? load_scalar<T>(in + i1) : 0.0f;
    unsigned m = max(__float_as_uint(x0) & 0x7fffffffu, __float_as_uint(x1) & 0x7fffffffu);
#pragma unroll
    for (int off = kWarp / 2; off > 0; off >>= 1) m = max(m, __shfl_xor_sync(0xffffffffu, m, off));
    const float s = block_scale(m);
    const float r = __frcp_rn(s);
    const bool fast = fast_scale(s);
    if (i0 < count) {
      const int q = quantise_one(x0, s, r, fast);
      if constexpr (kFake) fake_out[i0] = __fmul_rn(static_cast<float>(q), s);
      else codes[i0] = static_cast<int8_t>(q);
    }
    if (i1 < count) {
      const int q = quantise_one(x1, s, r, fast);
      if constexpr (kFake) fake_out[i1] = __fmul_rn(static_cast<float>(q), s);
      else codes[i1] = static_cast<int8_t>(q);
    }
    if constexpr (!kFake) {
      if (lane == 0) scales[b] = s;
    }
  }
}

// Segment table of a grouped launch, passed as a kernel parameter (no device
// allocation). unit_end is the inclusive prefix sum of tiles per segment.
struct GroupedArgs {
  const void *input[CF_MAX_SEGMENTS];
  int8_t *codes[CF_MAX_SEGMENTS];
  float *scales[CF_MAX_SEGMENTS];
  int64_t unit_end[CF_MAX_SEGMENTS];  // inclusive prefix sum of units per segment
  int nseg;
};

// ---------------------------------------------------------------------------
// TMA-staged quantiser (the main path).
//
// A "tile" is kBlocks blocks of 64 elements (32 KB of input), contiguous in
// memory. Thread 0 streams tiles into a ring of
// kStages shared-memory buffers with bulk copies (cp.async.bulk, completion on
// an mbarrier), so each SM keeps (kStages - 1) tiles of loads in flight no
// matter how many registers the arithmetic needs. Each warp quantises its share
// of the tile from shared memory (4 lanes per block, conflict-free 16-byte
// loads, two-step shuffle absmax) into a triple-buffered shared staging area, and thread 0 writes the tile's codes and
// scales back with bulk stores. Tiles are dealt round-robin to a persistent grid
// of one CTA per SM, across every segment of a grouped launch.
// ---------------------------------------------------------------------------
template <typename T>
struct TmaQuantCfg {
  static constexpr int kThreads = sizeof(T) == 4 ? 256 : 512;
  static constexpr int kStages = 5;
  static constexpr int kBlocks = sizeof(T) == 4 ? 128 : 256;  // quant blocks per tile (32 KB)
  static constexpr int kTileElems = kBlocks * kQuantBlockSize;  // 8192 (f32) / 16384
  static constexpr int kInBytes = kTileElems * static_cast<int>(sizeof(T));
  static constexpr int kWarpElems = kTileElems / (kThreads / kWarp);  // per warp
  static constexpr int kCodeBufs = 3;
  static constexpr size_t kSmemBytes = static_cast<size_t>(kStages) * kInBytes +
                                       kCodeBufs * kTileElems + kCodeBufs * kBlocks * 4 +
                                       kStages * 8 + 16;
};

template <typename T>
__global__ void __launch_bounds__(TmaQuantCfg<T>::kThreads, 1)
    quantize_tma_kernel(const __grid_constant__ GroupedArgs args, unsigned *error_word) {
  using C = TmaQuantCfg<T>;
  extern __shared__ __align__(128) uint8_t smem[];
  uint8_t *in_buf = smem;
  uint8_t *code_buf = smem + C::kStages * C::kInBytes;
  float *scale_buf = reinterpret_cast<float *>(code_buf + C::kCodeBufs * C::kTileElems);
  uint64_t *full = reinterpret_cast<uint64_t *>(scale_buf + C::kCodeBufs * C::kBlocks);
  __shared__ int abort_flag;

  const int tid = threadIdx.x;
  const int64_t total = args.unit_end[args.nseg - 1];
  const int64_t first = blockIdx.x;
  const int64_t step = gridDim.x;
  const int64_t n_mine = first < total ? (total - first + step - 1) / step : 0;

  if (tid == 0) {
    for (int s = 0; s < C::kStages; ++s) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
    abort_flag = 0;
  }
  __syncthreads();

  int seg_p = 0;  // producer's segment cursor (thread 0 only)
  auto issue_load = [&](int64_t j) {
    const int64_t tile = first + j * step;
    while (tile >= args.unit_end[seg_p]) ++seg_p;
    const int64_t seg_begin = seg_p == 0 ? 0 : args.unit_end[seg_p - 1];
    const T *src = static_cast<const T *>(args.input[seg_p]) + (tile - seg_begin) * C::kTileElems;
    const int s = static_cast<int>(j % C::kStages);
    ptx::mbar_expect_tx(&full[s], C::kInBytes);
    ptx::bulk_load(in_buf + s * C::kInBytes, src, C::kInBytes, &full[s]);
  };

  if (tid == 0) {
    for (int64_t j = 0; j < n_mine && j < C::kStages - 1; ++j) issue_load(j);
  }

  int seg_c = 0;
  for (int64_t j = 0; j < n_mine; ++j) {
    const int s = static_cast<int>(j % C::kStages);
    const uint32_t parity = static_cast<uint32_t>((j / C::kStages) & 1);
    const bool timed_out = !ptx::mbar_wait(&full[s], parity);
    if (__syncthreads_or(timed_out)) {
      if (tid == 0) {
        atomicOr(error_word, kDevErrTimeout);
        abort_flag = 1;
      }
      break;
    }
    const int64_t tile = first + j * step;
    while (tile >= args.unit_end[seg_c]) ++seg_c;
    const int64_t seg_begin = seg_c == 0 ? 0 : args.unit_end[seg_c - 1];
    const int64_t elem0 = (tile - seg_begin) * C::kTileElems;

    // Each warp quantises a contiguous 1/kWarps of the tile in steps of 8
    // blocks (Quad layout: 4 lanes per block, conflict-free 16-byte loads).
    using Q = Quad<T>;
    const int lane = tid & (kWarp - 1);
    const int warp = tid / kWarp;
    const int cb = static_cast<int>(j % C::kCodeBufs);
    const uint8_t *src = in_buf + s * C::kInBytes;
    uint8_t *codes_out = code_buf + cb * C::kTileElems;
    float *scales_out = scale_buf + cb * C::kBlocks;
#pragma unroll 2
    for (int st = 0; st < C::kWarpElems / Q::kStepElems; ++st) {
      const int e0 = warp * C::kWarpElems + st * Q::kStepElems;
      Q::step(src + e0 * static_cast<int>(sizeof(T)), codes_out + e0,
              scales_out + e0 / kQuantBlockSize, lane);
    }
    ptx::fence_proxy_async_smem();
    __syncthreads();
    if (tid == 0) {
      ptx::bulk_store(args.codes[seg_c] + elem0, code_buf + cb * C::kTileElems, C::kTileElems);
      ptx::bulk_store(args.scales[seg_c] + elem0 / kQuantBlockSize, scale_buf + cb * C::kBlocks,
                      C::kBlocks * 4);
      ptx::bulk_commit();
      if (j + C::kStages - 1 < n_mine) issue_load(j + C::kStages - 1);
      // The staging buffer written next iteration was last read by the store
      // two iterations ago; at most one group (this one) may still be reading.
      ptx::bulk_wait_read<1>();
    }
  }
  if (tid == 0) {
    ptx::bulk_wait_all();
    // On abort, drain loads still in flight (bounded) before the CTA exits.
    if (abort_flag) {
      for (int s = 0; s < C::kStages; ++s) ptx::mbar_wait(&full[s], 0, 100000000ull);
    }
  }
}

// ---------------------------------------------------------------------------
// Dequantiser: each lane turns 4 codes (one 4-byte load) into one float4 store.
// ---------------------------------------------------------------------------
constexpr int kDequantUnroll = 8;
constexpr int kDequantUnitElems = kDequantUnroll * kWarp * 4;

__global__ void __launch_bounds__(kThreads)
    dequantize_vec_kernel(const int8_t *__restrict__ codes, const float *__restrict__ scales,
                          float *__restrict__ out, int64_t nunits) {
  const int lane = threadIdx.x & (kWarp - 1);
  const int64_t warp = (static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x) / kWarp;
  const int64_t nwarps = static_cast<int64_t>(gridDim.x) * (kThreads / kWarp);
  for (int64_t u = warp; u < nunits; u += nwarps) {
    const int64_t base = u * kDequantUnitElems;
    unsigned w[kDequantUnroll];
    float s[kDequantUnroll];
#pragma unroll
    for (int j = 0; j < kDequantUnroll; ++j) {
      const int64_t e0 = base + j * (kWarp * 4) + lane * 4;
      w[j] = ld_stream_u32(codes + e0);
      s[j] = __ldg(scales + e0 / kQuantBlockSize);
    }
#pragma unroll
    for (int j = 0; j < kDequantUnroll; ++j) {
      const int64_t e0 = base + j * (kWarp * 4) + lane * 4;
      const int q0 = static_cast<int>(static_cast<int8_t>(w[j] & 0xffu));
      const int q1 = static_cast<int>(static_cast<int8_t>((w[j] >> 8) & 0xffu));
      const int q2 = static_cast<int>(static_cast<int8_t>((w[j] >> 16) & 0xffu));
      const int q3 = static_cast<int>(static_cast<int8_t>(w[j] >> 24));
      st_stream_f4(out + e0, __fmul_rn(static_cast<float>(q0), s[j]),
                   __fmul_rn(static_cast<float>(q1), s[j]), __fmul_rn(static_cast<float>(q2), s[j]),
                   __fmul_rn(static_cast<float>(q3), s[j]));
    }
  }
}

__global__ void __launch_bounds__(kThreads)
    dequantize_scalar_kernel(const int8_t *__restrict__ codes, const float *__restrict__ scales,
                             float *__restrict__ out, int64_t first, int64_t count) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kThreads;
  for (int64_t i = first + static_cast<int64_t>(blockIdx.x) * kThreads + threadIdx.x; i < count;
       i += stride) {
    out[i] = __fmul_rn(static_cast<float>(codes[i]), __ldg(scales + i / kQuantBlockSize));
  }
}

// ---------------------------------------------------------------------------
// Host side.
// ---------------------------------------------------------------------------
constexpr int kQuantUnroll = 4;
// Resident CTAs per SM the grid is sized for (256 threads each).
constexpr int kCtasPerSm = 4;

unsigned grid_for(int64_t warps_of_work) {
  const int64_t ctas_needed = (warps_of_work + (kThreads / kWarp) - 1) / (kThreads / kWarp);
  const int64_t cap = static_cast<int64_t>(sm_count()) * kCtasPerSm;
  return static_cast<unsigned>(std::max<int64_t>(1, std::min(ctas_needed, cap)));
}

// Register-path quantisation of elements [0, count) of one tensor (vectorised
// units where aligned, then the scalar tail).
template <typename T, bool kFake>
int quantize_registers(const T *in, int8_t *codes, float *scales, float *fake_out, int64_t count,
                       cudaStream_t stream) {
  using U = QuantUnit<T, kQuantUnroll>;
  const int64_t nblocks = (count + kQuantBlockSize - 1) / kQuantBlockSize;
  const bool vec_ok = aligned_to(in, 16) &&
                      (kFake ? aligned_to(fake_out, 16)
                             : aligned_to(codes, sizeof(T) == 4 ? 4 : 8));
  const int64_t nunits = vec_ok ? count / U::kElems : 0;
  if (nunits > 0) {
    quantize_vec_kernel<T, kQuantUnroll, kFake>
        <<<grid_for(nunits), kThreads, 0, stream>>>(in, codes, scales, fake_out, nunits);
    if (int st = check_launch()) return st;
  }
  const int64_t first_block = nunits * (U::kElems / kQuantBlockSize);
  if (first_block < nblocks) {
    quantize_scalar_kernel<T, kFake><<<grid_for(nblocks - first_block), kThreads, 0, stream>>>(
        in, codes, scales, fake_out, first_block, nblocks, count);
    if (int st = check_launch()) return st;
  }
  return CF_OK;
}

template <typename T>
bool tma_eligible(const void *in, const int8_t *codes, const float *scales) {
  return aligned_to(in, 16) && aligned_to(codes, 16) && aligned_to(scales, 16);
}

template <typename T>
int launch_tma_quant(const GroupedArgs &args, int64_t tiles, cudaStream_t stream) {
  using C = TmaQuantCfg<T>;
  CFB_TRY_CUDA(cudaFuncSetAttribute(quantize_tma_kernel<T>,
                                    cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    static_cast<int>(C::kSmemBytes)));
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(tiles, sm_count())));
  quantize_tma_kernel<T><<<grid, C::kThreads, C::kSmemBytes, stream>>>(args, err);
  return check_launch();
}

// Whole tiles through the TMA-staged kernel, the rest through the register path.
template <typename T, bool kFake>
int quantize_typed(const void *input, int8_t *codes, float *scales, float *fake_out,
                   int64_t count, cudaStream_t stream) {
  const T *in = static_cast<const T *>(input);
  if constexpr (!kFake) {
    using C = TmaQuantCfg<T>;
    const int64_t tiles = tma_eligible<T>(in, codes, scales) ? count / C::kTileElems : 0;
    if (tiles > 0) {
      GroupedArgs args;
      args.nseg = 1;
      args.input[0] = in;
      args.codes[0] = codes;
      args.scales[0] = scales;
      args.unit_end[0] = tiles;
      if (int st = launch_tma_quant<T>(args, tiles, stream)) return st;
      const int64_t done = tiles * C::kTileElems;
      if (done == count) return CF_OK;
      return quantize_registers<T, false>(in + done, codes + done,
                                          scales + done / kQuantBlockSize, nullptr, count - done,
                                          stream);
    }
  }
  return quantize_registers<T, kFake>(in, codes, scales, fake_out, count, stream);
}

template <bool kFake>
int quantize_dispatch(const void *input, int dtype, int8_t *codes, float *scales,
                      float *fake_out, int64_t count, cudaStream_t stream) {
  switch (dtype) {
    case CF_DTYPE_F32:
      return quantize_typed<float, kFake>(input, codes, scales, fake_out, count, stream);
    case CF_DTYPE_BF16:
      return quantize_typed<__nv_bfloat16, kFake>(input, codes, scales, fake_out, count, stream);
    case CF_DTYPE_F16:
      return quantize_typed<__half, kFake>(input, codes, scales, fake_out, count, stream);
    default:
      return CF_ERR_UNSUPPORTED;
  }
}

template <typename T>
int quantize_many_typed(const cf_quant_segment *segs, int nseg, cudaStream_t stream) {
  using C = TmaQuantCfg<T>;
  GroupedArgs args;
  args.nseg = 0;
  int64_t tiles = 0;
  for (int i = 0; i < nseg; ++i) {
    const cf_quant_segment &sg = segs[i];
    if (sg.count == 0) continue;
    const int64_t seg_tiles =
        tma_eligible<T>(sg.input, sg.codes, sg.scales) ? sg.count / C::kTileElems : 0;
    const int64_t done = seg_tiles * C::kTileElems;
    if (seg_tiles > 0) {
      tiles += seg_tiles;
      args.input[args.nseg] = sg.input;
      args.codes[args.nseg] = sg.codes;
      args.scales[args.nseg] = sg.scales;
      args.unit_end[args.nseg] = tiles;
      ++args.nseg;
    }
    if (done < sg.count) {
      const T *in = static_cast<const T *>(sg.input);
      if (int st = quantize_registers<T, false>(in + done, sg.codes + done,
                                                sg.scales + done / kQuantBlockSize, nullptr,
                                                sg.count - done, stream)) {
        return st;
      }
    }
  }
  if (args.nseg == 0) return CF_OK;
  return launch_tma_quant<T>(args, tiles, stream);
}

}  // namespace
}  // namespace cfb

extern "C" {

int64_t cf_quant_scale_count(int64_t count) {
  return count <= 0 ? 0 : (count + cfb::kQuantBlockSize - 1) / cfb::kQuantBlockSize;
}

int cf_quantize_int8(const void *input, int dtype, int8_t *codes, float *scales, int64_t count,
                     cf_stream_t stream) {
  if (count < 0) return CF_ERR_INVALID_ARGUMENT;
  if (count == 0) return CF_OK;
  if (input == nullptr || codes == nullptr || scales == nullptr) return CF_ERR_INVALID_ARGUMENT;
  return cfb::quantize_dispatch<false>(input, dtype, codes, scales, nullptr, count,
                                       reinterpret_cast<cudaStream_t>(stream));
}

int cf_quantize_dequantize(const void *input, int dtype, float *output, int64_t count,
                           cf_stream_t stream) {
  if (count < 0) return CF_ERR_INVALID_ARGUMENT;
  if (count == 0) return CF_OK;
  if (input == nullptr || output == nullptr) return CF_ERR_INVALID_ARGUMENT;
  return cfb::quantize_dispatch<true>(input, dtype, nullptr, nullptr, output, count,
                                      reinterpret_cast<cudaStream_t>(stream));
}

int cf_quantize_int8_many(const cf_quant_segment *segments, int nseg, int dtype,
                          cf_stream_t stream) {
  if (nseg < 0 || (nseg > 0 && segments == nullptr)) return CF_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < nseg; ++i) {
    const cf_quant_segment &sg = segments[i];
    if (sg.count < 0) return CF_ERR_INVALID_ARGUMENT;
    if (sg.count > 0 && (sg.input == nullptr || sg.codes == nullptr || sg.scales == nullptr)) {
      return CF_ERR_INVALID_ARGUMENT;
    }
  }
  if (dtype != CF_DTYPE_F32 && dtype != CF_DTYPE_BF16 && dtype != CF_DTYPE_F16) {
    return CF_ERR_UNSUPPORTED;
  }
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  for (int first = 0; first < nseg; first += CF_MAX_SEGMENTS) {
    const int n = std::min(CF_MAX_SEGMENTS, nseg - first);
    int st = CF_OK;
    switch (dtype) {
      case CF_DTYPE_F32: st = cfb::quantize_many_typed<float>(segments + first, n, s); break;
      case CF_DTYPE_BF16: st = cfb::quantize_many_typed<__nv_bfloat16>(segments + first, n, s); break;
      default: st = cfb::quantize_many_typed<__half>(segments + first, n, s); break;
    }
    if (st != CF_OK) return st;
  }
  return CF_OK;
}

int cf_dequantize_int8(const int8_t *codes, const float *scales, float *output, int64_t count,
                       cf_stream_t stream) {
  if (count < 0) return CF_ERR_INVALID_ARGUMENT;
  if (count == 0) return CF_OK;
  if (codes == nullptr || scales == nullptr || output == nullptr) return CF_ERR_INVALID_ARGUMENT;
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  const bool vec_ok = cfb::aligned_to(codes, 4) && cfb::aligned_to(output, 16);
  const int64_t nunits = vec_ok ? count / cfb::kDequantUnitElems : 0;
  if (nunits > 0) {
    cfb::dequantize_vec_kernel<<<cfb::grid_for(nunits), cfb::kThreads, 0, s>>>(codes, scales,
                                                                              output, nunits);
    if (int st = cfb::check_launch()) return st;
  }
  const int64_t first = nunits * cfb::kDequantUnitElems;
  if (first < count) {
    const int64_t rest = count - first;
    cfb::dequantize_scalar_kernel<<<cfb::grid_for((rest + 31) / 32), cfb::kThreads, 0, s>>>(
        codes, scales, output, first, count);
    if (int st = cfb::check_launch()) return st;
  }
  return CF_OK;
}

}  // extern "C"
