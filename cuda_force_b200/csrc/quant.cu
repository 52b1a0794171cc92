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
//   * main path (quantize_tma_kernel): a persistent grid in which every warp
//     streams 1024-element tiles through its own 3-stage shared-memory ring
//     with bulk copies (TMA engine) and writes codes and scales back with bulk
//     stores; tails, misaligned tensors
//     and fake-quant use a register-streaming kernel whose lanes issue UNROLL
//     independent 16-byte loads before touching any of them;
//   * a 64-element block is spread over 16 lanes (f32) or 8 lanes (f16/bf16);
//     the absmax is a shuffle-xor max over those lanes of |x| bit patterns as
//     unsigned integers, which orders non-negative floats exactly and makes a
//     NaN win, the same propagation as torch.amax;
//   * codes: fl32(x / s) is formed without a divide, as q0 = x * r, a residual
//     FMA and one correction FMA (r = fl32(1/s)); the half-to-even rounding is
//     an add of 1.5 * 2^23 whose low bits are the code. Verified equal to the
//     IEEE quotient for all bf16/fp16 (x, absmax) pairs on the CPU; blocks with
//     NaN/inf or extreme scales fall back to the IEEE division;
//   * codes are packed 4 or 8 per store; the register path writes them with
//     streaming stores (st.global.cs).
#include <cuda_bf16.h>
#include <cuda_fp16.h>

#include <algorithm>
#include <type_traits>

#include "cf_common.cuh"
#include "ptx.cuh"
#include "quant_math.cuh"

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

// ---------------------------------------------------------------------------
// Quantisation core shared by every kernel.
// ---------------------------------------------------------------------------
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
__device__ __forceinline__ __nv_bfloat162 as_bf162(uint32_t w) {
  return *reinterpret_cast<__nv_bfloat162 *>(&w);
}
__device__ __forceinline__ uint32_t bf162_bits(__nv_bfloat162 h) {
  return *reinterpret_cast<uint32_t *>(&h);
}
// Packed |x| maximum of a 16-byte bf16 vector, two lanes per instruction;
// __hmax2_nan returns NaN when either operand is NaN.
__device__ __forceinline__ uint32_t vec_absmax_bf16x2(const uint4 &v) {
  const __nv_bfloat162 a = __hmax2_nan(__habs2(as_bf162(v.x)), __habs2(as_bf162(v.y)));
  const __nv_bfloat162 b = __hmax2_nan(__habs2(as_bf162(v.z)), __habs2(as_bf162(v.w)));
  return bf162_bits(__hmax2_nan(a, b));
}
// bf16: the bf16 pattern shifted left by 16 is the float pattern.
__device__ __forceinline__ unsigned vec_absmax_bits(const uint4 &v, __nv_bfloat16 *) {
  const unsigned m = vec_absmax_bf16x2(v);
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
    const float s = block_scale(m);
    const float r = __frcp_rn(s);
    const bool fast = quotient_path_ok(m, s);
    float f[kPerVec];
    if constexpr (kPerVec == 4) {
      unpack(v, f);
    } else {
      unpack(v, f, static_cast<T *>(nullptr));
    }
    uint32_t mb[kPerVec];
#pragma unroll
    for (int e = 0; e < kPerVec; ++e) mb[e] = fast ? code_bits_fast(f[e], s, r) : code_bits_exact(f[e], s);
#pragma unroll
    for (int w = 0; w < kWords; ++w) {
      codes[w] = __byte_perm(__byte_perm(mb[4 * w], mb[4 * w + 1], 0x0040u),
                             __byte_perm(mb[4 * w + 2], mb[4 * w + 3], 0x0040u), 0x5410u);
    }
    scale = s;
  }
};


// Shared-memory layout of the TMA kernel: 4 lanes per 64-element block, 16
// elements (kChunks 16-byte chunks) per lane, 8 blocks per warp step.
//
// Lane 4b+i of a step owns chunks 4*((j + b/2) % kChunks) + i (j = 0 ..
// kChunks-1) of block b. Within one load instruction j the 32 chunk indices
// then cover every residue mod 8 exactly four times, so the 16-byte shared
// loads are bank-conflict-free while each lane's chunks stay in one block; the
// code stores (4 or 8 bytes per chunk) spread evenly over the banks too.
template <typename T>
struct Quad {
  static constexpr int kPerChunk = 16 / static_cast<int>(sizeof(T));  // elements per chunk
  static constexpr int kChunks = 16 / kPerChunk;                       // chunks per lane
  static constexpr int kStepElems = 8 * kQuantBlockSize;               // 8 blocks per step

  static __device__ __forceinline__ int chunk_of(int lane, int j) {
    const int b = lane >> 2;
    return 4 * ((j + (b >> 1)) % kChunks) + (lane & 3);
  }

  // Per-lane byte offsets inside a step, fixed for the whole kernel.
  struct Offsets {
    int in[kChunks];    // input chunk offsets (bytes)
    int code[kChunks];  // code offsets (bytes = elements)
    int block;          // block of this lane within the step
  };

  static __device__ __forceinline__ Offsets offsets(int lane) {
    Offsets o;
    o.block = lane >> 2;
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int elem = o.block * kQuantBlockSize + chunk_of(lane, j) * kPerChunk;
      o.in[j] = elem * static_cast<int>(sizeof(T));
      o.code[j] = elem;
    }
    return o;
  }

  // Quantises one warp step: reads from `src` (the step's 512 elements),
  // writes codes to `codes` (512 bytes) and 8 scales to `scales`.
  static __device__ __forceinline__ void step(const uint8_t *src, uint8_t *codes, float *scales,
                                              const Offsets &o, int lane) {
    uint4 v[kChunks];
#pragma unroll
    for (int j = 0; j < kChunks; ++j) v[j] = *reinterpret_cast<const uint4 *>(src + o.in[j]);
    unsigned m = 0u;
    if constexpr (std::is_same_v<T, __nv_bfloat16>) {
      uint32_t packed = vec_absmax_bf16x2(v[0]);
#pragma unroll
      for (int j = 1; j < kChunks; ++j) {
        packed = bf162_bits(__hmax2_nan(as_bf162(packed), as_bf162(vec_absmax_bf16x2(v[j]))));
      }
      m = max(packed << 16, packed & 0xffff0000u);
    } else {
#pragma unroll
      for (int j = 0; j < kChunks; ++j) m = max(m, vec_absmax_bits(v[j], static_cast<T *>(nullptr)));
    }
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 2));
    m = max(m, __shfl_xor_sync(0xffffffffu, m, 1));
    const float s = block_scale(m);
    const bool fast = quotient_path_ok(m, s);
    const float r = __frcp_rn(s);
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
#pragma unroll
    for (int e = 0; e < 16; ++e) mb[e] = code_bits_fast(f[e], s, r);
    if (__any_sync(0xffffffffu, !fast)) {
      // Blocks holding NaN/inf or with extreme scales: IEEE division.
#pragma unroll
      for (int e = 0; e < 16; ++e) mb[e] = fast ? mb[e] : code_bits_exact(f[e], s);
    }
#pragma unroll
    for (int j = 0; j < kChunks; ++j) {
      const int e0 = j * kPerChunk;
      uint8_t *dst = codes + o.code[j];
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
    if ((lane & 3) == 0) scales[o.block] = s;
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
    if (i0 < count) {
      const int q = static_cast<int8_t>(code_bits_exact(x0, s) & 0xffu);
      if constexpr (kFake) fake_out[i0] = __fmul_rn(static_cast<float>(q), s);
      else codes[i0] = static_cast<int8_t>(q);
    }
    if (i1 < count) {
      const int q = static_cast<int8_t>(code_bits_exact(x1, s) & 0xffu);
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
// Every warp runs its own pipeline; there is no CTA-wide barrier. A warp tile
// is 1024 contiguous elements (16 blocks). Lane 0 keeps kStages - 1 tiles of
// input in flight with bulk copies (cp.async.bulk global -> shared, completion
// on the warp's mbarriers); the warp quantises a landed tile in two 8-block
// steps (Quad layout), stages 1 KB of codes and 64 B of scales in shared
// memory, and lane 0 writes them back with bulk stores (shared -> global).
// Warp tiles are dealt round-robin over a persistent grid of one CTA per SM,
// across every segment of a grouped launch.
// ---------------------------------------------------------------------------
template <typename T>
struct TmaQuantCfg {
  static constexpr int kWarps = 20;
  static constexpr int kThreads = kWarps * kWarp;
  static constexpr int kStages = sizeof(T) == 4 ? 4 : 3;
  static constexpr int kCodeBufs = 2;
  // per warp tile: 2 KB of input for every dtype (512 fp32 / 1024 16-bit elements)
  static constexpr int kTileElems = 2048 / static_cast<int>(sizeof(T));
  static constexpr int kBlocks = kTileElems / kQuantBlockSize;  // 16
  static constexpr int kInBytes = kTileElems * static_cast<int>(sizeof(T));
  // per warp: input ring, code staging, scale staging, barriers
  static constexpr int kWarpBytes = kStages * kInBytes + kCodeBufs * kTileElems +
                                    kCodeBufs * kBlocks * 4 + 64;
  static constexpr size_t kSmemBytes = static_cast<size_t>(kWarps) * kWarpBytes;
};

template <typename T>
__global__ void __launch_bounds__(TmaQuantCfg<T>::kThreads, 1)
    quantize_tma_kernel(const __grid_constant__ GroupedArgs args, unsigned *error_word) {
  using C = TmaQuantCfg<T>;
  using Q = Quad<T>;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  uint8_t *mine = smem + warp * C::kWarpBytes;
  uint8_t *in_buf = mine;
  uint8_t *code_buf = in_buf + C::kStages * C::kInBytes;
  float *scale_buf = reinterpret_cast<float *>(code_buf + C::kCodeBufs * C::kTileElems);
  uint64_t *full = reinterpret_cast<uint64_t *>(scale_buf + C::kCodeBufs * C::kBlocks);

  const int64_t total = args.unit_end[args.nseg - 1];
  const int64_t first = static_cast<int64_t>(blockIdx.x) * C::kWarps + warp;
  const int64_t step = static_cast<int64_t>(gridDim.x) * C::kWarps;
  const int64_t n_mine = first < total ? (total - first + step - 1) / step : 0;

  if (lane == 0) {
    for (int s = 0; s < C::kStages; ++s) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
  }
  __syncwarp();

  int seg_p = 0;    // lane 0's segment cursor for loads
  int p_stage = 0;  // lane 0's next load stage (loads are issued in tile order)
  auto issue_load = [&](int64_t j) {
    const int64_t tile = first + j * step;
    while (tile >= args.unit_end[seg_p]) ++seg_p;
    const int64_t seg_begin = seg_p == 0 ? 0 : args.unit_end[seg_p - 1];
    const T *src = static_cast<const T *>(args.input[seg_p]) + (tile - seg_begin) * C::kTileElems;
    const int s = p_stage;
    p_stage = p_stage + 1 == C::kStages ? 0 : p_stage + 1;
    ptx::mbar_expect_tx(&full[s], C::kInBytes);
    ptx::bulk_load(in_buf + s * C::kInBytes, src, C::kInBytes, &full[s]);
  };
  if (lane == 0) {
    for (int64_t j = 0; j < n_mine && j < C::kStages - 1; ++j) issue_load(j);
  }

  const typename Q::Offsets offs = Q::offsets(lane);
  int seg_c = 0;
  int64_t issued = n_mine < C::kStages - 1 ? n_mine : C::kStages - 1;
  bool aborted = false;
  int s = 0, cb = 0;
  uint32_t parity = 0;
  for (int64_t j = 0; j < n_mine; ++j) {
    const bool ok = ptx::mbar_wait_idle(&full[s], parity);
    if (__any_sync(0xffffffffu, !ok)) {
      if (lane == 0) atomicOr(error_word, kDevErrTimeout);
      aborted = true;
      break;
    }
    const int64_t tile = first + j * step;
    while (tile >= args.unit_end[seg_c]) ++seg_c;
    const int64_t seg_begin = seg_c == 0 ? 0 : args.unit_end[seg_c - 1];
    const int64_t elem0 = (tile - seg_begin) * C::kTileElems;

    const uint8_t *src = in_buf + s * C::kInBytes;
    uint8_t *codes_out = code_buf + cb * C::kTileElems;
    float *scales_out = scale_buf + cb * C::kBlocks;
#pragma unroll
    for (int st = 0; st < C::kTileElems / Q::kStepElems; ++st) {
      const int e0 = st * Q::kStepElems;
      Q::step(src + e0 * static_cast<int>(sizeof(T)), codes_out + e0,
              scales_out + e0 / kQuantBlockSize, offs, lane);
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      ptx::bulk_store(args.codes[seg_c] + elem0, codes_out, C::kTileElems);
      ptx::bulk_store(args.scales[seg_c] + elem0 / kQuantBlockSize, scales_out, C::kBlocks * 4);
      ptx::bulk_commit();
      // The next tile goes into the stage of tile j - 1, whose reads finished
      // before the previous iteration's __syncwarp.
      if (issued < n_mine) issue_load(issued++);
      // The staging buffer written next was last read by the store of tile
      // j + 1 - kCodeBufs: allow only the kCodeBufs - 1 newest stores pending.
      ptx::bulk_wait_read<C::kCodeBufs - 1>();
    }
    __syncwarp();
    if (++s == C::kStages) {
      s = 0;
      parity ^= 1u;
    }
    cb = cb + 1 == C::kCodeBufs ? 0 : cb + 1;
  }
  if (lane == 0) {
    ptx::bulk_wait_all();
    if (aborted) {
      // Let loads still in flight land (bounded) before the CTA's shared memory goes away.
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

// Bulk-copy staged dequantiser: like the TMA quantiser, every warp runs its
// own pipeline. Lane 0 keeps tiles of 2048 codes and their 32 scales in
// flight with cp.async.bulk (3 stages); the warp turns a landed tile into
// 8 KB of fp32 in a double-buffered staging slot, and lane 0 writes the slot
// back with one bulk store. Whole tiles only; 16-byte aligned operands.
struct DequantTmaCfg {
  static constexpr int kWarps = 8;
  static constexpr int kThreads = kWarps * kWarp;
  static constexpr int kTile = 2048;                      // codes per tile
  static constexpr int kScales = kTile / kQuantBlockSize;  // 32
  static constexpr int kStages = 3;
  static constexpr int kInBytes = kTile + kScales * 4;     // 2176
  static constexpr int kOutBufs = 2;
  static constexpr int kOutBytes = kTile * 4;              // 8 KB
  static constexpr int kWarpBytes = kStages * kInBytes + kOutBufs * kOutBytes + 64;
  static constexpr size_t kSmemBytes = static_cast<size_t>(kWarps) * kWarpBytes;
  static_assert(kInBytes % 16 == 0 && kWarpBytes % 16 == 0, "bulk copy alignment");
};

__global__ void __launch_bounds__(DequantTmaCfg::kThreads, 1)
    dequantize_tma_kernel(const int8_t *__restrict__ codes, const float *__restrict__ scales,
                          float *__restrict__ out, int64_t ntiles, unsigned *error_word) {
  using C = DequantTmaCfg;
  extern __shared__ __align__(128) uint8_t smem[];
  const int lane = threadIdx.x & (kWarp - 1);
  const int warp = threadIdx.x / kWarp;
  uint8_t *mine = smem + warp * C::kWarpBytes;
  uint8_t *out_buf = mine + C::kStages * C::kInBytes;
  uint64_t *full = reinterpret_cast<uint64_t *>(out_buf + C::kOutBufs * C::kOutBytes);
  const int64_t first = static_cast<int64_t>(blockIdx.x) * C::kWarps + warp;
  const int64_t step = static_cast<int64_t>(gridDim.x) * C::kWarps;
  const int64_t n_mine = first < ntiles ? (ntiles - first + step - 1) / step : 0;
  if (lane == 0) {
    for (int s = 0; s < C::kStages; ++s) ptx::mbar_init(&full[s], 1);
    ptx::fence_mbar_init();
  }
  __syncwarp();
  int p_stage = 0;
  auto issue_load = [&](int64_t j) {
    const int64_t tile = first + j * step;
    uint8_t *dst = mine + p_stage * C::kInBytes;
    ptx::mbar_expect_tx(&full[p_stage], C::kInBytes);
    ptx::bulk_load(dst, codes + tile * C::kTile, C::kTile, &full[p_stage]);
    ptx::bulk_load(dst + C::kTile, scales + tile * C::kScales, C::kScales * 4, &full[p_stage]);
    p_stage = p_stage + 1 == C::kStages ? 0 : p_stage + 1;
  };
  if (lane == 0) {
    for (int64_t j = 0; j < n_mine && j < C::kStages - 1; ++j) issue_load(j);
  }
  int64_t issued = n_mine < C::kStages - 1 ? n_mine : C::kStages - 1;
  bool aborted = false;
  int s = 0, ob = 0;
  uint32_t parity = 0;
  for (int64_t j = 0; j < n_mine; ++j) {
    const bool ok = ptx::mbar_wait_idle(&full[s], parity);
    if (__any_sync(0xffffffffu, !ok)) {
      if (lane == 0) atomicOr(error_word, kDevErrTimeout);
      aborted = true;
      break;
    }
    const uint8_t *in = mine + s * C::kInBytes;
    const float *sc = reinterpret_cast<const float *>(in + C::kTile);
    float *dst = reinterpret_cast<float *>(out_buf + ob * C::kOutBytes);
    // Lane l handles codes [16 i + 4 l, +4) of each 512-code quarter: 4-byte
    // shared loads and 16-byte shared stores, both conflict-free.
#pragma unroll
    for (int i = 0; i < C::kTile / (kWarp * 4); ++i) {
      const int e = i * (kWarp * 4) + lane * 4;
      const uint32_t w = *reinterpret_cast<const uint32_t *>(in + e);
      const float scale = sc[e / kQuantBlockSize];
      const int q0 = static_cast<int>(static_cast<int8_t>(w & 0xffu));
      const int q1 = static_cast<int>(static_cast<int8_t>((w >> 8) & 0xffu));
      const int q2 = static_cast<int>(static_cast<int8_t>((w >> 16) & 0xffu));
      const int q3 = static_cast<int>(static_cast<int8_t>(w >> 24));
      *reinterpret_cast<float4 *>(dst + e) =
          make_float4(__fmul_rn(static_cast<float>(q0), scale), __fmul_rn(static_cast<float>(q1), scale),
                      __fmul_rn(static_cast<float>(q2), scale), __fmul_rn(static_cast<float>(q3), scale));
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
      const int64_t tile = first + j * step;
      ptx::bulk_store(out + tile * C::kTile, dst, C::kOutBytes);
      ptx::bulk_commit();
      // The input stage read just now is refilled next; the staging slot
      // written next was last read by the store of tile j + 1 - kOutBufs.
      if (issued < n_mine) issue_load(issued++);
      ptx::bulk_wait_read<C::kOutBufs - 1>();
    }
    __syncwarp();
    if (++s == C::kStages) {
      s = 0;
      parity ^= 1u;
    }
    ob ^= 1;
  }
  if (lane == 0) {
    ptx::bulk_wait_all();
    if (aborted) {
      for (int st = 0; st < C::kStages; ++st) ptx::mbar_wait(&full[st], 0, 100000000ull);
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
  if (int st = allow_dynamic_smem<quantize_tma_kernel<T>>(C::kSmemBytes)) return st;
  unsigned *err = device_error_word();
  if (err == nullptr) return record_cuda_error(cudaGetLastError());
  const int64_t ctas = (tiles + C::kWarps - 1) / C::kWarps;
  const unsigned grid = static_cast<unsigned>(std::max<int64_t>(1, std::min<int64_t>(ctas, sm_count())));
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
  using DC = cfb::DequantTmaCfg;
  // Large tensors: whole 2048-code tiles through the bulk-copy kernel, the rest
  // below. At 1 G elements it moves 5740 GB/s against 5659 for the register
  // path; at benchmark config 1's 16.7 M elements its pipeline fill costs more
  // than it saves (3875 against 4155 GB/s), so smaller tensors stay below.
  constexpr int64_t kBulkMin = int64_t{1} << 26;
  if (cfb::aligned_to(codes, 16) && cfb::aligned_to(scales, 16) && cfb::aligned_to(output, 16) &&
      count >= kBulkMin) {
    if (int st = cfb::allow_dynamic_smem<cfb::dequantize_tma_kernel>(DC::kSmemBytes)) return st;
    unsigned *err = cfb::device_error_word();
    if (err == nullptr) return cfb::record_cuda_error(cudaGetLastError());
    const int64_t ntiles = count / DC::kTile;
    const int64_t ctas = (ntiles + DC::kWarps - 1) / DC::kWarps;
    const unsigned grid = static_cast<unsigned>(
        std::max<int64_t>(1, std::min<int64_t>(ctas, cfb::sm_count())));
    cfb::dequantize_tma_kernel<<<grid, DC::kThreads, DC::kSmemBytes, s>>>(codes, scales, output,
                                                                          ntiles, err);
    if (int st = cfb::check_launch()) return st;
    const int64_t done = ntiles * DC::kTile;
    codes += done;
    scales += done / cfb::kQuantBlockSize;
    output += done;
    count -= done;
    if (count == 0) return CF_OK;
  }
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
