// Exact block-INT8 quantisation arithmetic shared by the kernels that produce
// codes (the quantiser and the fused LoRA merge): scale = fl32(absmax / 127)
// (1 when not > 0), code = clamp(rint_half_even(fl32(x / scale)), -127, 127),
// as the reference computes it (cuda/src/quantization.cu:34-45,
// cpp/src/bindings.cpp:298-318).
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace cfb {

// Block scale from the absmax bit pattern: fl32(absmax / 127), or 1 when that
// is not > 0. A NaN pattern (above 0x7f800000) gives NaN / 127 = NaN -> 1.
__device__ __forceinline__ float block_scale(unsigned absmax_bits) {
  const float s = __fdiv_rn(__uint_as_float(absmax_bits), 127.0f);
  return s > 0.0f ? s : 1.0f;
}

__device__ __forceinline__ int clamp_code(int v) { return min(max(v, -127), 127); }

// Division-free code of one element. With r = fl32(1/s) (correctly rounded)
// and s in [2^-100, 2^100]:
//   q0 = fl(x * r);  e = fma(-q0, s, x) (exact residual);  q = fma(e, r, q0)
// gives q = fl32(x / s) (Markstein's correction step); the code is then
// rint_half_even(q), produced by adding 1.5 * 2^23, which leaves the integer in
// the low bits of the sum (the code byte is read from there; |q| <= 127 needs
// no clamp). tests/native/verify_quotient.c checks this against the IEEE
// division for every bf16 and fp16 (x, absmax) pair and a large fp32 sample.
__device__ __forceinline__ uint32_t code_bits_fast(float x, float s, float r) {
  const float q0 = __fmul_rn(x, r);
  const float e = __fmaf_rn(-q0, s, x);
  const float q = __fmaf_rn(e, r, q0);
  return __float_as_uint(__fadd_rn(q, 12582912.0f));  // 1.5 * 2^23
}

// Reference-exact code by IEEE division, for every other block.
__device__ __forceinline__ uint32_t code_bits_exact(float x, float s) {
  return static_cast<uint32_t>(clamp_code(__float2int_rn(__fdiv_rn(x, s))));
}

// Blocks on the division-free path: no NaN/inf in the block and a scale whose
// residual arithmetic stays in the normal range.
__device__ __forceinline__ bool quotient_path_ok(unsigned absmax_bits, float s) {
  return absmax_bits < 0x7f800000u && s >= 0x1p-100f && s <= 0x1p100f;
}

}  // namespace cfb
