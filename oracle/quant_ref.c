/* Plain-C restatement of the reference's block-INT8 quantisation.
 *
 * TEST INFRASTRUCTURE ONLY: never linked into the product.
 *
 * Follows python/cudaforge/ops.py:215-240 and cpp/src/bindings.cpp:298-329:
 *   scale = fl32(absmax / 127.0f), 1.0f when not > 0 (absmax NaN -> NaN -> 1);
 *   code  = clamp(rint(fl32(x / scale)), -127, 127), NaN -> 0 (round half to
 *           even: the default FE_TONEAREST mode of rintf);
 *   deq   = fl32(code * scale).
 * Must be built without -ffast-math (see Makefile). */
#include <math.h>
#include <stdint.h>
#include <string.h>

#define QBLOCK 64

static float bf16_to_f32(uint16_t h) {
  uint32_t u = (uint32_t)h << 16;
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static float f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu;
  const uint32_t man = h & 0x3ffu;
  uint32_t u;
  if (exp == 0) {
    if (man == 0) {
      u = sign;
    } else { /* subnormal half: value = man * 2^-24, exact in float */
      float f = (float)man * 5.9604644775390625e-08f;
      memcpy(&u, &f, sizeof u);
      u |= sign;
    }
  } else if (exp == 31) {
    u = sign | 0x7f800000u | (man << 13);
  } else {
    u = sign | ((exp + 112u) << 23) | (man << 13);
  }
  float f;
  memcpy(&f, &u, sizeof f);
  return f;
}

static float load(const void *in, int dtype, int64_t i) {
  switch (dtype) {
    case 0: return ((const float *)in)[i];
    case 1: return f16_to_f32(((const uint16_t *)in)[i]);
    default: return bf16_to_f32(((const uint16_t *)in)[i]);
  }
}

/* dtype: 0 = f32, 1 = f16, 2 = bf16 (the cf_dtype codes). */
void oracle_quantize(const void *in, int dtype, int8_t *codes, float *scales, int64_t count) {
  const int64_t nblocks = (count + QBLOCK - 1) / QBLOCK;
  for (int64_t b = 0; b < nblocks; ++b) {
    float absmax = 0.0f;
    int has_nan = 0;
    for (int j = 0; j < QBLOCK; ++j) {
      const int64_t i = b * QBLOCK + j;
      const float v = i < count ? fabsf(load(in, dtype, i)) : 0.0f;
      if (isnan(v)) has_nan = 1;
      else if (v > absmax) absmax = v;
    }
    float s = has_nan ? NAN : absmax / 127.0f;
    if (!(s > 0.0f)) s = 1.0f;
    scales[b] = s;
    for (int j = 0; j < QBLOCK; ++j) {
      const int64_t i = b * QBLOCK + j;
      if (i >= count) break;
      float q = rintf(load(in, dtype, i) / s);
      if (isnan(q)) q = 0.0f;
      if (q > 127.0f) q = 127.0f;
      if (q < -127.0f) q = -127.0f;
      codes[i] = (int8_t)q;
    }
  }
}

void oracle_dequantize(const int8_t *codes, const float *scales, float *out, int64_t count) {
  for (int64_t i = 0; i < count; ++i) out[i] = (float)codes[i] * scales[i / QBLOCK];
}
