/* Exhaustive check of the quantiser's division-free code path.
 *
 * TEST INFRASTRUCTURE: compiled and run by tests/test_quotient.py on the CPU.
 *
 * For a block scale s = fl32(absmax / 127) with 2^-100 <= s <= 2^100 and
 * r = fl32(1 / s) (correctly rounded), the kernels compute
 *     q0 = fl(x * r);  e = fma(-q0, s, x);  q = fma(e, r, q0)
 * and take the code as rint_half_even(q). The reference computes
 * rint_half_even(fl32(x / s)). This program compares the two codes for every
 * pair (absmax, x) with absmax a positive finite value of the 16-bit format and
 * x any value of that format with |x| <= absmax, and for a large seeded sample
 * of fp32 pairs (plus quotients steered onto half-integers). It prints the
 * number of pairs checked and of mismatches. Build without -ffast-math.
 */
#include <math.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

static float from_bits(uint32_t u) { float f; memcpy(&f, &u, 4); return f; }

static float half_to_float(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t exp = (h >> 10) & 0x1fu, man = h & 0x3ffu;
  if (exp == 0) {
    float f = (float)man * 5.9604644775390625e-08f;
    return sign ? -f : f;
  }
  return from_bits(sign | ((exp + 112u) << 23) | (man << 13));
}

static int code_ref(float x, float s) { return (int)rintf(x / s); }

static int code_fast(float x, float s, float r) {
  const float q0 = x * r;
  const float e = fmaf(-q0, s, x);
  const float q = fmaf(e, r, q0);
  return (int)rintf(q);
}

static int usable(float s) { return s >= 0x1p-100f && s <= 0x1p100f; }

static long long check16(int is_bf16, long long *checked) {
  long long bad = 0;
  for (uint32_t a = 1; a < 0x7c00u || (is_bf16 && a < 0x7f80u); ++a) {
    const float amax = is_bf16 ? from_bits(a << 16) : half_to_float((uint16_t)a);
    const float s = amax / 127.0f;
    if (!usable(s)) continue;
    const float r = 1.0f / s;
    for (uint32_t xb = 0; xb <= a; ++xb) {
      for (int sign = 0; sign < 2; ++sign) {
        const uint16_t h = (uint16_t)(xb | (sign ? 0x8000u : 0u));
        const float x = is_bf16 ? from_bits((uint32_t)h << 16) : half_to_float(h);
        ++*checked;
        if (code_ref(x, s) != code_fast(x, s, r)) {
          if (bad < 5) printf("mismatch %s amax=%a x=%a\n", is_bf16 ? "bf16" : "f16", amax, x);
          ++bad;
        }
      }
    }
  }
  return bad;
}

static uint64_t rng = 0x9e3779b97f4a7c15ull;
static uint64_t next(void) {
  rng ^= rng << 13; rng ^= rng >> 7; rng ^= rng << 17;
  return rng;
}

static long long check32(long long n, long long *checked) {
  long long bad = 0;
  for (long long i = 0; i < n; ++i) {
    const uint64_t u = next();
    /* absmax: random exponent in a wide normal range, random mantissa */
    const int ex = (int)(u % 160) - 80;
    const float amax = ldexpf(1.0f + (float)((u >> 8) & 0x7fffff) / 8388608.0f, ex);
    const float s = amax / 127.0f;
    if (!usable(s)) continue;
    const float r = 1.0f / s;
    float x;
    const int mode = (int)((u >> 40) % 3);
    if (mode == 0) {            /* uniform in [-amax, amax] */
      x = amax * ((float)(int32_t)(next() & 0xffffffffu) / 2147483648.0f);
    } else {                    /* steered onto (k + 1/2) * s, +- a few ulps */
      const int k = (int)(next() % 254) - 127;
      x = ((float)k + 0.5f) * s;
      const int ulps = (int)(next() % 5) - 2;
      uint32_t xb; memcpy(&xb, &x, 4); xb += ulps; memcpy(&x, &xb, 4);
      if (fabsf(x) > amax) x = amax;
    }
    ++*checked;
    if (code_ref(x, s) != code_fast(x, s, r)) {
      if (bad < 5) printf("mismatch f32 amax=%a x=%a\n", amax, x);
      ++bad;
    }
  }
  return bad;
}

int main(int argc, char **argv) {
  const long long n32 = argc > 1 ? atoll(argv[1]) : 200000000LL;
  long long c16 = 0, cbf = 0, c32 = 0;
  const long long bbf = check16(1, &cbf);
  const long long b16 = check16(0, &c16);
  const long long b32 = check32(n32, &c32);
  printf("bf16 pairs %lld mismatches %lld\n", cbf, bbf);
  printf("f16 pairs %lld mismatches %lld\n", c16, b16);
  printf("f32 samples %lld mismatches %lld\n", c32, b32);
  return (bbf || b16 || b32) ? 1 : 0;
}
