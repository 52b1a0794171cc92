/* The C ABI used from plain C, as a cgo / JNI / FFI binding would see it.
 *
 * TEST INFRASTRUCTURE: compiled with gcc -std=c99 -Wall -Wextra -Werror
 * -pedantic against include/cudaforge_b200.h and linked against
 * libcudaforge_b200.so by tests/test_host.py; runs on a host without a GPU.
 * Every call below returns before touching a device: pure helpers, empty
 * inputs and argument errors. Prints "ok" and exits 0 when all hold.
 */
#include <stdio.h>
#include <string.h>

#include "cudaforge_b200.h"

#define EXPECT(cond)                                               \
  do {                                                             \
    if (!(cond)) {                                                 \
      fprintf(stderr, "line %d: %s\n", __LINE__, #cond);           \
      return 1;                                                    \
    }                                                              \
  } while (0)

int main(void) {
  static float dummy[64];
  void *p = dummy;
  cf_quant_segment seg;

  EXPECT(CF_QUANT_BLOCK_SIZE == 64);
  EXPECT(cf_quant_scale_count(0) == 0 && cf_quant_scale_count(1) == 1);
  EXPECT(cf_quant_scale_count(64) == 1 && cf_quant_scale_count(65) == 2);
  EXPECT(cf_status_string(CF_OK) != NULL && strlen(cf_status_string(CF_ERR_MISALIGNED)) > 0);
  EXPECT(cf_build_info() != NULL);
  EXPECT(cf_lora_linear_workspace_bytes(8192, 16) >= (size_t)8192 * 16 * 2);

  /* empty inputs are no-ops */
  EXPECT(cf_quantize_int8(p, CF_DTYPE_BF16, NULL, NULL, 0, NULL) == CF_OK);
  EXPECT(cf_dequantize_int8(NULL, NULL, NULL, 0, NULL) == CF_OK);
  EXPECT(cf_quantize_int8_many(NULL, 0, CF_DTYPE_F32, NULL) == CF_OK);
  EXPECT(cf_fused_residual_rmsnorm(p, NULL, p, CF_DTYPE_BF16, p, NULL, 0, 4096, 1e-6f,
                                   CF_DTYPE_BF16, NULL) == CF_OK);

  /* argument errors */
  EXPECT(cf_quantize_int8(p, CF_DTYPE_F32, NULL, NULL, -1, NULL) == CF_ERR_INVALID_ARGUMENT);
  EXPECT(cf_quantize_int8(NULL, CF_DTYPE_F32, (int8_t *)p, dummy, 64, NULL) ==
         CF_ERR_INVALID_ARGUMENT);
  memset(&seg, 0, sizeof seg);
  seg.count = -5;
  EXPECT(cf_quantize_int8_many(&seg, 1, CF_DTYPE_F32, NULL) == CF_ERR_INVALID_ARGUMENT);
  EXPECT(cf_fused_residual_rmsnorm(p, p, p, CF_DTYPE_BF16, p, NULL, 4, 64, 1e-6f, CF_DTYPE_BF16,
                                   NULL) == CF_ERR_INVALID_ARGUMENT);
  EXPECT(cf_fused_residual_rmsnorm(p, NULL, p, CF_DTYPE_F16, p, NULL, 4, 64, 1e-6f,
                                   CF_DTYPE_BF16, NULL) == CF_ERR_UNSUPPORTED);
  EXPECT(cf_w8_swiglu_int8(p, NULL, dummy, (int8_t *)p, dummy, p, 32, 128, 128, CF_DTYPE_BF16,
                           NULL) == CF_ERR_INVALID_ARGUMENT);
  puts("ok");
  return 0;
}
