/*
 * cudaforge_b200.h — C ABI of the B200 (sm_100a) quantised-linear hot path.
 *
 * Every entry point takes plain device pointers, 64-bit element counts, a
 * dtype code and a CUDA stream, launches asynchronously on that stream and
 * returns a cf_status code. Nothing here allocates device memory: outputs and
 * the optional workspace are owned by the caller, exactly like the launchers
 * of the reference (CudaForge) whose interfaces these entry points replace.
 *
 * Counts are int64_t. The reference launchers take `int count`
 * (cuda/include/cudaforge/quantization.cuh:40-48; cpp/src/bindings.cpp:202,217),
 * which overflows for tensors above 2^31 elements.
 *
 * Block quantisation contract (identical to the reference):
 *   blocks of CF_QUANT_BLOCK_SIZE consecutive elements of the flattened tensor,
 *   scale_b = fl32(absmax_b / 127), replaced by 1.0 when it is not > 0,
 *   code_i  = clamp(rint_half_even(fl32(x_i / scale_b)), -127, 127), NaN -> 0,
 *   dequant = fl32(code_i * scale_b).
 */
#ifndef CUDAFORGE_B200_H_
#define CUDAFORGE_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define CF_API __attribute__((visibility("default")))
#else
#define CF_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Same value as kQuantBlockSize (reference cuda/include/cudaforge/quantization.cuh:18). */
#define CF_QUANT_BLOCK_SIZE 64

/* A cudaStream_t. Declared here so the header needs no CUDA include. */
typedef struct CUstream_st *cf_stream_t;

typedef enum cf_status {
  CF_OK = 0,
  CF_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, shape mismatch   */
  CF_ERR_UNSUPPORTED = 2,      /* dtype / layout / shape this build cannot run */
  CF_ERR_MISALIGNED = 3,       /* a pointer violates the documented alignment  */
  CF_ERR_CUDA = 4,             /* a CUDA runtime call failed; see cf_last_cuda_error() */
  CF_ERR_DEVICE_TIMEOUT = 5,   /* a bounded device-side wait gave up            */
  CF_ERR_WORKSPACE = 6,        /* workspace missing or smaller than required    */
  CF_ERR_NO_DEVICE = 7         /* current device is not an sm_100 part          */
} cf_status;

typedef enum cf_dtype {
  CF_DTYPE_F32 = 0,
  CF_DTYPE_F16 = 1,
  CF_DTYPE_BF16 = 2
} cf_dtype;

/* Storage order of a 2-D operand. "REF" is the order the reference op uses,
 * "T" is its transpose (contiguous). For W: REF = [in, out] (reference
 * lora_linear, cuda/include/cudaforge/lora_linear.cuh:22-31), T = [out, in]
 * (nn.Linear). For A: REF = [in, rank], T = [rank, in]. For B: REF =
 * [rank, out], T = [out, rank]. T is what training/lora.py stores. */
typedef enum cf_layout {
  CF_LAYOUT_REF = 0,
  CF_LAYOUT_T = 1
} cf_layout;

/* ---- block INT8 quantisation -------------------------------------------- */

/* Number of block scales for `count` elements: ceil(count / 64), 0 for count <= 0.
 * Replaces quant_scale_count (reference cuda/src/quantization.cu:80-82). */
CF_API int64_t cf_quant_scale_count(int64_t count);

/* input: `count` elements of `dtype` (f32, f16 or bf16); codes: int8[count];
 * scales: float[cf_quant_scale_count(count)].
 * Replaces launch_quantize_int8 (reference cuda/include/cudaforge/quantization.cuh:40-41,
 * kernel cuda/src/quantization.cu:18-47), which accepts f32 only. */
CF_API int cf_quantize_int8(const void *input, int dtype, int8_t *codes, float *scales,
                     int64_t count, cf_stream_t stream);

/* codes: int8[count]; scales: float[cf_quant_scale_count(count)]; output: float[count].
 * Replaces launch_dequantize_int8 (reference quantization.cuh:44-45, kernel
 * quantization.cu:49-57). */
CF_API int cf_dequantize_int8(const int8_t *codes, const float *scales, float *output,
                       int64_t count, cf_stream_t stream);

/* Quantise then dequantise in one pass ("fake quantisation"); output float[count].
 * Replaces launch_quantize_dequantize (reference quantization.cuh:50-51,
 * kernel quantization.cu:59-76). */
CF_API int cf_quantize_dequantize(const void *input, int dtype, float *output, int64_t count,
                           cf_stream_t stream);

/* One tensor of a grouped quantisation. */
typedef struct cf_quant_segment {
  const void *input;
  int8_t *codes;
  float *scales;
  int64_t count;
} cf_quant_segment;

/* Quantises `nseg` independent tensors of one dtype in a single launch (the
 * segment table travels as a kernel parameter, at most CF_MAX_SEGMENTS per
 * launch; longer lists are split into several launches). Each segment has the
 * semantics of cf_quantize_int8. No counterpart launcher in the reference: it
 * is the batched form of launch_quantize_int8 used to quantise a whole layer
 * stack without one launch per tensor. */
#define CF_MAX_SEGMENTS 256
CF_API int cf_quantize_int8_many(const cf_quant_segment *segments, int nseg, int dtype,
                          cf_stream_t stream);

/* ---- LoRA linear --------------------------------------------------------- */

/* y[m, n] = sum_k x[m,k] W[k,n] + scale * sum_j (sum_k x[m,k] A[k,j]) B[j,n]
 * x: [m, k] row-major, y: [m, n] row-major, all operands of `dtype` (f32,
 * f16 or bf16), fp32 accumulation. f32 runs on the tensor cores as three tf32
 * products of a hi/lo operand split (hi*hi + hi*lo + lo*hi), which keeps fp32
 * accuracy. `w`, `a`, `b` are stored as described by cf_layout.
 * Requirements: rows of whole 16-byte units (k and n multiples of 8 for
 * f16/bf16, of 4 for f32; zero-pad otherwise), rank in {16, 32, 64} (smaller
 * ranks are zero-padded by the caller), all pointers 16-byte aligned.
 * Workspace: cf_lora_linear_workspace_bytes(m, rank) bytes of device memory
 * (enough for every dtype), 16-byte aligned, holding the down-projection
 * P = scale * x A between two launches. Replaces launch_lora_linear (reference
 * cuda/include/cudaforge/lora_linear.cuh:45-48) and lora_workspace_bytes
 * (cuda/src/lora_linear.cu:218-223), whose kernels are f32 only. */
CF_API size_t cf_lora_linear_workspace_bytes(int64_t m, int64_t rank);
CF_API int cf_lora_linear(const void *x, const void *w, int w_layout, const void *a, int a_layout,
                   const void *b, int b_layout, void *y, int64_t m, int64_t k, int64_t n,
                   int64_t rank, float scale, int dtype, void *workspace,
                   size_t workspace_bytes, cf_stream_t stream);

/* c[m, n] = a[m, k] b[k, n] in fp32 on the tensor cores, a and c row-major,
 * b stored as cf_layout says. precise != 0: three tf32 products of a hi/lo
 * split, fp32 accuracy (replaces launch_matmul, reference
 * cuda/include/cudaforge/lora_linear.cuh:58-59, CUDA-core FMA); precise == 0:
 * one tf32 product (replaces launch_matmul_tensor_core,
 * cuda/include/cudaforge/tensor_core_matmul.cuh:40-41, TF32 WMMA, whose shape
 * restrictions do not apply here). Requirements: k and n multiples of 4,
 * pointers 16-byte aligned. */
CF_API int cf_matmul_f32(const float *a, const float *b, int b_layout, float *c, int64_t m,
                         int64_t n, int64_t k, int precise, cf_stream_t stream);

/* Same product with W given as block-INT8: w_codes int8[n, k] (the output of
 * cf_quantize_int8 on an nn.Linear weight [out, in]) and w_scales
 * float[n * k / 64]. Semantics: lora_linear(x, dequantize(w_codes, w_scales)^T,
 * a, b, scale). No counterpart in the reference, which has no INT8-weight
 * linear; its semantic definition composes the reference's dequantize_int8
 * (cpp/src/bindings.cpp:320-329) with lora_linear (bindings.cpp:255-258). */
CF_API int cf_lora_linear_int8(const void *x, const int8_t *w_codes, const float *w_scales,
                        const void *a, int a_layout, const void *b, int b_layout, void *y,
                        int64_t m, int64_t k, int64_t n, int64_t rank, float scale, int dtype,
                        void *workspace, size_t workspace_bytes, cf_stream_t stream);

/* RMSNorm (with an optional residual add) folded into the W8 + LoRA linear:
 *   residual_out = x + residual                 (when residual is given)
 *   h = residual given ? residual_out : x
 *   y = lora_linear_int8(rmsnorm(h, norm_weight, eps), w_codes, w_scales, a, b, scale)
 * the composition of the reference's fused_residual_rmsnorm and its linear
 * in a LLaMA block (python/cudaforge/ops.py:335-382 then :289-332, as
 * examples/transformer_block.py:84-87 chain them; no single counterpart).
 * For m > 128 the normalised activations are never written: one pass writes
 * residual_out and each row's 1/rms; the W8 kernel multiplies every code by
 * the norm weight of its input feature as it converts it and every output
 * row by its row scale; the adapter's A is pre-multiplied by the norm weight.
 * m <= 128 normalises into the workspace and runs the decode kernel.
 * bf16/f16 only; norm_weight in the activation dtype; rank 16, 32 or 64;
 * workspace >= cf_rmsnorm_lora_linear_int8_workspace_bytes (256-byte aligned). */
CF_API size_t cf_rmsnorm_lora_linear_int8_workspace_bytes(int64_t m, int64_t k, int64_t rank);
CF_API int cf_rmsnorm_lora_linear_int8(const void *x, const void *residual,
                                       const void *norm_weight, float eps, const int8_t *w_codes,
                                       const float *w_scales, const void *a, int a_layout,
                                       const void *b, int b_layout, void *y, void *residual_out,
                                       int64_t m, int64_t k, int64_t n, int64_t rank, float scale,
                                       int dtype, void *workspace, size_t workspace_bytes,
                                       cf_stream_t stream);

/* Column-sharded W8 linear with the output all-gather fused into the kernel.
 * This rank computes output features [col0, col0 + n) (its rows of the int8
 * weight, w_codes [n, k], and its columns of b) and writes them into every
 * destination y_dest[0 .. n_dest-1]: each a [m, ldy] row-major matrix,
 * typically the same buffer on each GPU of a tensor-parallel group mapped into
 * this process (peer / symmetric memory over NVLink). y_dest[self_dest] is
 * this GPU's own copy. The epilogue stages each 32-row x 128-column block of
 * a finished tile in shared memory and TMA-stores it to its own copy, then to
 * every other destination. 1 <= n_dest <= 8, 0 <= self_dest <
 * n_dest, n a multiple of 128, ldy and col0 multiples of 8, destinations
 * 16-byte aligned. The caller orders the ranks (a barrier after the calls)
 * before reading a destination.
 * No counterpart in the reference, which has no multi-GPU linear; it replaces
 * the compute-then-all-gather pair of the column-sharded configuration. */
CF_API int cf_lora_linear_int8_allgather(const void *x, const int8_t *w_codes,
                                         const float *w_scales, const void *a, int a_layout,
                                         const void *b, int b_layout, int n_dest,
                                         void *const *y_dest, int self_dest, int64_t ldy,
                                         int64_t col0,
                                         int64_t m, int64_t k, int64_t n, int64_t rank,
                                         float scale, int dtype, void *workspace,
                                         size_t workspace_bytes, cf_stream_t stream);

/* cf_lora_linear_int8_allgather with the exchange done by NVLink SHARP
 * multicast (no counterpart in the reference, which has no multi-GPU path for
 * this op; it stands in for the NCCL all-gather of the column-sharded linear).
 * y_multicast is the multicast address of a [m, ldy] buffer that every rank
 * has bound to one multicast object (y_local is this GPU's own copy of it):
 * each 16-byte piece of this call's columns [col0, col0 + n) is written once
 * with a multimem store, and the switch delivers it to every rank's copy, so
 * each rank sends its slice over NVLink once instead of once per peer. The
 * caller orders the ranks afterwards (a barrier) before reading y. Same
 * shape rules as cf_lora_linear_int8_allgather (n a multiple of 128, ldy and
 * col0 multiples of 8). */
CF_API int cf_lora_linear_int8_allgather_mc(const void *x, const int8_t *w_codes,
                                            const float *w_scales, const void *a, int a_layout,
                                            const void *b, int b_layout, void *y_local,
                                            void *y_multicast, int64_t ldy, int64_t col0,
                                            int64_t m, int64_t k, int64_t n, int64_t rank,
                                            float scale, int dtype, void *workspace,
                                            size_t workspace_bytes, cf_stream_t stream);

/* Workspace bytes of cf_lora_linear_int8_allgather_ce: the down-projection
 * workspace of cf_lora_linear_workspace_bytes plus 256 bytes of row-group
 * counters. */
CF_API size_t cf_lora_linear_int8_allgather_ce_workspace_bytes(int64_t m, int64_t rank);

/* Column-sharded W8 linear with the output all-gather on the copy engines.
 * Same product, destinations and argument rules as
 * cf_lora_linear_int8_allgather, plus self_dest, the index in y_dest of this
 * GPU's own destination. The kernel writes only y_dest[self_dest] and counts
 * finished tiles per row group (up to 16 groups of 512-row blocks); one copy
 * stream per other destination waits on each group's count (a stream
 * wait-value operation) and copies that group's [rows, n] block into its
 * destination while later groups are still being computed. The copies join
 * `stream` before the call returns its work, so later work on `stream` sees
 * every destination written. Calls on one device serialise their enqueueing.
 * No counterpart in the reference (see cf_lora_linear_int8_allgather). */
CF_API int cf_lora_linear_int8_allgather_ce(const void *x, const int8_t *w_codes,
                                            const float *w_scales, const void *a, int a_layout,
                                            const void *b, int b_layout, int n_dest,
                                            void *const *y_dest, int self_dest, int64_t ldy,
                                            int64_t col0, int64_t m, int64_t k, int64_t n,
                                            int64_t rank, float scale, int dtype,
                                            void *workspace, size_t workspace_bytes,
                                            cf_stream_t stream);

/* LoRA merge + block-INT8 quantisation in one pass:
 *   codes, scales = quantize_int8(w + scaling * (lora_b @ lora_a))
 * with the module layouts of training/lora.py:95-102 (w [n, k] = [out, in],
 * lora_a [rank, k], lora_b [n, rank]), all contiguous and of `dtype` (f16 or
 * bf16). The merged value is rounded as the module computes it in its dtype
 * (product, times scaling, plus w, each rounded to the dtype) and quantised
 * with the reference's arithmetic; the merged weight itself is never stored.
 * codes int8 [n, k], scales float [n * k / 64]. Requirements: k % 64 == 0,
 * rank in {16, 32, 64} (smaller ranks zero-padded by the caller), pointers
 * 16-byte aligned (scales 4). No counterpart launcher in the reference: it
 * replaces merged_weight() followed by quantize_int8 (training/lora.py:95-111,
 * cpp/src/bindings.cpp:198-209). */
CF_API int cf_lora_merge_quantize_int8(const void *w, const void *lora_a, const void *lora_b,
                                       int64_t n, int64_t k, int64_t rank, float scaling,
                                       int dtype, int8_t *codes, float *scales,
                                       cf_stream_t stream);

/* The gate and up projections of a LLaMA MLP with SwiGLU fused:
 *   y[m, n] = silu(g) * u,  g = x gate_W^T,  u = x up_W^T
 * with block-INT8 weights (gate_codes / up_codes int8 [n, k], scales float
 * [n * k / 64], as cf_quantize_int8 produces them from nn.Linear weights) and
 * x, y of `dtype` (f16 or bf16). g and u are rounded to `dtype` as the two
 * projections' outputs would be, silu(v) = v / (1 + exp(-v)) and the product
 * are computed in fp32 and rounded once; only y is written. Replaces
 * gate(x), up(x), swiglu(gate, up) of the reference's transformer block
 * (examples/transformer_block.py:84-87; swiglu: cuda/src/activations.cu:68-76,
 * python/cudaforge/ops.py:407-440). Requirements: k % 64 == 0, n % 8 == 0,
 * pointers 16-byte aligned (scales 4). */
CF_API int cf_w8_swiglu_int8(const void *x, const int8_t *gate_codes, const float *gate_scales,
                             const int8_t *up_codes, const float *up_scales, void *y, int64_t m,
                             int64_t k, int64_t n, int dtype, cf_stream_t stream);

/* Residual add + RMSNorm over rows of length cols (rows x cols, contiguous):
 *   residual_out = x + residual                 (rounded to dtype)
 *   output = residual_out * rsqrt(mean(residual_out^2) + eps) * weight
 * (fp32 arithmetic, rounded once to dtype). Replaces the reference's
 * fused_residual_rmsnorm (cpp/src/bindings.cpp:129-151,
 * cuda/include/cudaforge/fused_norm.cuh; semantics python/cudaforge/ops.py:
 * 164-171, 188-192), which runs fp32 only; here dtype is f32, bf16 or f16 and
 * weight [cols] is of dtype or f32 (weight_dtype). residual and residual_out
 * both NULL give the reference's rmsnorm (cpp/src/bindings.cpp:65-80): output =
 * x * rsqrt(mean(x^2) + eps) * weight. output may alias x and residual_out may
 * alias residual. Any alignment works; 16-byte aligned pointers and rows of a
 * whole number of 16-byte chunks take the vector path. */
CF_API int cf_fused_residual_rmsnorm(const void *x, const void *residual, const void *weight,
                                     int weight_dtype, void *output, void *residual_out,
                                     int64_t rows, int64_t cols, float eps, int dtype,
                                     cf_stream_t stream);

/* Allocation-free form of cf_lora_linear, for callers that cannot allocate the
 * workspace: hosts whose device memory is reserved up front by another
 * allocator, foreign-language hosts without a CUDA allocator, and loops that
 * must not pay cudaMalloc's device synchronisation. No counterpart in the
 * reference. The workspace is a 4 MiB device array inside the library, held by
 * every GPU that loads it until exit: m * rank * 2 bytes for bf16/f16 calls
 * (m <= 131072 at rank 16) or m * rank * 4 bytes for fp32 calls (m <= 65536 at
 * rank 16), rounded up to 256, must fit, else CF_ERR_WORKSPACE and nothing is
 * launched. Calls on one device
 * share the array; calls that overlap on the GPU race on it. The first call on
 * a device looks up the array's address (make it before any stream capture).
 * Same arguments and semantics as cf_lora_linear otherwise. */
CF_API int cf_lora_linear_noalloc(const void *x, const void *w, int w_layout, const void *a,
                                  int a_layout, const void *b, int b_layout, void *y, int64_t m,
                                  int64_t k, int64_t n, int64_t rank, float scale, int dtype,
                                  cf_stream_t stream);

/* ---- status -------------------------------------------------------------- */

/* Human-readable text for a cf_status value. */
CF_API const char *cf_status_string(int status);

/* The cudaError_t of the most recent CF_ERR_CUDA returned on this thread. */
CF_API int cf_last_cuda_error(void);

/* Reads and clears the device-side error word of the current device (set by a
 * kernel whose bounded wait gave up). Synchronises with the device. Returns
 * CF_OK or CF_ERR_DEVICE_TIMEOUT (CF_ERR_CUDA if the read itself fails). */
CF_API int cf_device_status(void);

/* Test hook for the bounded-wait path (no counterpart in the reference; its
 * closest is the sticky / non-sticky split of CudaError::is_sticky,
 * cuda/include/cudaforge/cuda_error.cuh:15-41). Launches one warp that waits
 * on a barrier nothing arrives on, with the bounded wait every kernel here
 * uses, limited to limit_ns (1 ms .. 2 s, else CF_ERR_INVALID_ARGUMENT). The
 * wait runs out, the kernel records CF_ERR_DEVICE_TIMEOUT in the device error
 * word and returns: nothing faults, and the context stays usable. */
CF_API int cf_debug_expire_wait(uint64_t limit_ns, cf_stream_t stream);

/* Build information: "sm_100a" architecture tag and version string. */
CF_API const char *cf_build_info(void);

#ifdef __cplusplus
}
#endif

#endif /* CUDAFORGE_B200_H_ */
