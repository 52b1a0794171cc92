"""B200-native (sm_100a) quantised-linear hot path with the operator API of
CudaForge's ``cudaforge.ops``: block-INT8 quantise / dequantise and the LoRA
linear (bf16/fp16 or block-INT8 weight)."""

from __future__ import annotations

from cuda_force_b200.ops import (
    CUDA_KERNELS_AVAILABLE,
    KERNEL_DTYPES,
    QUANT_BLOCK_SIZE,
    backend_report,
    dequantize_int8,
    fused_residual_rmsnorm,
    kernel_supports,
    lora_linear,
    lora_linear_int8,
    lora_merge_quantize_int8,
    matmul_f32,
    quantization_error,
    quantize_dequantize,
    quantize_int8,
    quantize_int8_many,
    rmsnorm,
    rmsnorm_lora_linear_int8,
    w8_swiglu_int8,
)

__version__ = "0.1.0"

__all__ = [
    "CUDA_KERNELS_AVAILABLE",
    "KERNEL_DTYPES",
    "QUANT_BLOCK_SIZE",
    "__version__",
    "backend_report",
    "dequantize_int8",
    "fused_residual_rmsnorm",
    "kernel_supports",
    "lora_linear",
    "lora_linear_int8",
    "lora_merge_quantize_int8",
    "matmul_f32",
    "quantization_error",
    "quantize_dequantize",
    "quantize_int8",
    "quantize_int8_many",
    "rmsnorm",
    "rmsnorm_lora_linear_int8",
    "w8_swiglu_int8",
]
