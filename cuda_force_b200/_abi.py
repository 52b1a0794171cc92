"""ctypes binding of the C ABI in ``include/cudaforge_b200.h``.

This is the binding a non-PyTorch host (or a test) uses: raw device pointers,
int64 sizes and a ``cudaStream_t`` as an integer. It loads the in-tree
``libcudaforge_b200.so`` and declares every exported entry point's signature.
"""

from __future__ import annotations

import ctypes
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libcudaforge_b200.so"

CF_OK = 0
CF_ERR_INVALID_ARGUMENT = 1
CF_ERR_UNSUPPORTED = 2
CF_ERR_MISALIGNED = 3
CF_ERR_CUDA = 4
CF_ERR_DEVICE_TIMEOUT = 5
CF_ERR_WORKSPACE = 6
CF_ERR_NO_DEVICE = 7

CF_DTYPE_F32 = 0
CF_DTYPE_F16 = 1
CF_DTYPE_BF16 = 2

CF_LAYOUT_REF = 0
CF_LAYOUT_T = 1

CF_MAX_SEGMENTS = 256

_p = ctypes.c_void_p
_i64 = ctypes.c_int64
_int = ctypes.c_int


class QuantSegment(ctypes.Structure):
    _fields_ = [("input", _p), ("codes", _p), ("scales", _p), ("count", _i64)]


# name -> (restype, argtypes); the complete exported surface of the header.
SIGNATURES: dict[str, tuple[object, list[object]]] = {
    "cf_quant_scale_count": (_i64, [_i64]),
    "cf_quantize_int8": (_int, [_p, _int, _p, _p, _i64, _p]),
    "cf_dequantize_int8": (_int, [_p, _p, _p, _i64, _p]),
    "cf_quantize_dequantize": (_int, [_p, _int, _p, _i64, _p]),
    "cf_quantize_int8_many": (_int, [ctypes.POINTER(QuantSegment), _int, _int, _p]),
    "cf_lora_linear_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "cf_lora_linear": (
        _int,
        [_p, _p, _int, _p, _int, _p, _int, _p, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _p,
         ctypes.c_size_t, _p],
    ),
    "cf_lora_linear_int8": (
        _int,
        [_p, _p, _p, _p, _int, _p, _int, _p, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _p,
         ctypes.c_size_t, _p],
    ),
    "cf_lora_linear_int8_allgather": (
        _int,
        [_p, _p, _p, _p, _int, _p, _int, _int, ctypes.POINTER(_p), _int, _i64, _i64, _i64, _i64,
         _i64, _i64, ctypes.c_float, _int, _p, ctypes.c_size_t, _p],
    ),
    "cf_lora_linear_int8_allgather_mc": (
        _int,
        [_p, _p, _p, _p, _int, _p, _int, _p, _p, _i64, _i64, _i64, _i64, _i64, _i64,
         ctypes.c_float, _int, _p, ctypes.c_size_t, _p],
    ),
    "cf_lora_linear_int8_allgather_ce_workspace_bytes": (ctypes.c_size_t, [_i64, _i64]),
    "cf_lora_linear_int8_allgather_ce": (
        _int,
        [_p, _p, _p, _p, _int, _p, _int, _int, ctypes.POINTER(_p), _int, _i64, _i64, _i64, _i64,
         _i64, _i64, ctypes.c_float, _int, _p, ctypes.c_size_t, _p],
    ),
    "cf_matmul_f32": (_int, [_p, _p, _int, _p, _i64, _i64, _i64, _int, _p]),
    "cf_w8_swiglu_int8": (_int, [_p, _p, _p, _p, _p, _p, _i64, _i64, _i64, _int, _p]),
    "cf_fused_residual_rmsnorm": (
        _int, [_p, _p, _p, _int, _p, _p, _i64, _i64, ctypes.c_float, _int, _p]),
    "cf_lora_merge_quantize_int8": (
        _int, [_p, _p, _p, _i64, _i64, _i64, ctypes.c_float, _int, _p, _p, _p]),
    "cf_rmsnorm_lora_linear_int8_workspace_bytes": (ctypes.c_size_t, [_i64, _i64, _i64]),
    "cf_rmsnorm_lora_linear_int8": (
        _int,
        [_p, _p, _p, ctypes.c_float, _p, _p, _p, _int, _p, _int, _p, _p, _i64, _i64, _i64, _i64,
         ctypes.c_float, _int, _p, ctypes.c_size_t, _p],
    ),
    "cf_lora_linear_noalloc": (
        _int,
        [_p, _p, _int, _p, _int, _p, _int, _p, _i64, _i64, _i64, _i64, ctypes.c_float, _int, _p],
    ),
    "cf_status_string": (ctypes.c_char_p, [_int]),
    "cf_last_cuda_error": (_int, []),
    "cf_device_status": (_int, []),
    "cf_debug_expire_wait": (_int, [ctypes.c_uint64, ctypes.c_void_p]),
    "cf_build_info": (ctypes.c_char_p, []),
}

_LIB: ctypes.CDLL | None = None


def load() -> ctypes.CDLL:
    """Load the library (once) and attach the signatures. Raises if it is missing."""
    global _LIB
    if _LIB is not None:
        return _LIB
    if not LIB_PATH.exists():
        raise ImportError(
            f"{LIB_PATH.name} is not built; run `python -m cuda_force_b200._build` "
            "(or __graft_entry__.build())"
        )
    lib = ctypes.CDLL(str(LIB_PATH))
    for name, (restype, argtypes) in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.restype = restype
        fn.argtypes = argtypes
    _LIB = lib
    return lib


class CfError(RuntimeError):
    """A non-zero cf_status from the C ABI."""

    def __init__(self, status: int, where: str):
        lib = load()
        text = lib.cf_status_string(status).decode()
        extra = f" (cudaError {lib.cf_last_cuda_error()})" if status == CF_ERR_CUDA else ""
        super().__init__(f"{where}: {text}{extra}")
        self.status = status


def check(status: int, where: str) -> None:
    if status != CF_OK:
        raise CfError(status, where)
