"""numpy restatement of the reference's block-INT8 quantisation.

TEST INFRASTRUCTURE ONLY (see oracle/__init__.py).

Follows python/cudaforge/ops.py:215-240 (``_quantize_int8_reference``,
``_dequantize_int8_reference``) and cpp/src/bindings.cpp:298-329, which compute:

    flat   = x.reshape(-1).float()                      (bf16/fp16 upcast exactly)
    padded = zero-pad flat to a multiple of 64, view [-1, 64]
    scale  = amax(|block|) / 127.0     (fp32 IEEE division; NaN propagates)
    scale  = where(scale > 0, scale, 1)
    codes  = clamp(round_half_even(block / scale), -127, 127).to(int8)
    deq    = codes.float() * scale     (fp32 multiply)

numpy float32 arithmetic is IEEE round-to-nearest, ``np.rint`` rounds half to
even, and NaN codes convert to 0 (matching the reference's observed behaviour,
pinned by tests/golden).
"""

from __future__ import annotations

import numpy as np

BLOCK = 64


def _as_f32(x: np.ndarray) -> np.ndarray:
    x = np.asarray(x)
    if x.dtype == np.float32:
        return x.reshape(-1)
    if x.dtype == np.float16:
        return x.reshape(-1).astype(np.float32)
    if x.dtype == np.uint16:  # bfloat16 bit patterns
        return (x.reshape(-1).astype(np.uint32) << 16).view(np.float32)
    raise TypeError(f"unsupported dtype {x.dtype}")


def scale_count(count: int) -> int:
    return 0 if count <= 0 else (count + BLOCK - 1) // BLOCK


def quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Returns (codes int8 [count], scales float32 [ceil(count/64)]).

    ``x`` is float32, float16, or uint16 holding bfloat16 bit patterns.
    """
    flat = _as_f32(x)
    count = flat.size
    nblocks = scale_count(count)
    padded = np.zeros(nblocks * BLOCK, dtype=np.float32)
    padded[:count] = flat
    grouped = padded.reshape(nblocks, BLOCK)
    with np.errstate(invalid="ignore", divide="ignore", over="ignore"):
        absmax = np.abs(grouped).max(axis=1)  # NaN propagates, like torch.amax
        scales = (absmax / np.float32(127.0)).astype(np.float32)
        scales = np.where(scales > 0, scales, np.float32(1.0)).astype(np.float32)
        q = np.rint(grouped / scales[:, None]).astype(np.float32)
        q = np.clip(q, -127, 127)
    q = np.where(np.isnan(q), np.float32(0), q)
    codes = q.reshape(-1)[:count].astype(np.int8)
    return codes, scales


def dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    codes = np.asarray(codes).reshape(-1)
    count = codes.size
    block_of = np.arange(count) // BLOCK
    return (codes.astype(np.float32) * np.asarray(scales, dtype=np.float32)[block_of]).astype(
        np.float32
    )


def quantize_dequantize(x: np.ndarray) -> np.ndarray:
    codes, scales = quantize(x)
    return dequantize(codes, scales)


# ---------------------------------------------------------------------------
# The C restatement (oracle/quant_ref.c), loaded through ctypes.
# ---------------------------------------------------------------------------
_C_LIB = None


def c_library():
    """Loads oracle/_build/liboracle_quant.so, building it with make if needed."""
    global _C_LIB
    if _C_LIB is not None:
        return _C_LIB
    import ctypes
    import subprocess
    from pathlib import Path

    here = Path(__file__).resolve().parent
    so = here / "_build" / "liboracle_quant.so"
    if not so.exists():
        subprocess.run(["make", "-s", "-C", str(here)], check=True)
    lib = ctypes.CDLL(str(so))
    p, i64, i = ctypes.c_void_p, ctypes.c_int64, ctypes.c_int
    lib.oracle_quantize.argtypes = [p, i, p, p, i64]
    lib.oracle_quantize.restype = None
    lib.oracle_dequantize.argtypes = [p, p, p, i64]
    lib.oracle_dequantize.restype = None
    _C_LIB = lib
    return lib


_DTYPE_CODE = {np.dtype(np.float32): 0, np.dtype(np.float16): 1, np.dtype(np.uint16): 2}


def c_quantize(x: np.ndarray) -> tuple[np.ndarray, np.ndarray]:
    """Same contract as quantize(), computed by the C restatement."""
    lib = c_library()
    x = np.ascontiguousarray(x).reshape(-1)
    count = x.size
    codes = np.empty(count, dtype=np.int8)
    scales = np.empty(scale_count(count), dtype=np.float32)
    lib.oracle_quantize(x.ctypes.data, _DTYPE_CODE[x.dtype], codes.ctypes.data,
                        scales.ctypes.data, count)
    return codes, scales


def c_dequantize(codes: np.ndarray, scales: np.ndarray) -> np.ndarray:
    lib = c_library()
    codes = np.ascontiguousarray(codes, dtype=np.int8).reshape(-1)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    out = np.empty(codes.size, dtype=np.float32)
    lib.oracle_dequantize(codes.ctypes.data, scales.ctypes.data, out.ctypes.data, codes.size)
    return out
