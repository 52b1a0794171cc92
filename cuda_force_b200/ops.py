"""Operator API of the quantised-linear hot path, mirroring ``cudaforge.ops``.

Same function names, argument meaning and ``ValueError`` messages as the
reference wrapper (python/cudaforge/ops.py: ``QUANT_BLOCK_SIZE`` :41,
``lora_linear`` :289-332, ``quantize_int8`` :449-460, ``dequantize_int8``
:463-476, ``quantization_error`` :479-488, ``backend_report`` :109-122), with
three differences that are deliberate:

* there is no host fallback. The reference drops to an ATen composition when
  the extension is absent, the tensor is on the CPU, the dtype is not float32,
  or autograd is needed. Here every call runs the sm_100a kernels through
  ``torch.ops.cudaforge``; a CPU tensor, a missing extension or a
  grad-requiring input raises instead of silently changing implementation;
* bfloat16 and float16 reach the kernels as well as float32 (the reference
  gates its CUDA path on float32, ops.py:329 and :457); float32 linears run
  on the tensor cores as three tf32 products (hi*hi + hi*lo + lo*hi), which
  keeps fp32 accuracy;
* ``lora_linear`` accepts ``weight``/``lora_a``/``lora_b`` either contiguous in
  the reference's layout or as the transpose of a contiguous tensor (the
  nn.Linear / ``training/lora.py`` storage), without copying.

``rmsnorm`` and ``fused_residual_rmsnorm`` (ops.py:248-275, :335-382) keep
the reference's names, arguments and messages and take all three dtypes.

Additive ops: ``lora_linear_int8`` (W as block-INT8 codes + scales),
``quantize_dequantize`` (fake quantisation) and ``quantize_int8_many``.
"""

from __future__ import annotations

from dataclasses import dataclass
from pathlib import Path

import torch

# Block size for int8 quantisation. Must match kQuantBlockSize in
# cuda_force_b200/csrc/cf_common.cuh and CF_QUANT_BLOCK_SIZE in
# include/cudaforge_b200.h.
QUANT_BLOCK_SIZE = 64

_SHIM = Path(__file__).resolve().parent / "_C.so"


def _load_extension() -> tuple[bool, str]:
    if not _SHIM.exists():
        return False, f"{_SHIM.name} not built; run `python -m cuda_force_b200._build`"
    try:
        torch.ops.load_library(str(_SHIM))
    except OSError as error:  # pragma: no cover - surfaced through backend_report
        return False, f"extension present but failed to load: {error}"
    return True, "extension loaded with sm_100a kernels"


_EXTENSION_LOADED, _LOAD_MESSAGE = _load_extension()

#: True when the extension is loaded and a CUDA device is visible.
CUDA_KERNELS_AVAILABLE: bool = _EXTENSION_LOADED and torch.cuda.is_available()

#: Storage dtypes with a kernel. Quantisation and lora_linear accept all
#: three; lora_linear_int8 takes float16 / bfloat16 activations.
KERNEL_DTYPES: frozenset[torch.dtype] = frozenset({torch.float32, torch.float16, torch.bfloat16})
LINEAR_DTYPES: frozenset[torch.dtype] = KERNEL_DTYPES
INT8_LINEAR_DTYPES: frozenset[torch.dtype] = frozenset({torch.float16, torch.bfloat16})


@dataclass(frozen=True)
class BackendReport:
    """Which implementation runs, and why."""

    extension_loaded: bool
    cuda_compiled: bool
    cuda_device_available: bool
    device_name: str | None
    message: str

    @property
    def using_custom_kernels(self) -> bool:
        return self.extension_loaded and self.cuda_compiled and self.cuda_device_available

    def __str__(self) -> str:
        path = "custom CUDA kernels" if self.using_custom_kernels else "no usable kernels"
        return f"cuda_force_b200: {path} on {self.device_name or 'no GPU'} ({self.message})"


def backend_report() -> BackendReport:
    available = torch.cuda.is_available()
    return BackendReport(
        extension_loaded=_EXTENSION_LOADED,
        cuda_compiled=_EXTENSION_LOADED,
        cuda_device_available=available,
        device_name=torch.cuda.get_device_name(0) if available else None,
        message=_LOAD_MESSAGE,
    )


def kernel_supports(dtype: torch.dtype) -> bool:
    return dtype in KERNEL_DTYPES


def _require(op: str, *tensors: torch.Tensor) -> None:
    if not _EXTENSION_LOADED:
        raise RuntimeError(f"{op}: {_LOAD_MESSAGE}")
    for t in tensors:
        if not t.is_cuda:
            raise RuntimeError(f"{op}: CUDA tensors required (this build has no CPU path)")
    if torch.is_grad_enabled() and any(t.requires_grad for t in tensors):
        raise RuntimeError(f"{op}: inference-only kernels; no backward is implemented")


def _as_stored(t: torch.Tensor) -> torch.Tensor:
    """Contiguous, or the transpose of a contiguous 2-D tensor; otherwise a copy."""
    if t.is_contiguous() or (t.dim() == 2 and t.t().is_contiguous()):
        return t
    return t.contiguous()


def quantize_int8(x: torch.Tensor) -> tuple[torch.Tensor, torch.Tensor]:
    """Block-wise symmetric int8 quantisation.

    Returns ``(quantised, scales)``: int8 codes shaped like ``x`` and float32
    scales, one per ``QUANT_BLOCK_SIZE`` elements of the flattened tensor.
    """
    _require("quantize_int8", x)
    quantised, scales = torch.ops.cudaforge.quantize_int8(x.contiguous())
    return quantised, scales


def dequantize_int8(quantised: torch.Tensor, scales: torch.Tensor) -> torch.Tensor:
    """Inverse of :func:`quantize_int8` (float32 output). Lossy by construction."""
    expected = (quantised.numel() + QUANT_BLOCK_SIZE - 1) // QUANT_BLOCK_SIZE
    if scales.numel() != expected:
        raise ValueError(
            f"expected {expected} block scales for {quantised.numel()} elements, "
            f"got {scales.numel()}"
        )
    _require("dequantize_int8", quantised, scales)
    return torch.ops.cudaforge.dequantize_int8(quantised.contiguous(), scales.contiguous())


def quantize_dequantize(x: torch.Tensor) -> torch.Tensor:
    """Fake quantisation: ``dequantize_int8(*quantize_int8(x))`` in one pass."""
    _require("quantize_dequantize", x)
    return torch.ops.cudaforge.quantize_dequantize(x.contiguous())


def quantize_int8_many(tensors: list[torch.Tensor]) -> list[tuple[torch.Tensor, torch.Tensor]]:
    """Quantise several tensors of one dtype in one launch."""
    if not tensors:
        return []
    _require("quantize_int8_many", *tensors)
    flat = torch.ops.cudaforge.quantize_int8_many([t.contiguous() for t in tensors])
    return [(flat[2 * i], flat[2 * i + 1]) for i in range(len(tensors))]


def rmsnorm(x: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6) -> torch.Tensor:
    """Root-mean-square normalisation over the last dimension.

    ``x * rsqrt(mean(x^2) + eps) * weight`` in fp32, rounded once to x's dtype
    (reference ops.py:164-171, :248-275). ``x`` is ``[..., hidden]``; ``weight``
    is ``[hidden]`` of any float dtype (read as float32, like the reference).
    """
    if weight.ndim != 1:
        raise ValueError(f"weight must be 1-D, got shape {tuple(weight.shape)}")
    if x.shape[-1] != weight.shape[0]:
        raise ValueError(
            f"weight length {weight.shape[0]} does not match the last dimension "
            f"of x, which is {x.shape[-1]}"
        )
    if x.numel() == 0:
        return x.clone()
    _require("rmsnorm", x, weight)
    rows = x.contiguous().view(-1, x.shape[-1])
    return torch.ops.cudaforge.rmsnorm(rows, weight.contiguous(), float(eps)).view(x.shape)


def fused_residual_rmsnorm(
    x: torch.Tensor, residual: torch.Tensor, weight: torch.Tensor, eps: float = 1e-6
) -> tuple[torch.Tensor, torch.Tensor]:
    """Residual add followed by RMSNorm, in one pass over the rows.

    Returns ``(normalised, residual_out)`` with ``residual_out = x + residual``
    rounded to x's dtype and ``normalised = rmsnorm(residual_out, weight, eps)``
    (reference ops.py:188-192, :335-382). ``x`` and ``residual`` share a shape
    ``[..., hidden]`` and dtype; ``weight`` is ``[hidden]``.
    """
    if x.shape != residual.shape:
        raise ValueError(
            f"x and residual must have the same shape, got {tuple(x.shape)} "
            f"and {tuple(residual.shape)}"
        )
    if weight.ndim != 1 or weight.shape[0] != x.shape[-1]:
        raise ValueError(f"weight must be 1-D of length {x.shape[-1]}, got {tuple(weight.shape)}")
    if x.numel() == 0:
        return x.clone(), residual.clone()
    _require("fused_residual_rmsnorm", x, residual, weight)
    hidden = x.shape[-1]
    normalised, summed = torch.ops.cudaforge.fused_residual_rmsnorm(
        x.contiguous().view(-1, hidden), residual.contiguous().view(-1, hidden),
        weight.contiguous(), float(eps))
    return normalised.view(x.shape), summed.view(x.shape)


def matmul_f32(a: torch.Tensor, b: torch.Tensor, precise: bool = True) -> torch.Tensor:
    """``a @ b`` for float32 ``a [m, k]`` and ``b [k, n]`` on the tensor cores.

    ``precise=True`` keeps fp32 accuracy with three tf32 products of a hi/lo
    split (the reference's ``launch_matmul``, lora_linear.cuh:58-59);
    ``precise=False`` is one tf32 product (its ``launch_matmul_tensor_core``,
    tensor_core_matmul.cuh:40-41). ``b`` may be the transpose of a contiguous
    ``[n, k]`` tensor. Feature counts that are not multiples of 4 are
    zero-padded.
    """
    import ctypes

    from cuda_force_b200 import _abi

    if a.dim() != 2 or b.dim() != 2 or a.shape[1] != b.shape[0]:
        raise ValueError(f"matmul_f32 needs a [m, k] and b [k, n], got {tuple(a.shape)} and "
                         f"{tuple(b.shape)}")
    if a.dtype != torch.float32 or b.dtype != torch.float32:
        raise ValueError("matmul_f32 takes float32 tensors")
    _require("matmul_f32", a, b)
    m, k = a.shape
    n = b.shape[1]
    kp, np_ = -(-k // 4) * 4, -(-n // 4) * 4
    a = a.contiguous()
    if kp != k:
        a = torch.nn.functional.pad(a, (0, kp - k))
    if kp != k or np_ != n:
        b = torch.nn.functional.pad(b, (0, np_ - n, 0, kp - k)).contiguous()
    b = _as_stored(b)
    layout = _abi.CF_LAYOUT_REF if b.is_contiguous() else _abi.CF_LAYOUT_T
    c = torch.empty(m, np_, dtype=torch.float32, device=a.device)
    stream = ctypes.c_void_p(torch.cuda.current_stream(a.device).cuda_stream)
    _abi.check(_abi.load().cf_matmul_f32(
        ctypes.c_void_p(a.data_ptr()), ctypes.c_void_p(b.data_ptr()), layout,
        ctypes.c_void_p(c.data_ptr()), m, np_, kp, 1 if precise else 0, stream), "cf_matmul_f32")
    return c if np_ == n else c[:, :n].contiguous()


def lora_merge_quantize_int8(
    weight: torch.Tensor, lora_a: torch.Tensor, lora_b: torch.Tensor, scaling: float
) -> tuple[torch.Tensor, torch.Tensor]:
    """``quantize_int8(weight + scaling * (lora_b @ lora_a))`` in one pass.

    The deployment step after LoRA training (training/lora.py:95-111: merge,
    then quantise the merged weight for a W8 linear) without materialising the
    merged weight. Module layouts: ``weight [out, in]``, ``lora_a [rank, in]``,
    ``lora_b [out, rank]``, all float16 or bfloat16; ``in`` a multiple of 64.
    Each merged value is rounded as the module computes it in its dtype.
    Returns ``(codes [out, in] int8, scales [out * in / 64] float32)``.
    """
    import ctypes

    from cuda_force_b200 import _abi

    if weight.dim() != 2:
        raise ValueError(f"weight must be [out_features, in_features], got {tuple(weight.shape)}")
    out_features, in_features = weight.shape
    if lora_a.dim() != 2 or lora_a.shape[1] != in_features:
        raise ValueError(f"lora_a must be [rank, in_features={in_features}], got "
                         f"{tuple(lora_a.shape)}")
    rank = lora_a.shape[0]
    if lora_b.dim() != 2 or tuple(lora_b.shape) != (out_features, rank):
        raise ValueError(f"lora_b must be [out_features, rank] = [{out_features}, {rank}], got "
                         f"{tuple(lora_b.shape)}")
    if weight.dtype not in (torch.float16, torch.bfloat16) or lora_a.dtype != weight.dtype \
            or lora_b.dtype != weight.dtype:
        raise ValueError("lora_merge_quantize_int8 takes float16 or bfloat16 tensors of one dtype")
    if in_features % QUANT_BLOCK_SIZE:
        raise ValueError(f"in_features must be a multiple of {QUANT_BLOCK_SIZE}, got {in_features}")
    if not 1 <= rank <= 64:
        raise ValueError(f"rank must be between 1 and 64, got {rank}")
    _require("lora_merge_quantize_int8", weight, lora_a, lora_b)
    padded = 16 if rank <= 16 else 32 if rank <= 32 else 64
    a = lora_a.contiguous()
    b = lora_b.contiguous()
    if padded != rank:
        a = torch.nn.functional.pad(a, (0, 0, 0, padded - rank))
        b = torch.nn.functional.pad(b, (0, padded - rank))
    w = weight.contiguous()
    codes = torch.empty(out_features, in_features, dtype=torch.int8, device=w.device)
    scales = torch.empty(out_features * in_features // QUANT_BLOCK_SIZE, dtype=torch.float32,
                         device=w.device)
    dtype = _abi.CF_DTYPE_BF16 if w.dtype == torch.bfloat16 else _abi.CF_DTYPE_F16
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream(w.device).cuda_stream)
    _abi.check(_abi.load().cf_lora_merge_quantize_int8(
        p(w), p(a), p(b), out_features, in_features, padded, float(scaling), dtype, p(codes),
        p(scales), stream), "cf_lora_merge_quantize_int8")
    return codes, scales


def w8_swiglu_int8(
    x: torch.Tensor,
    gate_codes: torch.Tensor,
    gate_scales: torch.Tensor,
    up_codes: torch.Tensor,
    up_scales: torch.Tensor,
) -> torch.Tensor:
    """``swiglu(x @ Wg.T, x @ Wu.T)`` for block-INT8 gate and up weights, in one kernel.

    ``gate_codes`` / ``up_codes`` are int8 ``[intermediate, hidden]`` (what
    :func:`quantize_int8` returns for the nn.Linear weights) with their 1-D
    float32 scales; ``x [..., hidden]`` is float16 or bfloat16. Matches
    ``swiglu(gate(x), up(x))`` of the reference's transformer block
    (examples/transformer_block.py:84-87) with the projections rounded to
    x's dtype; only the activated ``[..., intermediate]`` output is written.
    """
    import ctypes

    from cuda_force_b200 import _abi

    if gate_codes.dim() != 2 or up_codes.shape != gate_codes.shape:
        raise ValueError("gate_codes and up_codes must both be [intermediate, hidden], got "
                         f"{tuple(gate_codes.shape)} and {tuple(up_codes.shape)}")
    n, k = gate_codes.shape
    if x.shape[-1] != k:
        raise ValueError(f"x has {x.shape[-1]} input features but the weights expect {k}")
    expected = n * k // QUANT_BLOCK_SIZE
    if k % QUANT_BLOCK_SIZE or gate_scales.numel() != expected or up_scales.numel() != expected:
        raise ValueError(f"expected {expected} block scales per weight and hidden a multiple of "
                         f"{QUANT_BLOCK_SIZE}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("w8_swiglu_int8 takes float16 or bfloat16 activations")
    _require("w8_swiglu_int8", x, gate_codes, gate_scales, up_codes, up_scales)
    x2, lead = _flatten_tokens(x)
    m = x2.shape[0]
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    dtype = _abi.CF_DTYPE_BF16 if x.dtype == torch.bfloat16 else _abi.CF_DTYPE_F16
    p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
    gc, uc = gate_codes.contiguous(), up_codes.contiguous()
    gs, us = gate_scales.contiguous().reshape(-1), up_scales.contiguous().reshape(-1)
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _abi.check(_abi.load().cf_w8_swiglu_int8(p(x2), p(gc), p(gs), p(uc), p(us), p(y), m, k, n,
                                             dtype, stream), "cf_w8_swiglu_int8")
    return y.reshape(*lead, n)


def rmsnorm_lora_linear_int8(
    x: torch.Tensor,
    residual: torch.Tensor | None,
    norm_weight: torch.Tensor,
    w_codes: torch.Tensor,
    w_scales: torch.Tensor,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scale: float = 1.0,
    eps: float = 1e-6,
) -> tuple[torch.Tensor, torch.Tensor | None]:
    """``y = lora_linear_int8(rmsnorm(h, norm_weight, eps), ...)`` with ``h = x + residual``.

    The reference's ``fused_residual_rmsnorm`` (ops.py:335-382) followed by the
    W8 linear, as a LLaMA block chains them (examples/transformer_block.py:
    84-87), with the normalisation folded into the linear: the normalised
    activations are never written. Returns ``(y, residual_out)``
    (``residual_out`` is None without a residual). float16 / bfloat16 only;
    ``norm_weight`` in x's dtype.
    """
    import ctypes

    from cuda_force_b200 import _abi

    if w_codes.dim() != 2:
        raise ValueError(f"w_codes must be [out_features, in_features], got {tuple(w_codes.shape)}")
    n, k = w_codes.shape
    _check_lora_shapes(x, k, n, lora_a, lora_b)
    if norm_weight.numel() != k:
        raise ValueError(f"norm_weight must have {k} elements, got {norm_weight.numel()}")
    if residual is not None and residual.shape != x.shape:
        raise ValueError(f"x and residual must have the same shape, got {tuple(x.shape)} and "
                         f"{tuple(residual.shape)}")
    if x.dtype not in (torch.float16, torch.bfloat16):
        raise ValueError("rmsnorm_lora_linear_int8 takes float16 or bfloat16 activations")
    expected = n * k // QUANT_BLOCK_SIZE
    if k % QUANT_BLOCK_SIZE or w_scales.numel() != expected:
        raise ValueError(f"expected {expected} block scales for {w_codes.numel()} elements")
    tensors = [x, norm_weight, w_codes, w_scales, lora_a, lora_b]
    _require("rmsnorm_lora_linear_int8", *tensors, *([residual] if residual is not None else []))
    x2, lead = _flatten_tokens(x)
    m = x2.shape[0]
    r = lora_a.shape[1]
    rp = 16 if r <= 16 else 32 if r <= 32 else 64
    if r > 64:
        raise ValueError(f"adapter rank {r} above 64 is not supported")
    a, b = lora_a.to(x.dtype), lora_b.to(x.dtype)
    if rp != r:  # zero rank padding leaves the product unchanged
        a = torch.nn.functional.pad(a, (0, rp - r))
        b = torch.nn.functional.pad(b, (0, 0, 0, rp - r))
    a, b = a.contiguous(), b.contiguous()
    res2 = residual.reshape(m, k).contiguous() if residual is not None else None
    res_out = torch.empty_like(x2) if residual is not None else None
    y = torch.empty(m, n, dtype=x.dtype, device=x.device)
    lib = _abi.load()
    ws = torch.empty(lib.cf_rmsnorm_lora_linear_int8_workspace_bytes(m, k, rp), dtype=torch.uint8,
                     device=x.device)
    dtype = _abi.CF_DTYPE_BF16 if x.dtype == torch.bfloat16 else _abi.CF_DTYPE_F16
    p = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None  # noqa: E731
    stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
    _abi.check(lib.cf_rmsnorm_lora_linear_int8(
        p(x2), p(res2), p(norm_weight.to(x.dtype).contiguous()), float(eps), p(w_codes.contiguous()),
        p(w_scales.contiguous().reshape(-1)), p(a), _abi.CF_LAYOUT_REF, p(b), _abi.CF_LAYOUT_REF,
        p(y), p(res_out), m, k, n, rp, float(scale), dtype, p(ws), ws.numel(), stream),
        "cf_rmsnorm_lora_linear_int8")
    return (y.reshape(*lead, n),
            res_out.reshape(x.shape) if res_out is not None else None)


def quantization_error(x: torch.Tensor) -> torch.Tensor:
    """Maximum absolute round-trip error of int8 quantisation (<= scale / 2 per block)."""
    quantised, scales = quantize_int8(x)
    restored = dequantize_int8(quantised, scales)
    return (x.float() - restored).abs().max()


def _check_lora_shapes(
    x: torch.Tensor, in_features: int, out_features: int, lora_a: torch.Tensor, lora_b: torch.Tensor
) -> None:
    if x.shape[-1] != in_features:
        raise ValueError(f"x has {x.shape[-1]} input features but weight expects {in_features}")
    if lora_a.shape[0] != in_features:
        raise ValueError(
            f"lora_a must be [in_features, rank] with in_features={in_features}, "
            f"got {tuple(lora_a.shape)}"
        )
    if lora_b.shape[0] != lora_a.shape[1] or lora_b.shape[1] != out_features:
        raise ValueError(
            f"lora_b must be [rank, out_features] = "
            f"[{lora_a.shape[1]}, {out_features}], got {tuple(lora_b.shape)}"
        )


def _flatten_tokens(x: torch.Tensor) -> tuple[torch.Tensor, tuple[int, ...]]:
    lead = tuple(x.shape[:-1])
    return x.reshape(-1, x.shape[-1]).contiguous(), lead


def lora_linear(
    x: torch.Tensor,
    weight: torch.Tensor,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scale: float = 1.0,
) -> torch.Tensor:
    """LoRA-adapted linear layer: ``x @ weight + scale * (x @ lora_a) @ lora_b``.

    Args:
        x: ``[..., in_features]`` (float32, bfloat16 or float16).
        weight: ``[in_features, out_features]`` — contiguous, or ``W.t()`` of an
            nn.Linear weight ``W [out_features, in_features]``.
        lora_a: ``[in_features, rank]`` (or the transpose of ``[rank, in_features]``).
        lora_b: ``[rank, out_features]`` (or the transpose of ``[out_features, rank]``).
        scale: usually ``alpha / rank``.
    """
    _check_lora_shapes(x, weight.shape[0], weight.shape[1], lora_a, lora_b)
    _require("lora_linear", x, weight, lora_a, lora_b)
    x2, lead = _flatten_tokens(x)
    y = torch.ops.cudaforge.lora_linear(
        x2, _as_stored(weight), _as_stored(lora_a), _as_stored(lora_b), float(scale)
    )
    return y.reshape(*lead, y.shape[-1])


def lora_linear_int8(
    x: torch.Tensor,
    w_codes: torch.Tensor,
    w_scales: torch.Tensor,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scale: float = 1.0,
) -> torch.Tensor:
    """``lora_linear(x, dequantize_int8(w_codes, w_scales).T, lora_a, lora_b, scale)``.

    Args:
        w_codes: int8 ``[out_features, in_features]``, the codes
            :func:`quantize_int8` returns for an nn.Linear weight.
        w_scales: float32 block scales of ``w_codes`` (1-D).
    """
    if w_codes.dim() != 2:
        raise ValueError(f"w_codes must be [out_features, in_features], got {tuple(w_codes.shape)}")
    out_features, in_features = w_codes.shape
    _check_lora_shapes(x, in_features, out_features, lora_a, lora_b)
    expected = (w_codes.numel() + QUANT_BLOCK_SIZE - 1) // QUANT_BLOCK_SIZE
    if w_scales.numel() != expected:
        raise ValueError(
            f"expected {expected} block scales for {w_codes.numel()} elements, "
            f"got {w_scales.numel()}"
        )
    _require("lora_linear_int8", x, w_codes, w_scales, lora_a, lora_b)
    x2, lead = _flatten_tokens(x)
    y = torch.ops.cudaforge.lora_linear_int8(
        x2, w_codes.contiguous(), w_scales.contiguous().reshape(-1), _as_stored(lora_a),
        _as_stored(lora_b), float(scale)
    )
    return y.reshape(*lead, y.shape[-1])
