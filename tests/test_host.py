"""Host-side checks that need no GPU: the C-ABI library loads and exports every
symbol the header declares, argument validation, constants, and the Python
wrapper's error behaviour (mirroring the reference's tests/python/test_ops.py
ValueError cases)."""

from __future__ import annotations

import ctypes
import re
from pathlib import Path

import numpy as np
import pytest
import torch

import cuda_force_b200 as cf
from cuda_force_b200 import _abi
from cuda_force_b200 import ops
from tests.helpers import golden_cases, norm_cases, numpy_to_torch

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "cudaforge_b200.h"


def declared_functions() -> list[str]:
    text = HEADER.read_text()
    return re.findall(r"^CF_API\s+[\w\s\*]+?\b(cf_\w+)\(", text, flags=re.M)


def test_header_declares_the_abi():
    names = declared_functions()
    assert "cf_quantize_int8" in names and "cf_lora_linear_int8" in names
    assert len(names) == len(set(names))


def test_library_exports_every_declared_symbol():
    lib = _abi.load()
    for name in declared_functions():
        assert hasattr(lib, name), f"{name} declared in the header but not exported"
    assert set(declared_functions()) == set(_abi.SIGNATURES), "ctypes binding out of sync"


def test_build_info_names_the_architecture():
    assert b"sm_100a" in _abi.load().cf_build_info()


def test_block_size_agrees_across_languages():
    cuh = (ROOT / "cuda_force_b200" / "csrc" / "cf_common.cuh").read_text()
    m = re.search(r"inline\s+constexpr\s+\w+\s+kQuantBlockSize\s*=\s*(\d+)\s*;", cuh)
    assert m and int(m.group(1)) == ops.QUANT_BLOCK_SIZE
    h = re.search(r"#define\s+CF_QUANT_BLOCK_SIZE\s+(\d+)", HEADER.read_text())
    assert h and int(h.group(1)) == ops.QUANT_BLOCK_SIZE


@pytest.mark.parametrize(("count", "expected"), [(0, 0), (1, 1), (64, 1), (65, 2), (-5, 0),
                                                 (2**31 + 1, 2**25 + 1)])
def test_scale_count_known_answers(count, expected):
    assert _abi.load().cf_quant_scale_count(count) == expected


def test_status_strings():
    lib = _abi.load()
    assert lib.cf_status_string(_abi.CF_OK) == b"ok"
    assert b"timed out" in lib.cf_status_string(_abi.CF_ERR_DEVICE_TIMEOUT)
    assert lib.cf_status_string(99) == b"unknown status"


def test_abi_validates_arguments_before_touching_the_device():
    lib = _abi.load()
    null = None
    assert lib.cf_quantize_int8(null, 0, null, null, 0, null) == _abi.CF_OK  # empty is a no-op
    assert lib.cf_quantize_int8(null, 0, null, null, 64, null) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_quantize_int8(null, 0, null, null, -1, null) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_dequantize_int8(null, null, null, 64, null) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_quantize_dequantize(null, 0, null, 64, null) == _abi.CF_ERR_INVALID_ARGUMENT
    fake = ctypes.c_void_p(0x1000)
    assert lib.cf_quantize_int8(fake, 7, fake, fake, 64, null) == _abi.CF_ERR_UNSUPPORTED
    segs = (_abi.QuantSegment * 1)(_abi.QuantSegment(None, None, None, 64))
    assert lib.cf_quantize_int8_many(segs, 1, 0, null) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_quantize_int8_many(segs, 0, 0, null) == _abi.CF_OK


def test_lora_abi_validates_shapes_and_workspace():
    lib = _abi.load()
    f = ctypes.c_void_p(0x1000)
    args = dict(m=128, k=256, n=256, r=16)
    ws = lib.cf_lora_linear_workspace_bytes(args["m"], args["r"])
    assert ws >= args["m"] * args["r"] * 2
    call = lambda m, k, n, r, ws_bytes, wsp=f: lib.cf_lora_linear(  # noqa: E731
        f, f, 1, f, 0, f, 0, f, m, k, n, r, 2.0, _abi.CF_DTYPE_BF16, wsp, ws_bytes, None)
    assert call(128, 100, 256, 16, ws) == _abi.CF_ERR_UNSUPPORTED        # k % 64 != 0
    assert call(128, 256, 250, 16, ws) == _abi.CF_ERR_UNSUPPORTED        # n % 16 != 0
    assert call(128, 256, 256, 24, ws) == _abi.CF_ERR_UNSUPPORTED        # rank not 16/32/64
    assert call(128, 256, 256, 16, 128 * 16 * 2 - 16) == _abi.CF_ERR_WORKSPACE  # P is 16-bit here
    assert call(128, 256, 256, 16, ws, None) == _abi.CF_ERR_WORKSPACE
    assert call(-1, 256, 256, 16, ws) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_lora_linear(None, f, 1, f, 0, f, 0, f, 128, 256, 256, 16, 2.0,
                              _abi.CF_DTYPE_BF16, f, ws, None) == _abi.CF_ERR_INVALID_ARGUMENT
    # fp32 rows must be whole 16-byte units (k, n multiples of 4) ...
    assert lib.cf_lora_linear(f, f, 1, f, 0, f, 0, f, 128, 258, 256, 16, 2.0,
                              _abi.CF_DTYPE_F32, f, ws, None) == _abi.CF_ERR_UNSUPPORTED
    # ... and its workspace holds P in fp32
    assert ws >= args["m"] * args["r"] * 4
    # int8 weights take 16-bit activations only
    assert lib.cf_lora_linear_int8(f, f, f, f, 0, f, 0, f, 128, 256, 256, 16, 2.0,
                                   _abi.CF_DTYPE_F32, f, ws, None) == _abi.CF_ERR_UNSUPPORTED
    misaligned = ctypes.c_void_p(0x1008)
    assert lib.cf_lora_linear(misaligned, f, 1, f, 0, f, 0, f, 128, 256, 256, 16, 2.0,
                              _abi.CF_DTYPE_BF16, f, ws, None) == _abi.CF_ERR_MISALIGNED
    assert lib.cf_lora_linear(f, f, 1, f, 0, f, 0, f, 0, 256, 256, 16, 2.0,
                              _abi.CF_DTYPE_BF16, f, ws, None) == _abi.CF_OK      # empty


def test_newer_entry_points_validate_before_touching_the_device():
    # Every rejected call returns before any CUDA call, so this runs on a CPU
    # host; a call that passed validation would need a GPU and is not made.
    lib = _abi.load()
    f = ctypes.c_void_p(0x1000)
    odd = ctypes.c_void_p(0x1004)
    # fp32 matmul: k and n in whole 16-byte rows, 16-byte alignment, layouts
    assert lib.cf_matmul_f32(f, f, 0, f, 64, 64, 66, 1, None) == _abi.CF_ERR_UNSUPPORTED
    assert lib.cf_matmul_f32(f, f, 0, f, 64, 62, 64, 1, None) == _abi.CF_ERR_UNSUPPORTED
    assert lib.cf_matmul_f32(odd, f, 0, f, 64, 64, 64, 1, None) == _abi.CF_ERR_MISALIGNED
    assert lib.cf_matmul_f32(f, f, 7, f, 64, 64, 64, 1, None) == _abi.CF_ERR_INVALID_ARGUMENT
    assert lib.cf_matmul_f32(f, f, 0, f, 0, 64, 64, 1, None) == _abi.CF_OK    # empty
    # merge + quantise: 16-bit dtypes, whole 64-element blocks, ranks 16/32/64
    merge = lambda n, k, r, dt, w=f: lib.cf_lora_merge_quantize_int8(  # noqa: E731
        w, f, f, n, k, r, 2.0, dt, f, f, None)
    assert merge(64, 100, 16, _abi.CF_DTYPE_BF16) == _abi.CF_ERR_UNSUPPORTED
    assert merge(64, 128, 24, _abi.CF_DTYPE_BF16) == _abi.CF_ERR_UNSUPPORTED
    assert merge(64, 128, 16, _abi.CF_DTYPE_F32) == _abi.CF_ERR_UNSUPPORTED
    assert merge(64, 128, 16, _abi.CF_DTYPE_BF16, odd) == _abi.CF_ERR_MISALIGNED
    assert merge(-1, 128, 16, _abi.CF_DTYPE_BF16) == _abi.CF_ERR_INVALID_ARGUMENT
    assert merge(0, 128, 16, _abi.CF_DTYPE_BF16) == _abi.CF_OK
    # W8 gate/up + SwiGLU: 16-bit activations, k % 64, n % 8, alignment
    swiglu = lambda m, k, n, dt, x=f: lib.cf_w8_swiglu_int8(  # noqa: E731
        x, f, f, f, f, f, m, k, n, dt, None)
    assert swiglu(32, 100, 128, _abi.CF_DTYPE_BF16) == _abi.CF_ERR_UNSUPPORTED
    assert swiglu(32, 128, 100, _abi.CF_DTYPE_BF16) == _abi.CF_ERR_UNSUPPORTED
    assert swiglu(32, 128, 128, _abi.CF_DTYPE_F32) == _abi.CF_ERR_UNSUPPORTED
    assert swiglu(32, 128, 128, _abi.CF_DTYPE_BF16, odd) == _abi.CF_ERR_MISALIGNED
    assert lib.cf_w8_swiglu_int8(f, None, f, f, f, f, 32, 128, 128, _abi.CF_DTYPE_BF16,
                                 None) == _abi.CF_ERR_INVALID_ARGUMENT
    assert swiglu(0, 128, 128, _abi.CF_DTYPE_BF16) == _abi.CF_OK
    # residual add + RMSNorm: sizes, dtypes, residual / residual_out together
    norm = lambda rows, cols, dt, wdt, r=f, ro=f, x=f: lib.cf_fused_residual_rmsnorm(  # noqa: E731
        x, r, f, wdt, f, ro, rows, cols, 1e-6, dt, None)
    bf16 = _abi.CF_DTYPE_BF16
    assert norm(-1, 64, bf16, bf16) == _abi.CF_ERR_INVALID_ARGUMENT
    assert norm(4, -1, bf16, bf16) == _abi.CF_ERR_INVALID_ARGUMENT
    assert norm(4, 64, 7, 7) == _abi.CF_ERR_UNSUPPORTED
    assert norm(4, 64, bf16, _abi.CF_DTYPE_F16) == _abi.CF_ERR_UNSUPPORTED
    assert norm(4, 64, bf16, bf16, ro=None) == _abi.CF_ERR_INVALID_ARGUMENT
    assert norm(4, 64, bf16, bf16, x=None) == _abi.CF_ERR_INVALID_ARGUMENT
    assert norm(1 << 40, 1 << 20, bf16, bf16) == _abi.CF_ERR_INVALID_ARGUMENT
    assert norm(0, 64, bf16, bf16) == _abi.CF_OK
    assert norm(4, 0, bf16, bf16) == _abi.CF_OK


def test_python_wrappers_validate_shapes_on_the_host():
    w = torch.zeros(64, 100, dtype=torch.bfloat16)
    with pytest.raises(ValueError, match="multiple of 64"):
        cf.lora_merge_quantize_int8(w, torch.zeros(4, 100, dtype=torch.bfloat16),
                                    torch.zeros(64, 4, dtype=torch.bfloat16), 1.0)
    with pytest.raises(ValueError, match="lora_b must be"):
        cf.lora_merge_quantize_int8(torch.zeros(64, 128, dtype=torch.bfloat16),
                                    torch.zeros(4, 128, dtype=torch.bfloat16),
                                    torch.zeros(64, 5, dtype=torch.bfloat16), 1.0)
    codes = torch.zeros(128, 256, dtype=torch.int8)
    scales = torch.ones(128 * 256 // 64)
    with pytest.raises(ValueError, match="input features"):
        cf.w8_swiglu_int8(torch.zeros(2, 128, dtype=torch.bfloat16), codes, scales, codes, scales)
    with pytest.raises(ValueError, match="float32"):
        cf.matmul_f32(torch.zeros(4, 8, dtype=torch.bfloat16), torch.zeros(8, 4))
    with pytest.raises(ValueError, match=r"\[m, k\] and b \[k, n\]"):
        cf.matmul_f32(torch.zeros(4, 8), torch.zeros(9, 4))
    # rmsnorm / fused_residual_rmsnorm: the reference's messages (ops.py:260-266, :361-367)
    with pytest.raises(ValueError, match="weight must be 1-D"):
        cf.rmsnorm(torch.zeros(2, 8), torch.zeros(2, 8))
    with pytest.raises(ValueError, match="does not match the last dimension"):
        cf.rmsnorm(torch.zeros(2, 8), torch.zeros(9))
    with pytest.raises(ValueError, match="same shape"):
        cf.fused_residual_rmsnorm(torch.zeros(2, 8), torch.zeros(3, 8), torch.zeros(8))
    with pytest.raises(ValueError, match="1-D of length 8"):
        cf.fused_residual_rmsnorm(torch.zeros(2, 8), torch.zeros(2, 8), torch.zeros(7))
    empty = torch.zeros(0, 8)
    assert cf.rmsnorm(empty, torch.ones(8)).shape == (0, 8)
    assert [t.shape for t in cf.fused_residual_rmsnorm(empty, empty, torch.ones(8))] == [(0, 8)] * 2


def test_dispatcher_schemas_match_the_reference():
    # All ten, byte-identical to reference cpp/src/bindings.cpp:342-355.
    expected = {
        "rmsnorm": "cudaforge::rmsnorm(Tensor input, Tensor weight, float eps) -> Tensor",
        "softmax": "cudaforge::softmax(Tensor input) -> Tensor",
        "lora_linear": "cudaforge::lora_linear(Tensor x, Tensor w, Tensor a, Tensor b, float scale) -> Tensor",
        "sum": "cudaforge::sum(Tensor input) -> Tensor",
        "silu": "cudaforge::silu(Tensor input) -> Tensor",
        "gelu": "cudaforge::gelu(Tensor input) -> Tensor",
        "swiglu": "cudaforge::swiglu(Tensor gate, Tensor up) -> Tensor",
        "fused_residual_rmsnorm": ("cudaforge::fused_residual_rmsnorm(Tensor x, Tensor residual, "
                                   "Tensor weight, float eps) -> Tensor[]"),
        "quantize_int8": "cudaforge::quantize_int8(Tensor input) -> Tensor[]",
        "dequantize_int8": "cudaforge::dequantize_int8(Tensor quantised, Tensor scales) -> Tensor",
    }
    for name, schema in expected.items():
        assert str(getattr(torch.ops.cudaforge, name).default._schema) == schema


def test_reference_side_operators_keep_their_semantics():
    # softmax / sum / silu / gelu / swiglu are not accelerated here; they stay
    # registered as compositions of the reference semantics (bindings.cpp:250-295).
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 33, generator=g)
    assert torch.equal(torch.ops.cudaforge.softmax(x), torch.softmax(x, -1))
    assert torch.equal(torch.ops.cudaforge.sum(x), x.sum())
    assert torch.equal(torch.ops.cudaforge.silu(x), torch.nn.functional.silu(x))
    assert torch.equal(torch.ops.cudaforge.gelu(x), torch.nn.functional.gelu(x, approximate="tanh"))
    gate, up = x.bfloat16(), torch.randn(4, 33, generator=g).bfloat16()
    ref = (torch.nn.functional.silu(gate.float()) * up.float()).bfloat16()
    assert torch.equal(torch.ops.cudaforge.swiglu(gate, up), ref)
    with pytest.raises(RuntimeError, match="derivative for cudaforge::silu is not implemented"):
        torch.ops.cudaforge.silu(x.requires_grad_()).sum().backward()


def test_cpu_tensors_fail_loudly():
    # This package's API never computes on the host.
    with pytest.raises(RuntimeError, match="CUDA"):
        cf.quantize_int8(torch.randn(128))
    with pytest.raises(RuntimeError, match="CUDA"):
        cf.fused_residual_rmsnorm(torch.randn(2, 8), torch.randn(2, 8), torch.ones(8))
    # Additive ops have no host kernel in the dispatcher either.
    with pytest.raises((RuntimeError, NotImplementedError)):
        torch.ops.cudaforge.quantize_dequantize(torch.randn(128))


def test_extension_imports_as_the_reference_module():
    # python/cudaforge/ops.py:44-58 imports cudaforge._C and asks it whether
    # CUDA kernels were compiled in.
    import importlib

    mod = importlib.import_module("cuda_force_b200._C")
    assert mod.cuda_kernels_available() is True


@pytest.mark.parametrize("name", sorted(golden_cases()))
def test_dispatcher_host_kernels_match_reference_fixture(name):
    # Reference callers may pass host tensors to the registered ops
    # (python/cudaforge/ops.py:150-152); the host kernels keep the reference's
    # results bit for bit.
    case = golden_cases()[name]
    x = numpy_to_torch(case["dtype"], case["input"])
    codes, scales = torch.ops.cudaforge.quantize_int8(x)
    assert np.array_equal(codes.reshape(-1).numpy(), case["codes"])
    assert np.array_equal(scales.numpy().view(np.int32), case["scales"].view(np.int32))
    deq = torch.ops.cudaforge.dequantize_int8(codes, scales)
    assert np.array_equal(deq.reshape(-1).numpy(), case["deq"], equal_nan=True)


@pytest.mark.parametrize("name", sorted(norm_cases()))
def test_dispatcher_host_norm_matches_reference_fixture(name):
    case = norm_cases()[name]
    normalised, summed = torch.ops.cudaforge.fused_residual_rmsnorm(
        case["x"], case["residual"], case["weight"], case["eps"])
    assert torch.equal(normalised, case["normalised"]) and torch.equal(summed, case["summed"])
    plain = torch.ops.cudaforge.rmsnorm(case["x"], case["weight"], case["eps"])
    assert torch.equal(plain, case["plain"])


def test_dispatcher_host_lora_linear_is_the_reference_composition():
    g = torch.Generator().manual_seed(3)
    x, w = torch.randn(7, 129, generator=g), torch.randn(129, 65, generator=g)
    a, b = torch.randn(129, 3, generator=g), torch.randn(3, 65, generator=g)
    y = torch.ops.cudaforge.lora_linear(x, w, a, b, 0.5)
    assert torch.equal(y, x @ w + 0.5 * ((x @ a) @ b))


@pytest.mark.parametrize(
    ("shapes", "message"),
    [
        ({"x": (4, 31), "w": (32, 16), "a": (32, 4), "b": (4, 16)}, "input features"),
        ({"x": (4, 32), "w": (32, 16), "a": (31, 4), "b": (4, 16)}, "lora_a"),
        ({"x": (4, 32), "w": (32, 16), "a": (32, 4), "b": (5, 16)}, "lora_b"),
        ({"x": (4, 32), "w": (32, 16), "a": (32, 4), "b": (4, 15)}, "lora_b"),
    ],
)
def test_lora_rejects_mismatched_shapes(shapes, message):
    # Same cases and messages as the reference's tests/python/test_ops.py:141-161.
    with pytest.raises(ValueError, match=message):
        cf.lora_linear(torch.randn(*shapes["x"]), torch.randn(*shapes["w"]),
                       torch.randn(*shapes["a"]), torch.randn(*shapes["b"]))


def test_dequantize_rejects_a_wrong_scale_count():
    with pytest.raises(ValueError, match="block scales"):
        cf.dequantize_int8(torch.zeros(128, dtype=torch.int8), torch.ones(1))


def test_lora_int8_rejects_wrong_scale_count():
    with pytest.raises(ValueError, match="block scales"):
        cf.lora_linear_int8(torch.randn(2, 64), torch.zeros(16, 64, dtype=torch.int8),
                            torch.ones(3), torch.randn(64, 16), torch.randn(16, 16))


def test_backend_report_is_truthful_without_a_gpu():
    report = cf.backend_report()
    assert report.extension_loaded
    assert report.using_custom_kernels == torch.cuda.is_available()
    assert "cuda_force_b200" in str(report)


def test_autograd_inputs_are_rejected():
    x = torch.randn(4, 64, requires_grad=True)
    with pytest.raises(RuntimeError):
        cf.quantize_int8(x)


def test_header_is_plain_c_and_links_from_c(tmp_path):
    # A cgo / JNI / FFI binding sees the header as C: it must compile as
    # pedantic C99 and link against the library with no C++ runtime in sight.
    import subprocess

    root = Path(__file__).resolve().parents[1]
    exe = tmp_path / "abi_from_c"
    lib_dir = root / "cuda_force_b200"
    subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-Werror", "-pedantic",
                    f"-I{root / 'include'}", str(root / "tests" / "native" / "abi_from_c.c"),
                    "-o", str(exe), f"-L{lib_dir}", "-l:libcudaforge_b200.so",
                    f"-Wl,-rpath,{lib_dir}"], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0 and out.stdout.strip() == "ok", out.stdout + out.stderr
