"""Test helpers: golden fixture access and tensor/ABI glue."""

from __future__ import annotations

import ctypes
import hashlib
import json
from pathlib import Path

import numpy as np
import torch

GOLDEN = Path(__file__).resolve().parent / "golden"

DTYPE_TAG_TO_TORCH = {"f32": torch.float32, "f16": torch.float16, "bf16": torch.bfloat16}
TORCH_TO_CF = {torch.float32: 0, torch.float16: 1, torch.bfloat16: 2}


def sha(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()


def golden_cases() -> dict[str, dict[str, np.ndarray | str]]:
    data = np.load(GOLDEN / "quant_cases.npz")
    meta = json.loads(str(data["__meta__"]))
    cases = {}
    for name, tag in meta.items():
        cases[name] = {
            "dtype": tag,
            "input": data[f"{name}/input"],
            "codes": data[f"{name}/codes"],
            "scales": data[f"{name}/scales"],
            "deq": data[f"{name}/deq"],
        }
    return cases


def norm_cases() -> dict[str, dict]:
    """Residual-add + RMSNorm fixtures as torch tensors (CPU), with eps and dtypes."""
    data = np.load(GOLDEN / "norm_cases.npz")
    meta = json.loads(str(data["__meta__"]))
    cases = {}
    for name, m in meta.items():
        tag, wtag = m["dtype"], m["weight_dtype"]
        cases[name] = {
            "dtype": DTYPE_TAG_TO_TORCH[tag],
            "eps": m["eps"],
            "x": numpy_to_torch(tag, data[f"{name}/x"]),
            "residual": numpy_to_torch(tag, data[f"{name}/residual"]),
            "weight": numpy_to_torch(wtag, data[f"{name}/weight"]),
            **{k: numpy_to_torch(tag, data[f"{name}/{k}"]) for k in ("normalised", "summed", "plain")},
        }
    return cases


def golden_hashes() -> dict[str, dict]:
    return json.loads((GOLDEN / "quant_hashes.json").read_text())


def regenerate(tag: str, spec: dict) -> np.ndarray:
    """Same generator as tests/golden/make_golden.py:regenerate (numpy PCG64)."""
    rng = np.random.default_rng(spec["seed"])
    x = rng.standard_normal(tuple(spec["shape"]), dtype=np.float32) * np.float32(spec["std"])
    if "outlier_p" in spec:
        mask = rng.random(x.shape, dtype=np.float32) < spec["outlier_p"]
        x = np.where(mask, x * np.float32(spec["outlier_mult"]), x).astype(np.float32)
    if tag == "f16":
        return x.astype(np.float16)
    if tag == "bf16":
        return torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    return x.astype(np.float32)


def numpy_to_torch(tag: str, arr: np.ndarray) -> torch.Tensor:
    t = torch.from_numpy(np.ascontiguousarray(arr))
    if tag == "bf16":
        return t.view(torch.int16).view(torch.bfloat16)
    return t


def torch_to_numpy_input(t: torch.Tensor) -> np.ndarray:
    """Tensor -> the oracle's input convention (bf16 as uint16 bits)."""
    t = t.detach().cpu().contiguous()
    if t.dtype == torch.bfloat16:
        return t.view(torch.int16).numpy().view(np.uint16)
    return t.numpy()


def ptr(t: torch.Tensor) -> ctypes.c_void_p:
    return ctypes.c_void_p(t.data_ptr())


def stream_ptr() -> ctypes.c_void_p:
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)
