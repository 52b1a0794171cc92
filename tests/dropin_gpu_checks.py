"""Checks run inside a process whose ``cudaforge`` is the reference's package with
this build's ``_C.so`` as its extension (see test_reference_dropin_gpu.py).

Every call goes through the reference's own wrapper (python/cudaforge/ops.py):
its dtype gate sends fp32 CUDA tensors to ``torch.ops.cudaforge.*``, which this
build's extension serves with its sm_100a kernels. The shapes and tolerances
follow the reference's on-GPU parity script (examples/kernel_parity.py:57-133)
and its operator tests (tests/python/test_ops.py:105-138, 174-229); quantise and
dequantise are also compared bit for bit with the reference's own host
implementation (ops.py:215-240) on the same values.
"""

from __future__ import annotations

import json
import sys

import torch


def main() -> int:
    import cudaforge
    from cudaforge import _C, ops

    dev = torch.device("cuda", 0)
    report = ops.backend_report()
    out: dict = {"report": str(report), "extension": _C.__file__, "checks": []}
    assert report.using_custom_kernels, report
    torch.manual_seed(0)

    def check(name: str, err: float, tol: float) -> None:
        out["checks"].append({"name": name, "error": err, "tol": tol, "ok": err <= tol})

    for rows, cols in [(1, 1), (4, 17), (8, 128), (33, 1023), (16, 4096)]:
        x = torch.randn(rows, cols, device=dev)
        w = torch.randn(cols, device=dev)
        ref = x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        check(f"rmsnorm {rows}x{cols}", (ops.rmsnorm(x, w) - ref).abs().max().item(), 1e-4)
        r = torch.randn(rows, cols, device=dev)
        got, summed = ops.fused_residual_rmsnorm(x, r, w, 1e-6)
        s = x + r
        ref = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + 1e-6) * w
        check(f"fused_residual_rmsnorm {rows}x{cols}",
              max((got - ref).abs().max().item(), (summed - s).abs().max().item()), 1e-4)

    for batch, k, n, rank in [(1, 8, 4, 2), (7, 129, 65, 3), (64, 1024, 1024, 16)]:
        # the parity script's shapes and its tolerance (max absolute error 1e-2)
        x, w = torch.randn(batch, k, device=dev), torch.randn(k, n, device=dev)
        a, b = torch.randn(k, rank, device=dev), torch.randn(rank, n, device=dev)
        xd, wd, ad, bd = (t.double() for t in (x, w, a, b))
        ref = xd @ wd + 2.0 * ((xd @ ad) @ bd)
        err = (ops.lora_linear(x, w, a, b, 2.0).double() - ref).abs().max().item()
        check(f"lora_linear {batch}x{k}x{n}r{rank} (parity script)", err, 1e-2)

    for batch, k, n, rank in [(1, 8, 4, 2), (4, 64, 32, 8), (7, 129, 65, 3), (16, 256, 256, 16)]:
        # the operator test: assert_close(rtol=1e-4, atol=1e-4) against the fp32 definition
        # evaluated on the host, scale 0.25
        x, w = torch.randn(batch, k), torch.randn(k, n)
        a, b = torch.randn(k, rank), torch.randn(rank, n)
        expected = x @ w + 0.25 * ((x @ a) @ b)
        y = ops.lora_linear(x.to(dev), w.to(dev), a.to(dev), b.to(dev), 0.25).cpu()
        excess = ((y - expected).abs() - 1e-4 * expected.abs()).max().item()
        check(f"lora_linear {batch}x{k}x{n}r{rank} (operator test)", excess, 1e-4)

    x, w, a = torch.randn(4, 32), torch.randn(32, 16), torch.randn(32, 4)
    y0 = ops.lora_linear(x.to(dev), w.to(dev), a.to(dev), torch.zeros(4, 16, device=dev), 1.0)
    check("lora_linear with zero B is the frozen layer",
          ((y0.cpu() - x @ w).abs() - 1e-5 * (x @ w).abs()).max().item(), 1e-5)
    b = torch.randn(4, 16)
    zw = torch.zeros(32, 16, device=dev)
    y1 = ops.lora_linear(x.to(dev), zw, a.to(dev), b.to(dev), 1.0)
    y2 = ops.lora_linear(x.to(dev), zw, a.to(dev), b.to(dev), 2.0)
    check("lora_linear is linear in scale",
          ((y2 - 2 * y1).abs() - 1e-4 * (2 * y1).abs()).max().item(), 1e-4)

    for count in [1, 63, 64, 65, 1000, 1 << 20]:
        x = torch.randn(count, device=dev) * 5.0
        q, s = ops.quantize_int8(x)
        restored = ops.dequantize_int8(q, s)
        bound = s.max().item() / 2 + 1e-6
        check(f"quant round trip {count}", (x - restored).abs().max().item(), bound)
        q_ref, s_ref = ops._quantize_int8_reference(x.cpu())
        same = (torch.equal(q.cpu(), q_ref) and torch.equal(s.cpu(), s_ref) and
                torch.equal(restored.cpu(), ops._dequantize_int8_reference(q_ref, s_ref)))
        check(f"quant bit-exact vs the reference's host implementation {count}",
              0.0 if same else 1.0, 0.0)
        check(f"quantization_error {count}",
              abs(ops.quantization_error(x).item() - (x - restored).abs().max().item()), 0.0)

    zeros = torch.zeros(128, device=dev)
    q, s = ops.quantize_int8(zeros)
    check("all-zero block round trips exactly",
          0.0 if bool((s > 0).all()) and torch.equal(ops.dequantize_int8(q, s), zeros) else 1.0, 0.0)
    try:
        ops.dequantize_int8(q, torch.ones(1, device=dev))
        check("wrong scale count raises ValueError('block scales')", 1.0, 0.0)
    except ValueError as error:
        check("wrong scale count raises ValueError('block scales')",
              0.0 if "block scales" in str(error) else 1.0, 0.0)
    torch.cuda.synchronize()
    out["package"] = cudaforge.__file__
    print(json.dumps(out))
    return 0 if all(c["ok"] for c in out["checks"]) else 1


if __name__ == "__main__":
    sys.exit(main())
