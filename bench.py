"""Benchmark of the quantised-linear hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]
                    [--workload NAME]

Multi-GPU: launched by torchrun (one rank per GPU, NCCL); RANK / LOCAL_RANK /
WORLD_SIZE come from the environment. Rank 0 prints one JSON line.

Default workload ``llama7b_stack_quant`` = benchmark config 2: block-INT8
quantisation of a Llama-2-7B-shaped bf16 weight stack (32 layers x [4 x
4096x4096, 2 x 11008x4096, 4096x11008], N(0, 0.02) with 0.1% of entries x20),
block 64 along the input dimension, layers sharded across ranks with no
communication ("strong" scaling: the stack is fixed, each rank quantises
32/N layers). Metric: aggregate algorithmic GB/s = 3.0625 B/element (2 B bf16
read, 1 B code + 4/64 B scale written) x elements / max-over-ranks time.

Other workloads (``--workload``) time the remaining benchmark configs for the
design notes; the driver's default line is config 2.

Timing rules: W >= 3 warm-up steps; the timed region is K steps bracketed by a
barrier and torch.cuda.synchronize() on both sides, timed with CUDA events on
the launching stream, max over ranks. Inputs are larger than L2 (126 MB) for
every workload listed as such in ``config.l2``; the others flush L2 between
steps by writing a 256 MiB buffer (outside the per-launch events).
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time
from pathlib import Path

import torch

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

CONFIG1_ROWS = 4096  # rows of 4096 fp32 for the config 1 workloads (--elements)
# config 5 all-gather: "mc" (NVLink multicast stores), "fused" (one peer store per rank),
# "ce" (copy engines), "nccl", or "auto" (mc where the GPUs support multicast, else fused)
COMM_MODE = "auto"
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}
BYTES_PER_ELEM_BF16_QUANT = 2 + 1 + 4 / 64


def load_peaks() -> tuple[dict, str]:
    path = ROOT / "MEASURED_PEAKS.json"
    if path.exists():
        return json.loads(path.read_text()), "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def size_matched_copy(nbytes: float, device, flush, steps: int = 10) -> dict | None:
    """A plain torch copy that moves the same bytes as one step, timed like the step.

    Half of ``nbytes`` is read and half written, with the same L2 flush before
    each launch and CUDA events around it: the best a copy kernel reaches at
    this size, where launch and ramp-up latency weigh on a short launch.
    """
    half = int(nbytes // 2) // 16 * 16
    if half <= 0 or nbytes > 4e9:
        return None
    src = torch.empty(half, dtype=torch.uint8, device=device).fill_(1)
    dst = torch.empty_like(src)
    for _ in range(3):
        dst.copy_(src)
    times = []
    for i in range(steps):
        if flush is not None:
            flush.fill_(i & 0xFF)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        dst.copy_(src)
        end.record()
        end.synchronize()
        times.append(start.elapsed_time(end))
    ms = statistics.median(times)
    del src, dst
    return {"gbs": round(2 * half / (ms * 1e-3) / 1e9, 1), "us": round(ms * 1e3, 2),
            "what": f"torch copy_ of {2 * half / 1e6:.1f} MB (half read, half written), same "
                    f"L2 flush, median of {steps}"}


def load_traffic() -> dict:
    path = ROOT / "profiles" / "traffic.json"
    return json.loads(path.read_text()) if path.exists() else {}


# ---------------------------------------------------------------------------
# Distributed plumbing
# ---------------------------------------------------------------------------
class Dist:
    def __init__(self, n_gpus: int):
        self.world = int(os.environ.get("WORLD_SIZE", "1"))
        self.rank = int(os.environ.get("RANK", "0"))
        self.local_rank = int(os.environ.get("LOCAL_RANK", "0"))
        if self.world != n_gpus and not (self.world == 1 and n_gpus == 1):
            if self.world == 1:
                raise SystemExit(f"--gpus {n_gpus} needs torchrun with {n_gpus} processes")
        self.pg = None
        if self.world > 1:
            import torch.distributed as dist

            torch.cuda.set_device(self.local_rank)
            dist.init_process_group("nccl", device_id=torch.device("cuda", self.local_rank))
            self.pg = dist

    @property
    def device(self) -> torch.device:
        return torch.device("cuda", self.local_rank)

    def barrier(self) -> None:
        if self.pg is not None:
            self.pg.barrier()

    def max(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.MAX)
        return t.item()

    def sum(self, value: float) -> float:
        if self.pg is None:
            return value
        t = torch.tensor([value], dtype=torch.float64, device=self.device)
        self.pg.all_reduce(t, op=self.pg.ReduceOp.SUM)
        return t.item()

    def close(self) -> None:
        if self.pg is not None:
            self.pg.destroy_process_group()


# ---------------------------------------------------------------------------
# Clock sampling during the timed region (NVML)
# ---------------------------------------------------------------------------
class ClockSampler:
    REASONS = {
        "sw_power_cap": 0x4,
        "hw_slowdown": 0x8,
        "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40,
        "hw_power_brake_slowdown": 0x80,
    }

    def __init__(self, index: int, period_s: float = 0.02):
        self.samples: list[tuple[int, int]] = []
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        try:
            import pynvml

            pynvml.nvmlInit()
            self._nvml = pynvml
            visible = os.environ.get("CUDA_VISIBLE_DEVICES")
            phys = int(visible.split(",")[index]) if visible else index
            self._handle = pynvml.nvmlDeviceGetHandleByIndex(phys)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._handle, pynvml.NVML_CLOCK_SM)
        except Exception:  # noqa: BLE001 - clocks are reported as unavailable
            self._nvml = None
        self.period = period_s

    def _run(self) -> None:
        n = self._nvml
        while not self._stop.is_set():
            try:
                mhz = n.nvmlDeviceGetClockInfo(self._handle, n.NVML_CLOCK_SM)
                reasons = n.nvmlDeviceGetCurrentClocksEventReasons(self._handle)
                self.samples.append((mhz, reasons))
            except Exception:  # noqa: BLE001
                pass
            time.sleep(self.period)

    def __enter__(self):
        if self._nvml is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        if self._thread is not None:
            self._thread.join()

    def summary(self) -> dict:
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": ["unavailable"]}
        reasons = set()
        for _, mask in self.samples:
            for name, bit in self.REASONS.items():
                if mask & bit:
                    reasons.add(name)
        return {
            "sm_mhz": statistics.median(m for m, _ in self.samples),
            "sm_max_mhz": self.max_mhz,
            "reasons": sorted(reasons),
            "samples": len(self.samples),
        }


# ---------------------------------------------------------------------------
# Workload: benchmark config 2 (Llama-2-7B stack, bf16, layer-sharded quantise)
# ---------------------------------------------------------------------------
LLAMA7B_LAYER = [(4096, 4096)] * 4 + [(11008, 4096)] * 2 + [(4096, 11008)]
LLAMA7B_LAYERS = 32


def llama_layer_weights(layer: int, device: torch.device, seed: int = 2026) -> list[torch.Tensor]:
    """N(0, 0.02) bf16 weights with 0.1% of entries multiplied by 20, seeded per layer."""
    g = torch.Generator(device=device).manual_seed(seed + layer)
    out = []
    for shape in LLAMA7B_LAYER:
        w = torch.randn(shape, device=device, generator=g, dtype=torch.float32) * 0.02
        mask = torch.rand(shape, device=device, generator=g) < 0.001
        w = torch.where(mask, w * 20.0, w).to(torch.bfloat16)
        out.append(w)
        del mask
    return out


class LlamaStackQuant:
    name = "llama7b_stack_quant"
    metric = "INT8 block quantise GB/s (Llama-2-7B bf16 stack)"
    unit = "GB/s"
    dtype = "bf16->int8"
    kernel = "quantize_tma_kernel<bf16>"
    bound = "hbm"
    scaling = "strong"
    flush_l2 = False

    def __init__(self, dist: Dist, n_layers: int = LLAMA7B_LAYERS):
        self.dist = dist
        self.n_layers = n_layers
        # layers l with l % world == rank (cuda_force_b200.sharding.layer_shard), computed here
        # so that building the workload imports nothing of the package (the reference arm).
        self.layers = list(range(dist.rank, n_layers, dist.world))
        self.elems_per_layer = sum(a * b for a, b in LLAMA7B_LAYER)

    def config(self) -> dict:
        return {
            "workload": "benchmark config 2: Llama-2-7B bf16 weight stack block-INT8 quantise",
            "layers": self.n_layers,
            "layer_shapes": [list(s) for s in LLAMA7B_LAYER],
            "block": 64,
            "elements": self.elems_per_layer * self.n_layers,
            "values": "N(0,0.02), 0.1% x20 outliers, seeded per layer",
            "parallelism": f"layer-sharded over {self.dist.world} GPU(s), no communication",
            "l2": "inputs larger than L2 (each step streams the rank's whole stack)",
        }

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        if reference:
            # the reference arm samples one 4096x4096 projection of layer 0
            self.inputs = [llama_layer_weights(0, dev)[0].cpu()]
            return
        from cuda_force_b200 import _abi
        from cuda_force_b200.sharding import layer_shard

        assert layer_shard(self.n_layers, self.dist.rank, self.dist.world) == self.layers
        self.lib = _abi.load()
        self.inputs, self.codes, self.scales = [], [], []
        for layer in self.layers:
            for w in llama_layer_weights(layer, dev):
                self.inputs.append(w)
                self.codes.append(torch.empty(w.shape, dtype=torch.int8, device=dev))
                self.scales.append(torch.empty(w.numel() // 64, dtype=torch.float32, device=dev))
        n = len(self.inputs)
        self.segs = (_abi.QuantSegment * n)(*[
            _abi.QuantSegment(i.data_ptr(), c.data_ptr(), s.data_ptr(), i.numel())
            for i, c, s in zip(self.inputs, self.codes, self.scales)
        ])
        self.nseg = n
        self.launches_per_step = (n + _abi.CF_MAX_SEGMENTS - 1) // _abi.CF_MAX_SEGMENTS
        self.work_per_step = BYTES_PER_ELEM_BF16_QUANT * self.elems_per_layer * len(self.layers)

    def step(self, stream: torch.cuda.Stream) -> None:
        from cuda_force_b200 import _abi

        _abi.check(self.lib.cf_quantize_int8_many(self.segs, self.nseg, _abi.CF_DTYPE_BF16,
                                                  stream.cuda_stream), "quantize_many")

    def verify(self) -> None:
        """Spot-check the timed outputs against the oracle (sampled blocks)."""
        from oracle import quant_ref

        g = torch.Generator().manual_seed(self.dist.rank)
        for idx in range(len(self.inputs)):
            flat_in = self.inputs[idx].reshape(-1)
            nblocks = flat_in.numel() // 64
            picks = torch.randint(0, nblocks, (8,), generator=g).tolist() + [nblocks - 1]
            for b in picks:
                x = flat_in[b * 64:(b + 1) * 64].cpu().view(torch.int16).numpy().view("uint16")
                rc, rs = quant_ref.quantize(x)
                got = self.codes[idx].reshape(-1)[b * 64:(b + 1) * 64].cpu().numpy()
                if not (got == rc).all() or self.scales[idx][b].item() != rs[0]:
                    raise SystemExit(f"parity failure in segment {idx} block {b}")

    # -- end to end through the public API with host buffers -----------------
    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        host_in = [w.cpu().pin_memory() for w in self.inputs[:7]]  # one layer's tensors
        per_layer = len(host_in)
        n_layers = len(self.layers)
        host_codes = [torch.empty(w.shape, dtype=torch.int8).pin_memory() for w in host_in]
        host_scales = [torch.empty(w.numel() // 64).pin_memory() for w in host_in]
        copy_stream = torch.cuda.Stream(device=dev)
        h2d = sum(t.numel() * 2 for t in host_in) * n_layers
        d2h = sum(c.numel() + s.numel() * 4 for c, s in zip(host_codes, host_scales)) * n_layers

        def one_step() -> None:
            # Layer-pipelined: H2D of layer i+1 on a copy stream overlaps the
            # quantisation and D2H of layer i on the compute stream.
            compute = torch.cuda.current_stream(dev)
            staged = [t.to(dev, non_blocking=True) for t in host_in]
            for layer in range(n_layers):
                ready = torch.cuda.Event()
                ready.record(compute)
                outs = cf.quantize_int8_many(staged)
                if layer + 1 < n_layers:
                    copy_stream.wait_stream(compute)
                    with torch.cuda.stream(copy_stream):
                        nxt = [t.to(dev, non_blocking=True) for t in host_in]
                    compute.wait_stream(copy_stream)
                    staged = nxt
                for (c, s), hc, hs in zip(outs, host_codes, host_scales):
                    hc.copy_(c, non_blocking=True)
                    hs.copy_(s, non_blocking=True)

        one_step()
        torch.cuda.synchronize(dev)
        self.dist.barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            one_step()
        torch.cuda.synchronize(dev)
        self.dist.barrier()
        elapsed = self.dist.max(time.perf_counter() - t0)
        total_bytes = self.dist.sum(self.work_per_step) * steps
        return {
            "value": total_bytes / elapsed / 1e9,
            "unit": self.unit,
            "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h),
            "steps": steps,
            "api": "cuda_force_b200.quantize_int8_many per layer, pinned host in/out",
            "note": "each layer's host source is one pinned layer-sized buffer re-sent per layer",
        }

    # -- CPU: the reference's own CPU implementation --------------------------
    def cpu_sample(self):
        """(fn, algorithmic bytes per call, kind, description) for the reference CPU path."""
        x = self.inputs[0].cpu()  # one [4096, 4096] bf16 projection
        fn, kind = reference_quantize_fn()

        def run() -> None:
            fn(x)

        return (run, BYTES_PER_ELEM_BF16_QUANT * x.numel(), kind,
                "one 4096x4096 bf16 projection of layer 0 per call")


def reference_quantize_fn():
    """The reference's CPU quantiser: its compiled CPU operator if built, else the port."""
    from oracle import build_ref

    if build_ref.load():
        return (lambda x: torch.ops.cudaforge_ref.quantize_int8(x)), "reference"
    from oracle import quant_ref

    return (lambda x: quant_ref.quantize(x.view(torch.int16).numpy().view("uint16")
                                         if x.dtype == torch.bfloat16 else x.numpy())), "port"


def quantize_weight(w: torch.Tensor, reference: bool = False):
    """Block-INT8 codes and scales of a weight: this package's kernel, or, for the
    reference arm, the reference's CPU operator (bit-identical output)."""
    if not reference:
        import cuda_force_b200 as cf

        return cf.quantize_int8(w)
    fn, _kind = reference_quantize_fn()
    out = fn(w.cpu())
    if isinstance(out[0], torch.Tensor):
        return out[0].reshape(w.shape), out[1]
    codes, scales = out
    return torch.from_numpy(codes).reshape(w.shape), torch.from_numpy(scales)


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    import platform

    return platform.processor() or "unknown"


class Config1Quant:
    """benchmark config 1: fp32 [4096, 4096] N(0,1) block-INT8 quantise (or dequantise)."""

    name = "config1_quant_f32"
    unit = "GB/s"
    bound = "hbm"
    scaling = "weak"
    flush_l2 = True
    dequant = False

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist
        op = "dequantise" if self.dequant else "quantise"
        self.rows = CONFIG1_ROWS
        self.metric = f"INT8 block {op} GB/s (fp32 {self.rows}x4096)"
        self.dtype = "int8->f32" if self.dequant else "f32->int8"
        self.kernel = "dequantize_vec_kernel" if self.dequant else "quantize_tma_kernel<f32>"

    def config(self) -> dict:
        return {"workload": (f"benchmark config 1: fp32 [4096,4096] N(0,1) block-64 "
                             f"{'dequantise' if self.dequant else 'quantise'}")
                if self.rows == 4096 else
                f"config 1 kernel at [{self.rows},4096] fp32 (size study, not a benchmark config)",
                "block": 64, "bytes_per_element": 4 + 1 + 4 / 64,
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "parallelism": f"{self.dist.world} independent replica(s)"}

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(1)
        self.x = torch.randn(self.rows, 4096, device=dev, generator=g)
        self.work_per_step = (4 + 1 + 4 / 64) * self.x.numel()
        if reference:
            return
        from cuda_force_b200 import _abi

        self.lib = _abi.load()
        self.codes = torch.empty(self.rows, 4096, dtype=torch.int8, device=dev)
        self.scales = torch.empty(self.rows * 64, device=dev)
        self.out = torch.empty(self.rows, 4096, device=dev)
        _abi.check(self.lib.cf_quantize_int8(self.x.data_ptr(), 0, self.codes.data_ptr(),
                                             self.scales.data_ptr(), self.x.numel(), None), "q")
        self.work_per_step = (4 + 1 + 4 / 64) * self.x.numel()
        self.launches_per_step = 1

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        if self.dequant:
            st = self.lib.cf_dequantize_int8(self.codes.data_ptr(), self.scales.data_ptr(),
                                             self.out.data_ptr(), self.x.numel(), stream.cuda_stream)
        else:
            st = self.lib.cf_quantize_int8(self.x.data_ptr(), 0, self.codes.data_ptr(),
                                           self.scales.data_ptr(), self.x.numel(), stream.cuda_stream)
        _abi.check(st, self.name)

    def verify(self) -> None:
        from oracle import quant_ref

        rows = min(self.rows, 4096)  # a bounded prefix on very large size studies
        rc, rs = quant_ref.quantize(self.x[:rows].cpu().numpy())
        assert (self.codes[:rows].cpu().numpy().reshape(-1) == rc).all(), "codes differ"
        if self.dequant:
            ref = quant_ref.dequantize(rc, rs)
            assert (self.out[:rows].cpu().numpy().reshape(-1) == ref).all(), "dequant differs"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        if self.dequant:
            h_in = [self.codes.cpu().pin_memory(), self.scales.cpu().pin_memory()]
            h_out = torch.empty(self.rows, 4096).pin_memory()
        else:
            h_in = [self.x.cpu().pin_memory()]
            h_out = [torch.empty(self.rows, 4096, dtype=torch.int8).pin_memory(),
                     torch.empty(self.rows * 64).pin_memory()]

        def one():
            d = [t.to(dev, non_blocking=True) for t in h_in]
            if self.dequant:
                h_out.copy_(cf.dequantize_int8(*d), non_blocking=True)
            else:
                c, s = cf.quantize_int8(d[0])
                h_out[0].copy_(c, non_blocking=True)
                h_out[1].copy_(s, non_blocking=True)

        h2d = sum(t.numel() * t.element_size() for t in h_in)
        d2h = (h_out.numel() * 4 if self.dequant
               else sum(t.numel() * t.element_size() for t in h_out))
        return timed_e2e(self, one, steps, h2d, d2h, "cuda_force_b200.(de)quantize_int8")

    def cpu_sample(self):
        x = self.x.cpu()
        from oracle import build_ref

        if build_ref.load():
            kind = "reference"
            if self.dequant:
                c, s = torch.ops.cudaforge_ref.quantize_int8(x)
                fn = lambda: torch.ops.cudaforge_ref.dequantize_int8(c, s)  # noqa: E731
            else:
                fn = lambda: torch.ops.cudaforge_ref.quantize_int8(x)  # noqa: E731
        else:
            from oracle import quant_ref

            kind = "port"
            fn = lambda: quant_ref.quantize(x.numpy())  # noqa: E731
        return fn, self.work_per_step, kind, "the full 4096x4096 tensor per call"


class Config1Dequant(Config1Quant):
    name = "config1_dequant_f32"
    dequant = True


def timed_e2e(wl, one_step, steps: int, h2d: int, d2h: int, api: str) -> dict:
    dev = wl.dist.device
    one_step()
    torch.cuda.synchronize(dev)
    wl.dist.barrier()
    t0 = time.perf_counter()
    for _ in range(steps):
        one_step()
    torch.cuda.synchronize(dev)
    wl.dist.barrier()
    elapsed = wl.dist.max(time.perf_counter() - t0)
    total = wl.dist.sum(wl.work_per_step) * steps
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    return {"value": total / elapsed / scale, "unit": wl.unit, "h2d_bytes_per_step": int(h2d),
            "d2h_bytes_per_step": int(d2h), "steps": steps, "api": api}


class LoraLinear:
    """benchmark config 3 (bf16 LoRA linear) and config 4 (W8 + LoRA, decode / prefill)."""

    name = "lora_bf16_8192x4096x4096"
    unit = "TFLOP/s"
    bound = "tensor"
    scaling = "weak"
    flush_l2 = True
    m, k, n, r, alpha = 8192, 4096, 4096, 16, 32.0
    int8 = False
    x_std, w_std, ab_std = 1.0, 0.02, 0.01
    main_kernel = "lora_gemm_kernel<256>"

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist
        self.metric = (f"{'W8+LoRA' if self.int8 else 'LoRA'} linear "
                       f"{'GB/s' if self.unit == 'GB/s' else 'TFLOP/s'} "
                       f"(x [{self.m},{self.k}], W [{self.n},{self.k}], r {self.r})")
        self.dtype = "bf16 x int8->bf16 (fp32 acc)" if self.int8 else "bf16 (fp32 acc)"
        self.kernel = self.main_kernel + " + down_proj_kernel (one call; PDL-overlapped)"

    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k + 2.0 * self.m * self.r * (self.k + self.n)

    def bytes(self) -> float:
        w = self.n * self.k * (1 + 4 / 64) if self.int8 else self.n * self.k * 2
        return w + 2 * (self.m * self.k + self.k * self.r + self.r * self.n + self.m * self.n)

    def config(self) -> dict:
        return {"workload": self.__doc__.strip().splitlines()[0] + f" [{self.name}]",
                "m": self.m, "k": self.k, "n": self.n, "rank": self.r, "alpha": self.alpha,
                "weight": "block-64 int8 codes + fp32 scales" if self.int8 else "bf16 [out, in]",
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "parallelism": f"{self.dist.world} independent replica(s)"}

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(3)
        self.x = (torch.randn(self.m, self.k, device=dev, generator=g) * self.x_std).to(torch.bfloat16)
        w = (torch.randn(self.n, self.k, device=dev, generator=g) * self.w_std).to(torch.bfloat16)
        self.a = (torch.randn(self.k, self.r, device=dev, generator=g) * self.ab_std).to(torch.bfloat16)
        self.b = (torch.randn(self.r, self.n, device=dev, generator=g) * self.ab_std).to(torch.bfloat16)
        self.scale = self.alpha / self.r
        self.work_per_step = self.bytes() if self.unit == "GB/s" else self.flops()
        if self.int8:
            self.codes, self.scales = quantize_weight(w, reference)
            self.w = None
        else:
            self.w = w
        if reference:
            return
        from cuda_force_b200 import _abi

        self.lib = _abi.load()
        self.y = torch.empty(self.m, self.n, dtype=torch.bfloat16, device=dev)
        self.ws_bytes = self.lib.cf_lora_linear_workspace_bytes(self.m, self.r)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.work_per_step = self.bytes() if self.unit == "GB/s" else self.flops()
        self.launches_per_step = 2

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        if self.int8:
            st = self.lib.cf_lora_linear_int8(
                self.x.data_ptr(), self.codes.data_ptr(), self.scales.data_ptr(), self.a.data_ptr(),
                _abi.CF_LAYOUT_REF, self.b.data_ptr(), _abi.CF_LAYOUT_REF, self.y.data_ptr(),
                self.m, self.k, self.n, self.r, self.scale, _abi.CF_DTYPE_BF16, self.ws.data_ptr(),
                self.ws_bytes, stream.cuda_stream)
        else:
            st = self.lib.cf_lora_linear(
                self.x.data_ptr(), self.w.data_ptr(), _abi.CF_LAYOUT_T, self.a.data_ptr(),
                _abi.CF_LAYOUT_REF, self.b.data_ptr(), _abi.CF_LAYOUT_REF, self.y.data_ptr(),
                self.m, self.k, self.n, self.r, self.scale, _abi.CF_DTYPE_BF16, self.ws.data_ptr(),
                self.ws_bytes, stream.cuda_stream)
        _abi.check(st, self.name)

    def _w_t(self):
        from oracle import linear_ref

        if self.int8:
            return linear_ref.dequantized_weight_t(self.codes, self.scales)
        return self.w.t()

    def verify(self) -> None:
        from oracle import linear_ref

        rows = torch.randperm(self.m, generator=torch.Generator().manual_seed(0))[:128]
        rows = rows.to(self.x.device)
        ref = linear_ref.lora_linear(self.x[rows], self._w_t(), self.a, self.b, self.scale)
        err = linear_ref.max_rel_error(self.y[rows], ref)
        assert err <= 2e-2, f"{self.name}: max relative error {err}"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hx = self.x.cpu().pin_memory()
        hy = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()

        def one():
            x = hx.to(dev, non_blocking=True)
            if self.int8:
                y = cf.lora_linear_int8(x, self.codes, self.scales, self.a, self.b, self.scale)
            else:
                y = cf.lora_linear(x, self.w.t(), self.a, self.b, self.scale)
            hy.copy_(y, non_blocking=True)

        return timed_e2e(self, one, steps, hx.numel() * 2, hy.numel() * 2,
                         "cuda_force_b200.lora_linear%s (weights resident, x in / y out)"
                         % ("_int8" if self.int8 else ""))

    def cpu_sample(self):
        from oracle import build_ref

        rows = min(self.m, 256)
        x = self.x[:rows].float().cpu()
        a, b = self.a.float().cpu(), self.b.float().cpu()
        have_ref = build_ref.load()
        kind = "reference" if have_ref else "port"
        if self.int8:
            codes, scales = self.codes.cpu(), self.scales.cpu()
        else:
            w_t = self.w.float().cpu().t().contiguous()

        def fn():
            if self.int8:
                wt = (torch.ops.cudaforge_ref.dequantize_int8(codes, scales) if have_ref
                      else codes.float()).reshape(self.n, self.k).t()
            else:
                wt = w_t
            if have_ref:
                torch.ops.cudaforge_ref.lora_linear(x, wt, a, b, self.scale)
            else:
                x @ wt + self.scale * ((x @ a) @ b)

        work = self.work_per_step * rows / self.m
        if self.unit == "GB/s":
            work = self.work_per_step  # decode: the sample is the whole problem
        return fn, work, kind, (f"{rows} of {self.m} rows in fp32 through the reference's CPU "
                                f"{'dequantize_int8 + ' if self.int8 else ''}lora_linear")


class W8Decode(LoraLinear):
    """benchmark config 4 decode: W8 + LoRA, x [32, 4096], W [11008, 4096] int8."""

    name = "w8_lora_decode_32x4096x11008"
    unit = "GB/s"
    bound = "hbm"
    m, k, n, r = 32, 4096, 11008, 16
    int8 = True
    main_kernel = "w8_decode_kernel<32> (split-K cluster of 3, 258 CTAs)"


class W8Prefill(LoraLinear):
    """benchmark config 4 prefill: W8 + LoRA, x [4096, 4096], W [11008, 4096] int8."""

    name = "w8_lora_prefill_4096x4096x11008"
    m, k, n, r = 4096, 4096, 11008, 16
    int8 = True
    main_kernel = "w8_wide_kernel (128 x 512 tiles, TMA-store epilogue)"


class NormW8Prefill(W8Prefill):
    """Residual add + RMSNorm folded into the config 4 prefill W8 + LoRA linear."""

    name = "rmsnorm_w8_lora_prefill_4096x4096x11008"
    main_kernel = ("norm statistics pass + w8_wide_kernel with the norm weight in the "
                   "conversion and the row scale in the epilogue")

    def __init__(self, dist: Dist, _layers: int = 0):
        super().__init__(dist, _layers)
        self.metric = ("residual + RMSNorm + W8+LoRA linear TFLOP/s of the linear "
                       "(x [4096,4096], W [11008,4096], r 16)")

    def config(self) -> dict:
        c = super().config()
        c["norm"] = "residual add + RMSNorm (eps 1e-6), weight 1 + N(0,0.1), folded into the linear"
        return c

    def setup(self, reference: bool = False) -> None:
        super().setup(reference)
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(13)
        self.res = torch.randn(self.m, self.k, device=dev, generator=g).to(torch.bfloat16)
        self.nw = (1 + 0.1 * torch.randn(self.k, device=dev, generator=g)).to(torch.bfloat16)
        if reference:
            return
        self.res_out = torch.empty_like(self.x)
        self.nws_bytes = self.lib.cf_rmsnorm_lora_linear_int8_workspace_bytes(self.m, self.k, self.r)
        self.nws = torch.empty(self.nws_bytes, dtype=torch.uint8, device=dev)
        self.launches_per_step = 4

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        _abi.check(self.lib.cf_rmsnorm_lora_linear_int8(
            self.x.data_ptr(), self.res.data_ptr(), self.nw.data_ptr(), 1e-6,
            self.codes.data_ptr(), self.scales.data_ptr(), self.a.data_ptr(), _abi.CF_LAYOUT_REF,
            self.b.data_ptr(), _abi.CF_LAYOUT_REF, self.y.data_ptr(), self.res_out.data_ptr(),
            self.m, self.k, self.n, self.r, self.scale, _abi.CF_DTYPE_BF16, self.nws.data_ptr(),
            self.nws_bytes, stream.cuda_stream), self.name)

    def verify(self) -> None:
        from oracle import linear_ref, norm_ref

        rows = torch.randperm(self.m, generator=torch.Generator().manual_seed(0))[:128]
        normed, summed = norm_ref.fused_residual_rmsnorm(self.x[rows.to(self.x.device)],
                                                         self.res[rows.to(self.x.device)],
                                                         self.nw, 1e-6)
        ref = linear_ref.lora_linear(normed, self._w_t(), self.a, self.b, self.scale)
        err = linear_ref.max_rel_error(self.y[rows.to(self.y.device)], ref)
        assert err <= 2e-2, f"{self.name}: max relative error {err}"
        assert torch.equal(self.res_out[rows.to(self.x.device)].cpu(), summed)

    def extra_record(self, steps: int, flush) -> dict:
        """The unfused route timed the same way: the norm kernel writes the normalised
        rows, then the plain W8 linear reads them."""
        from cuda_force_b200 import _abi

        normed = torch.empty_like(self.x)
        stream = torch.cuda.current_stream(self.dist.device)

        def unfused():
            _abi.check(self.lib.cf_fused_residual_rmsnorm(
                self.x.data_ptr(), self.res.data_ptr(), self.nw.data_ptr(), _abi.CF_DTYPE_BF16,
                normed.data_ptr(), self.res_out.data_ptr(), self.m, self.k, 1e-6,
                _abi.CF_DTYPE_BF16, stream.cuda_stream), "norm")
            _abi.check(self.lib.cf_lora_linear_int8(
                normed.data_ptr(), self.codes.data_ptr(), self.scales.data_ptr(),
                self.a.data_ptr(), _abi.CF_LAYOUT_REF, self.b.data_ptr(), _abi.CF_LAYOUT_REF,
                self.y.data_ptr(), self.m, self.k, self.n, self.r, self.scale,
                _abi.CF_DTYPE_BF16, self.ws.data_ptr(), self.ws_bytes, stream.cuda_stream), "lin")

        for _ in range(3):
            unfused()
        times = []
        for i in range(steps):
            if flush is not None:
                flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            unfused()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.mean(times)
        return {"unfused_ms_per_step": round(ms, 5),
                "unfused_tflops": round(self.work_per_step / ms / 1e9, 1),
                "how": "cf_fused_residual_rmsnorm (normalised rows written) then "
                       "cf_lora_linear_int8, same flush and CUDA events"}

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hx, hr = self.x.cpu().pin_memory(), self.res.cpu().pin_memory()
        hy = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()

        def one():
            y, _ = cf.rmsnorm_lora_linear_int8(hx.to(dev, non_blocking=True),
                                               hr.to(dev, non_blocking=True), self.nw,
                                               self.codes, self.scales, self.a, self.b,
                                               self.scale, 1e-6)
            hy.copy_(y, non_blocking=True)

        return timed_e2e(self, one, steps, 2 * hx.numel() * 2, hy.numel() * 2,
                         "cuda_force_b200.rmsnorm_lora_linear_int8 (x, residual in / y out)")

    def cpu_sample(self):
        fn, work, kind, sample = super().cpu_sample()
        return fn, work, kind, sample + " (norm not included)"


class LoraF32(LoraLinear):
    """fp32 LoRA linear (the reference's own CUDA dtype), benchmark config 3 shapes."""

    name = "lora_f32_8192x4096x4096"
    main_kernel = "lora_f32_kernel (three tf32 products)"
    # tf32 runs at half the bf16 rate and each fp32 multiply-add is three tf32 products.
    peak_divisor = 6
    peak_divisor_reason = "tf32 = bf16 / 2, three tf32 products per fp32 product"

    def __init__(self, dist: Dist, _layers: int = 0):
        super().__init__(dist, _layers)
        self.metric = (f"LoRA linear fp32 TFLOP/s (x [{self.m},{self.k}], W [{self.n},{self.k}], "
                       f"r {self.r})")
        self.dtype = "fp32 (three tf32 tensor-core products, fp32 accumulate)"

    def bytes(self) -> float:
        return 4 * (self.n * self.k + self.m * self.k + self.k * self.r + self.r * self.n
                    + self.m * self.n)

    def config(self) -> dict:
        c = super().config()
        c["weight"] = "fp32 [out, in] (passed as W.t(), K-major)"
        return c

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(3)
        self.x = torch.randn(self.m, self.k, device=dev, generator=g) * self.x_std
        self.w = torch.randn(self.n, self.k, device=dev, generator=g) * self.w_std
        self.a = torch.randn(self.k, self.r, device=dev, generator=g) * self.ab_std
        self.b = torch.randn(self.r, self.n, device=dev, generator=g) * self.ab_std
        self.scale = self.alpha / self.r
        self.work_per_step = self.flops()
        if reference:
            return
        from cuda_force_b200 import _abi

        self.lib = _abi.load()
        self.y = torch.empty(self.m, self.n, dtype=torch.float32, device=dev)
        self.ws_bytes = self.lib.cf_lora_linear_workspace_bytes(self.m, self.r)
        self.ws = torch.empty(self.ws_bytes, dtype=torch.uint8, device=dev)
        self.work_per_step = self.flops()
        self.launches_per_step = 2

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        st = self.lib.cf_lora_linear(
            self.x.data_ptr(), self.w.data_ptr(), _abi.CF_LAYOUT_T, self.a.data_ptr(),
            _abi.CF_LAYOUT_REF, self.b.data_ptr(), _abi.CF_LAYOUT_REF, self.y.data_ptr(),
            self.m, self.k, self.n, self.r, self.scale, _abi.CF_DTYPE_F32, self.ws.data_ptr(),
            self.ws_bytes, stream.cuda_stream)
        _abi.check(st, self.name)

    def verify(self) -> None:
        rows = torch.randperm(self.m, generator=torch.Generator().manual_seed(0))[:128]
        rows = rows.to(self.x.device)
        x = self.x[rows].double()
        ref = x @ self.w.t().double() + self.scale * ((x @ self.a.double()) @ self.b.double())
        err = ((self.y[rows].double() - ref).abs().max() / ref.abs().max()).item()
        assert err <= 1e-4, f"{self.name}: max relative error {err}"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hx = self.x.cpu().pin_memory()
        hy = torch.empty(self.m, self.n, dtype=torch.float32).pin_memory()

        def one():
            x = hx.to(dev, non_blocking=True)
            y = cf.lora_linear(x, self.w.t(), self.a, self.b, self.scale)
            hy.copy_(y, non_blocking=True)

        return timed_e2e(self, one, steps, hx.numel() * 4, hy.numel() * 4,
                         "cuda_force_b200.lora_linear fp32 (weights resident, x in / y out)")


class MergeQuant:
    """LoRA merge + block-INT8 quantise (training/lora.py:95-111, then quantize_int8)."""

    name = "lora_merge_quant_11008x4096_r16"
    unit = "GB/s"
    bound = "hbm"
    scaling = "weak"
    flush_l2 = True
    n, k, r, scaling_factor = 11008, 4096, 16, 2.0
    kernel = "lora_merge_quant_kernel"
    dtype = "bf16 -> int8 codes + fp32 scales"
    metric = "LoRA merge + block-INT8 quantise GB/s (W [11008,4096] bf16, r 16)"

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist

    def bytes(self) -> float:
        return self.n * self.k * (2 + 1 + 4 / 64) + 2 * self.r * (self.n + self.k)

    def config(self) -> dict:
        return {"workload": self.__doc__.strip() + f" [{self.name}]", "out": self.n, "in": self.k,
                "rank": self.r, "scaling": self.scaling_factor,
                "layouts": "W [out, in], lora_a [rank, in], lora_b [out, rank] (module layouts)",
                "values": "W N(0,0.02), lora_a and lora_b N(0,0.05)",
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "parallelism": f"{self.dist.world} independent replica(s)"}

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(9)
        self.w = (torch.randn(self.n, self.k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.a = (torch.randn(self.r, self.k, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        self.b = (torch.randn(self.n, self.r, device=dev, generator=g) * 0.05).to(torch.bfloat16)
        self.work_per_step = self.bytes()
        if reference:
            return
        from cuda_force_b200 import _abi

        self.codes = torch.empty(self.n, self.k, dtype=torch.int8, device=dev)
        self.scales = torch.empty(self.n * self.k // 64, dtype=torch.float32, device=dev)
        self.lib = _abi.load()
        self.work_per_step = self.bytes()
        self.launches_per_step = 1

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        st = self.lib.cf_lora_merge_quantize_int8(
            self.w.data_ptr(), self.a.data_ptr(), self.b.data_ptr(), self.n, self.k, self.r,
            self.scaling_factor, _abi.CF_DTYPE_BF16, self.codes.data_ptr(),
            self.scales.data_ptr(), stream.cuda_stream)
        _abi.check(st, self.name)

    def verify(self) -> None:
        import cuda_force_b200 as cf

        merged = self.w + self.scaling_factor * (self.b @ self.a)
        ref_codes, ref_scales = cf.quantize_int8(merged)
        diff = (self.codes.int() - ref_codes.int()).abs()
        assert diff.max().item() <= 1 and (diff > 0).float().mean().item() <= 1e-3, self.name
        rel = ((self.scales - ref_scales).abs() / ref_scales).max().item()
        assert rel <= 2.0 ** -7, f"{self.name}: scale error {rel}"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hw = self.w.cpu().pin_memory()
        hc = torch.empty(self.n, self.k, dtype=torch.int8).pin_memory()
        hs = torch.empty(self.n * self.k // 64, dtype=torch.float32).pin_memory()

        def one():
            w = hw.to(dev, non_blocking=True)
            codes, scales = cf.lora_merge_quantize_int8(w, self.a, self.b, self.scaling_factor)
            hc.copy_(codes, non_blocking=True)
            hs.copy_(scales, non_blocking=True)

        return timed_e2e(self, one, steps, hw.numel() * 2, hc.numel() + hs.numel() * 4,
                         "cuda_force_b200.lora_merge_quantize_int8 (adapter resident, W in, "
                         "codes and scales out)")

    def cpu_sample(self):
        from oracle import build_ref

        rows = 512
        w, a, b = self.w[:rows].cpu(), self.a.cpu(), self.b[:rows].cpu()
        have_ref = build_ref.load()

        def fn():
            merged = w + self.scaling_factor * (b @ a)   # the module's merged_weight()
            if have_ref:
                torch.ops.cudaforge_ref.quantize_int8(merged)
            else:
                from oracle import quant_ref

                quant_ref.quantize(merged.float().numpy().reshape(-1))

        return (fn, self.work_per_step * rows / self.n, "reference" if have_ref else "port",
                f"{rows} of {self.n} rows: merged_weight() in bf16 then the reference's CPU "
                f"quantize_int8")


class ResidualRMSNorm:
    """Residual add + RMSNorm before a LLaMA-7B projection (fused_residual_rmsnorm)."""

    name = "residual_rmsnorm_16384x4096_bf16"
    unit = "GB/s"
    bound = "hbm"
    scaling = "weak"
    flush_l2 = True
    rows, cols, eps = 16384, 4096, 1e-6
    kernel = "residual_rmsnorm_vec_kernel<bf16, bf16, 2>"
    dtype = "bf16 (fp32 sum of squares)"
    metric = "residual add + RMSNorm GB/s (x, residual [16384,4096] bf16)"

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist

    def bytes(self) -> float:
        # x and residual read, normalised and residual_out written; weight once
        return self.rows * self.cols * 2 * 4 + self.cols * 2

    def config(self) -> dict:
        return {"workload": self.__doc__.strip() + f" [{self.name}]", "rows": self.rows,
                "cols": self.cols, "eps": self.eps,
                "values": "x, residual N(0,1); weight 1 + N(0,0.1)",
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "parallelism": f"{self.dist.world} independent replica(s)"}

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(11)
        shape = (self.rows, self.cols)
        self.x = torch.randn(shape, device=dev, generator=g).to(torch.bfloat16)
        self.r = torch.randn(shape, device=dev, generator=g).to(torch.bfloat16)
        self.w = (1 + 0.1 * torch.randn(self.cols, device=dev, generator=g)).to(torch.bfloat16)
        self.work_per_step = self.bytes()
        if reference:
            return
        from cuda_force_b200 import _abi

        self.out = torch.empty_like(self.x)
        self.summed = torch.empty_like(self.x)
        self.lib = _abi.load()
        self.work_per_step = self.bytes()
        self.launches_per_step = 1

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        st = self.lib.cf_fused_residual_rmsnorm(
            self.x.data_ptr(), self.r.data_ptr(), self.w.data_ptr(), _abi.CF_DTYPE_BF16,
            self.out.data_ptr(), self.summed.data_ptr(), self.rows, self.cols, self.eps,
            _abi.CF_DTYPE_BF16, stream.cuda_stream)
        _abi.check(st, self.name)

    def verify(self) -> None:
        summed = self.x + self.r
        assert torch.equal(self.summed, summed), f"{self.name}: residual_out differs"
        f = summed.float()
        ref = (f * torch.rsqrt(f.pow(2).mean(-1, keepdim=True) + self.eps) * self.w.float())
        err = ((self.out.float() - ref).abs() / ref.abs().clamp_min(1e-30)).max().item()
        assert err <= 2.0 ** -7, f"{self.name}: normalised error {err}"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hx, hr = self.x.cpu().pin_memory(), self.r.cpu().pin_memory()
        ho, hs = torch.empty_like(hx).pin_memory(), torch.empty_like(hx).pin_memory()

        def one():
            x = hx.to(dev, non_blocking=True)
            r = hr.to(dev, non_blocking=True)
            out, summed = cf.fused_residual_rmsnorm(x, r, self.w, self.eps)
            ho.copy_(out, non_blocking=True)
            hs.copy_(summed, non_blocking=True)

        return timed_e2e(self, one, steps, 2 * hx.numel() * 2, 2 * ho.numel() * 2,
                         "cuda_force_b200.fused_residual_rmsnorm (weight resident, x and "
                         "residual in, normalised and residual_out out)")

    def cpu_sample(self):
        from oracle import build_ref

        rows = 2048
        x, r, w = self.x[:rows].cpu(), self.r[:rows].cpu(), self.w.cpu()
        if build_ref.load():
            fn = lambda: torch.ops.cudaforge_ref.fused_residual_rmsnorm(x, r, w, self.eps)  # noqa: E731
            kind = "reference"
        else:
            from oracle import norm_ref

            fn = lambda: norm_ref.fused_residual_rmsnorm(x, r, w, self.eps)  # noqa: E731
            kind = "port"
        return (fn, self.work_per_step * rows / self.rows, kind,
                f"{rows} of {self.rows} rows through the reference's CPU fused_residual_rmsnorm")


class W8SwiGLU:
    """LLaMA MLP gate + up projections with block-INT8 weights and SwiGLU fused."""

    name = "w8_swiglu_4096x4096x11008"
    unit = "TFLOP/s"
    bound = "tensor"
    scaling = "weak"
    flush_l2 = True
    m, k, n = 4096, 4096, 11008
    kernel = "w8_swiglu_kernel (gate and up tiles per stage, silu(g) * u in the epilogue)"
    dtype = "bf16 x int8->bf16 (fp32 acc)"
    metric = "W8 gate+up+SwiGLU TFLOP/s (x [4096,4096], Wg and Wu [11008,4096] int8)"

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist

    def flops(self) -> float:
        return 2 * 2.0 * self.m * self.n * self.k

    def config(self) -> dict:
        return {"workload": self.__doc__.strip() + f" [{self.name}]", "m": self.m, "k": self.k,
                "n": self.n, "weights": "block-64 int8 codes + fp32 scales (gate, up)",
                "values": "x N(0,1), Wg and Wu N(0,0.02)",
                "l2": "flushed between steps (256 MiB write outside the timed events)",
                "parallelism": f"{self.dist.world} independent replica(s)"}

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(11)
        self.x = torch.randn(self.m, self.k, device=dev, generator=g).to(torch.bfloat16)
        wg = (torch.randn(self.n, self.k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        wu = (torch.randn(self.n, self.k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        self.gc, self.gs = quantize_weight(wg, reference)
        self.uc, self.us = quantize_weight(wu, reference)
        del wg, wu
        self.work_per_step = self.flops()
        if reference:
            return
        from cuda_force_b200 import _abi

        self.y = torch.empty(self.m, self.n, dtype=torch.bfloat16, device=dev)
        self.lib = _abi.load()
        self.work_per_step = self.flops()
        self.launches_per_step = 1

    def step(self, stream) -> None:
        from cuda_force_b200 import _abi

        st = self.lib.cf_w8_swiglu_int8(
            self.x.data_ptr(), self.gc.data_ptr(), self.gs.data_ptr(), self.uc.data_ptr(),
            self.us.data_ptr(), self.y.data_ptr(), self.m, self.k, self.n, _abi.CF_DTYPE_BF16,
            stream.cuda_stream)
        _abi.check(st, self.name)

    def extra_record(self, steps: int, flush) -> dict:
        """The unfused route timed the same way: the gate and the up projection as two
        W8 linears (a zero rank-16 adapter, the smallest the entry point takes), then
        torch's silu(g) * u."""
        from cuda_force_b200 import _abi

        dev = self.dist.device
        r = 16
        a = torch.zeros(self.k, r, dtype=torch.bfloat16, device=dev)
        b = torch.zeros(r, self.n, dtype=torch.bfloat16, device=dev)
        g = torch.empty(self.m, self.n, dtype=torch.bfloat16, device=dev)
        u = torch.empty_like(g)
        ws_bytes = self.lib.cf_lora_linear_workspace_bytes(self.m, r)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=dev)
        stream = torch.cuda.current_stream(dev)

        def unfused():
            for codes, scales, out in ((self.gc, self.gs, g), (self.uc, self.us, u)):
                _abi.check(self.lib.cf_lora_linear_int8(
                    self.x.data_ptr(), codes.data_ptr(), scales.data_ptr(), a.data_ptr(),
                    _abi.CF_LAYOUT_REF, b.data_ptr(), _abi.CF_LAYOUT_REF, out.data_ptr(),
                    self.m, self.k, self.n, r, 1.0, _abi.CF_DTYPE_BF16, ws.data_ptr(), ws_bytes,
                    stream.cuda_stream), "w8 projection")
            torch.mul(torch.nn.functional.silu(g), u, out=self.y)

        for _ in range(3):
            unfused()
        times = []
        for i in range(steps):
            if flush is not None:
                flush.fill_(i & 0xFF)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            unfused()
            e1.record(stream)
            e1.synchronize()
            times.append(e0.elapsed_time(e1))
        ms = statistics.mean(times)
        return {"unfused_ms_per_step": round(ms, 5),
                "unfused_tflops": round(self.work_per_step / ms / 1e9, 1),
                "how": "two cf_lora_linear_int8 calls (zero rank-16 adapter) then torch "
                       "silu(g) * u, same flush and CUDA events"}

    def verify(self) -> None:
        from oracle import linear_ref

        rows = torch.randperm(self.m, generator=torch.Generator().manual_seed(0))[:64]
        rows = rows.to(self.x.device)
        xf = self.x[rows].float()
        g = (xf @ linear_ref.dequantized_weight_t(self.gc, self.gs).to(xf.device)).bfloat16().float()
        u = (xf @ linear_ref.dequantized_weight_t(self.uc, self.us).to(xf.device)).bfloat16().float()
        ref = g / (1.0 + torch.exp(-g)) * u
        err = ((self.y[rows].float() - ref).abs().max() / ref.abs().max()).item()
        assert err <= 2e-2, f"{self.name}: max relative error {err}"

    def e2e(self, steps: int) -> dict:
        import cuda_force_b200 as cf

        dev = self.dist.device
        hx = self.x.cpu().pin_memory()
        hy = torch.empty(self.m, self.n, dtype=torch.bfloat16).pin_memory()

        def one():
            x = hx.to(dev, non_blocking=True)
            hy.copy_(cf.w8_swiglu_int8(x, self.gc, self.gs, self.uc, self.us), non_blocking=True)

        return timed_e2e(self, one, steps, hx.numel() * 2, hy.numel() * 2,
                         "cuda_force_b200.w8_swiglu_int8 (weights resident, x in / h out)")

    def cpu_sample(self):
        from oracle import build_ref

        rows = 64
        x = self.x[:rows].float().cpu()
        gc, gs, uc, us = self.gc.cpu(), self.gs.cpu(), self.uc.cpu(), self.us.cpu()
        have_ref = build_ref.load()

        def fn():
            if have_ref:
                wg = torch.ops.cudaforge_ref.dequantize_int8(gc, gs).reshape(self.n, self.k)
                wu = torch.ops.cudaforge_ref.dequantize_int8(uc, us).reshape(self.n, self.k)
                torch.ops.cudaforge_ref.swiglu(x @ wg.t(), x @ wu.t())
            else:
                g, u = x @ gc.float().t(), x @ uc.float().t()
                g / (1.0 + torch.exp(-g)) * u

        return (fn, self.work_per_step * rows / self.m, "reference" if have_ref else "port",
                f"{rows} of {self.m} rows: the reference's CPU dequantize_int8, x @ W.T and "
                f"swiglu")


def _multicast_ok(dist: Dist) -> bool:
    if not torch.cuda.is_available():
        return False
    from cuda_force_b200.sharding import FusedGatherLinear

    return FusedGatherLinear.has_multicast(dist.device)


class W8ColumnSharded:
    """benchmark config 5: column-sharded W8 + LoRA on a Llama-70B MLP shape + NCCL all-gather."""

    name = "w8_lora_70b_colshard_16384x8192x28672"
    unit = "TFLOP/s"
    bound = "tensor"
    scaling = "strong"
    flush_l2 = False
    m, k, n, r, alpha = 16384, 8192, 28672, 64, 128.0
    chunks = 4
    kernel = "w8_wide_kernel + down_proj_kernel<64> per row chunk, NCCL all-gather overlapped"
    dtype = "bf16 x int8->bf16 (fp32 acc)"
    metric = ("W8+LoRA column-sharded linear TFLOP/s (x [16384,8192], W [28672,8192] int8, "
              "r 64, all-gather of y)")
    comm = None  # None = the --comm flag; "fused", "ce" or "nccl"

    def __init__(self, dist: Dist, _layers: int = 0):
        self.dist = dist
        if self.comm is None:
            self.comm = COMM_MODE
        if self.comm == "auto" and dist.world == 1:
            self.comm = "fused"
        # At N > 1 "auto" is resolved in setup(): asking whether the GPUs support
        # multicast imports this package, which the reference arm must not.

    def flops(self) -> float:
        return 2.0 * self.m * self.n * self.k + 2.0 * self.m * self.r * (self.k + self.n)

    def config(self) -> dict:
        g = self.dist.world
        return {"workload": self.__doc__.strip(), "m": self.m, "k": self.k, "n": self.n,
                "rank": self.r, "alpha": self.alpha, "weight": "block-64 int8 codes + fp32 scales",
                "parallelism": f"column-sharded over {g} GPU(s): {self.n // g} output features "
                               f"per rank, x and A replicated; all-gather of y "
                               + ("fused into the GEMM epilogue: multimem stores through y's "
                                  "NVLink multicast address where the GPUs support it, else "
                                  "TMA stores into every rank's copy" if self.comm == "auto"
                                  and g > 1 else
                                  "fused into the GEMM epilogue: each 16-byte piece written "
                                  "once through y's NVLink multicast address (multimem.st), "
                                  "the switch delivers it to every rank" if self.comm == "mc"
                                  and g > 1 else
                                  "fused into the GEMM epilogue (TMA stores into every rank's "
                                  "symmetric-memory y)" if self.comm == "fused" and g > 1 else
                                  "by the copy engines, one stream per peer, each row group "
                                  "pushed as soon as the kernel's counter says it is done "
                                  "(symmetric-memory y)" if self.comm == "ce" and g > 1 else
                                  f"by NCCL in {self.chunks} row chunks on a side stream"),
                "output": ("y [M, N] on every rank" if self.comm != "nccl" and g > 1 else
                           "rank-major [G, rows, N/G] per chunk (no relayout copy)"),
                "values": "x N(0,1), W N(0,0.015), A and B N(0,0.01); W and B seeded per rank",
                "l2": "inputs larger than L2 (x 268 MB, W codes 235 MB / G)"}

    def _slice(self, rank: int, reference: bool = False):
        """The int8 codes, scales and B columns that ``rank`` owns, regenerated from its seed."""
        from_cols = self.n // self.dist.world
        dev = self.dist.device
        gw = torch.Generator(device=dev).manual_seed(7 + rank)
        w = (torch.randn(from_cols, self.k, device=dev, generator=gw) * 0.015).to(torch.bfloat16)
        codes, scales = quantize_weight(w, reference)
        del w
        b = (torch.randn(self.r, from_cols, device=dev, generator=gw) * 0.01).to(torch.bfloat16)
        return codes, scales, b

    def setup(self, reference: bool = False) -> None:
        dev = self.dist.device
        g = torch.Generator(device=dev).manual_seed(5)
        self.x = torch.randn(self.m, self.k, device=dev, generator=g).to(torch.bfloat16)
        self.a = (torch.randn(self.k, self.r, device=dev, generator=g) * 0.01).to(torch.bfloat16)
        if reference:
            self.x = self.x[:256].cpu()  # the CPU sample's rows only
        self.codes, self.scales, self.b = self._slice(self.dist.rank, reference)
        self.scale = self.alpha / self.r
        self.work_per_step = self.flops() / self.dist.world
        self.last = None
        self.fused = None
        if reference:
            return
        if self.comm == "auto":
            self.comm = "mc" if _multicast_ok(self.dist) else "fused"
        if self.dist.world > 1 and self.comm in ("fused", "ce", "mc"):
            from cuda_force_b200.sharding import FusedGatherLinear

            mode = {"ce": "ce", "mc": "mc"}.get(self.comm, "kernel")
            self.fused = FusedGatherLinear(self.m, self.n, torch.bfloat16, dev, mode=mode)
            self.kernel = ("w8_wide_kernel with the all-gather fused into the epilogue "
                           "(multimem stores to y's NVLink multicast address) + "
                           "down_proj_kernel<64>" if mode == "mc" else
                           "w8_wide_kernel with the all-gather fused into the epilogue "
                           "(TMA stores to every rank over NVLink) + down_proj_kernel<64>"
                           if mode == "kernel" else
                           "w8_wide_kernel (local y + row-group counters) + down_proj_kernel<64>; "
                           "copy engines push finished row groups to the peers")
            self.launches_per_step = 2
        else:
            self.launches_per_step = 2 * (self.chunks if self.dist.world > 1 else 1)

    def step(self, stream) -> None:
        from cuda_force_b200.sharding import sharded_lora_linear_int8

        if self.fused is not None:
            self.last = self.fused(self.x, self.codes, self.scales, self.a, self.b, self.scale)
            return
        group = self.dist.pg.group.WORLD if self.dist.pg is not None else None
        self.last = sharded_lora_linear_int8(self.x, self.codes, self.scales, self.a, self.b,
                                             self.scale, group=group, chunks=self.chunks)

    def gathered_rows(self, rows: list[int], owner: int) -> torch.Tensor:
        """Rows ``rows`` of the columns that rank ``owner`` computed, read from this rank's
        gathered output."""
        width = self.codes.shape[0]
        if self.fused is not None:
            return self.last[rows][:, owner * width:(owner + 1) * width]
        chunk_rows = -(-self.m // (self.chunks if self.dist.world > 1 else 1))
        return torch.stack([self.last[r // chunk_rows][owner, r % chunk_rows] for r in rows])

    def verify(self) -> None:
        """Every rank's column slice of the gathered output, on sampled rows, against the oracle:
        the peer slices (written over NVLink by the peers) are rebuilt here from their seeds."""
        from oracle import linear_ref

        torch.cuda.synchronize(self.dist.device)
        rows = torch.randperm(self.m, generator=torch.Generator().manual_seed(0))[:64].tolist()
        rows.sort()
        for owner in range(self.dist.world):
            if owner == self.dist.rank:
                codes, scales, b = self.codes, self.scales, self.b
            else:
                codes, scales, b = self._slice(owner)
            w_t = linear_ref.dequantized_weight_t(codes, scales)
            ref = linear_ref.lora_linear(self.x[rows], w_t, self.a, b, self.scale)
            err = linear_ref.max_rel_error(self.gathered_rows(rows, owner), ref)
            if not err <= 2e-2:
                raise SystemExit(f"{self.name}: rank {self.dist.rank}'s copy of rank {owner}'s "
                                 f"columns has max relative error {err}")

    def exchange_record(self, step_ms: float, steps: int) -> dict | None:
        """Bytes each rank sends per step, and the exchange time: the step minus the same
        rank's compute alone (this rank's columns into a local y, no exchange)."""
        if self.dist.world < 2:
            return None
        from cuda_force_b200 import _abi

        lib = _abi.load()
        width = self.codes.shape[0]
        y = torch.empty(self.m, width, dtype=torch.bfloat16, device=self.dist.device)
        ws_bytes = lib.cf_lora_linear_workspace_bytes(self.m, self.r)
        ws = torch.empty(ws_bytes, dtype=torch.uint8, device=self.dist.device)
        stream = torch.cuda.current_stream(self.dist.device)

        def local():
            _abi.check(lib.cf_lora_linear_int8(
                self.x.data_ptr(), self.codes.data_ptr(), self.scales.data_ptr(),
                self.a.data_ptr(), _abi.CF_LAYOUT_REF, self.b.data_ptr(), _abi.CF_LAYOUT_REF,
                y.data_ptr(), self.m, self.k, width, self.r, self.scale, _abi.CF_DTYPE_BF16,
                ws.data_ptr(), ws_bytes, stream.cuda_stream), "local compute")

        for _ in range(3):
            local()
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(self.dist.device)
        start.record(stream)
        for _ in range(steps):
            local()
        end.record(stream)
        end.synchronize()
        local_ms = self.dist.max(start.elapsed_time(end) / steps)
        sent = (self.dist.world - 1) * self.m * width * 2
        exchange_ms = max(step_ms - local_ms, 0.0)
        return {"bytes_sent_per_rank_per_step": sent,
                "step_ms": round(step_ms, 4),
                "compute_only_ms": round(local_ms, 4),
                "exchange_ms": round(exchange_ms, 4),
                "compute_only_tflops_per_gpu": round(self.work_per_step / local_ms / 1e9, 1),
                "nvlink_gbs_over_step": round(sent / step_ms / 1e6, 1),
                "exchange_efficiency": round(local_ms / step_ms, 4),
                "how": "compute_only = this rank's columns into a local y (same kernels, no "
                       "exchange), CUDA events, max over ranks; exchange = step - compute_only"}

    def e2e(self, steps: int) -> dict:
        dev = self.dist.device
        hx = self.x.cpu().pin_memory()
        hy = torch.empty(self.dist.world * self.m * self.codes.shape[0],
                         dtype=torch.bfloat16).pin_memory()

        def one():
            from cuda_force_b200.sharding import sharded_lora_linear_int8

            x = hx.to(dev, non_blocking=True)
            group = self.dist.pg.group.WORLD if self.dist.pg is not None else None
            if self.fused is not None:
                parts = [self.fused(x, self.codes, self.scales, self.a, self.b, self.scale)]
            else:
                parts = sharded_lora_linear_int8(x, self.codes, self.scales, self.a, self.b,
                                                 self.scale, group=group, chunks=self.chunks)
            off = 0
            for part in parts:
                n = part.numel()
                hy[off:off + n].copy_(part.reshape(-1), non_blocking=True)
                off += n

        return timed_e2e(self, one, steps, hx.numel() * 2, hy.numel() * 2,
                         "cuda_force_b200.sharding.sharded_lora_linear_int8 "
                         "(weights resident, x in, gathered y out)")

    def cpu_sample(self):
        from oracle import build_ref

        rows = 256
        have_ref = build_ref.load()
        x = self.x[:rows].float().cpu()
        a, b = self.a.float().cpu(), self.b.float().cpu()
        codes, scales = self.codes.cpu(), self.scales.cpu()
        width = codes.shape[0]

        def fn():
            wt = (torch.ops.cudaforge_ref.dequantize_int8(codes, scales) if have_ref
                  else codes.float()).reshape(width, self.k).t()
            if have_ref:
                torch.ops.cudaforge_ref.lora_linear(x, wt, a, b, self.scale)
            else:
                x @ wt + self.scale * ((x @ a) @ b)

        work = (2.0 * rows * width * self.k + 2.0 * rows * self.r * (self.k + width))
        return fn, work, "reference" if have_ref else "port", (
            f"{rows} rows x this rank's {width} output features in fp32 through the reference's "
            f"CPU dequantize_int8 + lora_linear (W dequantised every call)")


class W8ColumnShardedNccl(W8ColumnSharded):
    """benchmark config 5 with the output all-gather done by NCCL (the unfused baseline)."""

    name = "w8_lora_70b_colshard_16384x8192x28672_nccl"
    comm = "nccl"


class W8ColumnShardedPeer(W8ColumnSharded):
    """benchmark config 5 with the all-gather fused as one TMA store per peer (no multicast)."""

    name = "w8_lora_70b_colshard_16384x8192x28672_peer"
    comm = "fused"


WORKLOADS = {w.name: w for w in (LlamaStackQuant, Config1Quant, Config1Dequant, LoraLinear,
                                W8Decode, W8Prefill, W8ColumnSharded, W8ColumnShardedNccl,
                                W8ColumnShardedPeer, NormW8Prefill,
                                LoraF32, MergeQuant,
                                W8SwiGLU, ResidualRMSNorm)}


# ---------------------------------------------------------------------------
# Runs
# ---------------------------------------------------------------------------
def time_cpu(fn, min_seconds: float = 10.0, max_calls: int = 50) -> float:
    fn()  # warm-up
    times = []
    t_start = time.perf_counter()
    while len(times) < 3 or (time.perf_counter() - t_start < min_seconds and len(times) < max_calls):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    return statistics.median(times)


# The benchmark configs reported beside the headline (config 2) in the same JSON line.
PER_CONFIG = ["config1_quant_f32", "config1_dequant_f32", "lora_bf16_8192x4096x4096",
              "w8_lora_decode_32x4096x11008", "w8_lora_prefill_4096x4096x11008",
              "w8_lora_70b_colshard_16384x8192x28672"]
PER_CONFIG_MULTI = ["w8_lora_70b_colshard_16384x8192x28672_nccl",
                    "w8_lora_70b_colshard_16384x8192x28672_peer"]


def measure(wl, args, dist: Dist, cpu_seconds: float) -> dict:
    """Times K steps of one workload under the bench rules and returns its report fields."""
    torch.cuda.set_device(dist.device)
    wl.setup()
    stream = torch.cuda.Stream(device=dist.device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=dist.device) if wl.flush_l2 else None
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            wl.step(stream)
    torch.cuda.synchronize(dist.device)
    wl.verify()

    starts = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    ends = [torch.cuda.Event(enable_timing=True) for _ in range(args.steps)]
    dist.barrier()
    torch.cuda.synchronize(dist.device)
    with ClockSampler(dist.local_rank) as clocks:
        with torch.cuda.stream(stream):
            for i in range(args.steps):
                if flush is not None:
                    flush.fill_(i & 0xFF)  # evict L2 outside the timed events
                starts[i].record(stream)
                wl.step(stream)
                ends[i].record(stream)
        torch.cuda.synchronize(dist.device)
    dist.barrier()
    per_step_ms = [s.elapsed_time(e) for s, e in zip(starts, ends)]
    if flush is not None:
        total_ms = sum(per_step_ms)
    else:
        total_ms = starts[0].elapsed_time(ends[-1])
    total_ms = dist.max(total_ms)
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    work_all = dist.sum(wl.work_per_step) * args.steps
    value = work_all / (total_ms * 1e-3) / scale

    peaks, peak_src = load_peaks()
    step_ms = statistics.mean(per_step_ms)
    achieved = wl.work_per_step / (step_ms * 1e-3) / scale
    if wl.bound == "hbm":
        peak, peak_key, peak_unit = peaks["hbm_gbs"], "hbm_gbs", "GB/s"
    else:
        peak, peak_key, peak_unit = peaks["bf16_tflops"], "bf16_tflops (burst)", "TFLOP/s"
    divisor = getattr(wl, "peak_divisor", 1)
    if divisor != 1:
        peak = round(peak / divisor, 2)
        peak_key += f" / {divisor} ({wl.peak_divisor_reason})"
    traffic_info = load_traffic().get(wl.name)
    traffic = traffic_info.get("dram_bytes_per_step") if traffic_info else None

    copy_ref = size_matched_copy(wl.work_per_step, dist.device, flush) if wl.bound == "hbm" else None
    exchange = (wl.exchange_record(total_ms / args.steps, args.steps)
                if hasattr(wl, "exchange_record") else None)
    extra = wl.extra_record(args.steps, flush) if hasattr(wl, "extra_record") else None
    e2e = wl.e2e(max(1, min(args.steps, args.e2e_steps)))

    cpu = None
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        fn, work, kind, sample = wl.cpu_sample()
        t = time_cpu(fn, min_seconds=cpu_seconds)
        cpu = {"value": work / t / scale, "unit": wl.unit, "cores": torch.get_num_threads(),
               "cpu_model": cpu_model(), "kind": kind,
               "sample": sample + f", median of >=3 calls over ~{cpu_seconds:g} s"}
    result = {
        "metric": wl.metric,
        "value": round(value, 3),
        "unit": wl.unit,
        "ms_per_step": round(total_ms / args.steps, 5),
        "scaling": wl.scaling,
        "dtype": wl.dtype,
        "config": wl.config(),
        "roofline": {
            "bound": wl.bound,
            "kernel": wl.kernel,
            "achieved": round(achieved, 2),
            "peak": peak,
            "peak_source": f"{peak_src} {peak_key}",
            "unit": peak_unit,
            "frac": round(achieved / peak, 4),
            "traffic": traffic,
            "algorithmic_per_launch_step": wl.work_per_step,
            "launches_per_step": wl.launches_per_step,
            **({"size_matched_copy": copy_ref} if copy_ref else {}),
        },
        "e2e": e2e,
        "gpu_launches": wl.launches_per_step * args.steps,
        "clocks": clocks.summary(),
        "cpu_baseline": cpu,
    }
    if dist.world > 1:
        result["per_gpu"] = round(value / dist.world, 3)
    if exchange is not None:
        result["comm"] = exchange
    if extra is not None:
        result["unfused"] = extra
    return result


def release(wl) -> None:
    """Drops a workload's device tensors before the next one is set up."""
    for name in list(vars(wl)):
        if name != "dist":
            delattr(wl, name)
    if torch.cuda.is_available():
        torch.cuda.synchronize()
        torch.cuda.empty_cache()


def run_ours(args, dist: Dist) -> dict | None:
    wl = WORKLOADS[args.workload](dist, args.layers)
    head = measure(wl, args, dist, cpu_seconds=10.0)
    release(wl)
    result = {
        "metric": head.pop("metric"),
        "value": head.pop("value"),
        "unit": head.pop("unit"),
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": head.pop("ms_per_step"),
        "higher_is_better": True,
        "scaling": head.pop("scaling"),
        "vs_baseline": None,
        "dtype": head.pop("dtype"),
        "data": "synthetic (seeded on device)",
        **head,
    }
    if args.per_config and args.workload == LlamaStackQuant.name:
        names = PER_CONFIG + (PER_CONFIG_MULTI if dist.world > 1 else [])
        per = {}
        launches = result["gpu_launches"]
        for name in names:
            sub = WORKLOADS[name](dist, args.layers)
            per[name] = measure(sub, args, dist, cpu_seconds=3.0)
            launches += per[name]["gpu_launches"]
            release(sub)
        result["per_config"] = per
        result["gpu_launches_all_configs"] = launches
    return result if dist.rank == 0 else None


def reference_entry(wl, args, dist: Dist, steps: int, warmup: int) -> dict:
    """The reference's own CPU implementation of one workload, timed on this host's cores."""
    wl.setup(reference=True)
    fn, work, kind, sample = wl.cpu_sample()
    scale = 1e9 if wl.unit == "GB/s" else 1e12
    for _ in range(max(1, warmup)):
        fn()
    times = []
    for _ in range(steps):
        t0 = time.perf_counter()
        fn()
        times.append(time.perf_counter() - t0)
    value = work * len(times) / sum(times) / scale
    return {
        "metric": wl.metric,
        "value": round(value, 6),
        "unit": wl.unit,
        "ms_per_step": round(1e3 * sum(times) / len(times), 3),
        "steps": steps,
        "config": {**wl.config(), "reference_sample": sample},
        "cpu_baseline": {"value": round(value, 6), "unit": wl.unit,
                         "cores": torch.get_num_threads(), "cpu_model": cpu_model(),
                         "kind": kind, "sample": sample},
        "e2e": {"value": round(value, 6), "unit": wl.unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_reference(args, dist: Dist) -> dict | None:
    """The reference's own CPU implementation of the path on this host's cores.

    Nothing of this package is imported on this arm: inputs come from torch's
    generators and the reference's compiled CPU operators quantise the weights.
    """
    if dist.rank != 0:
        return None
    torch.cuda.set_device(dist.device)
    torch.set_num_threads(os.cpu_count() or 1)
    wl = WORKLOADS[args.workload](dist, args.layers)
    head = reference_entry(wl, args, dist, args.steps, args.warmup)
    result = {
        "impl": "reference",
        "metric": head["metric"],
        "value": head["value"],
        "unit": head["unit"],
        "n_gpus": dist.world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": head["ms_per_step"],
        "higher_is_better": True,
        "scaling": wl.scaling,
        "vs_baseline": None,
        "dtype": wl.dtype,
        "data": "synthetic (seeded)",
        "config": head["config"],
        "cpu_baseline": head["cpu_baseline"],
        "e2e": head["e2e"],
    }
    if args.per_config and args.workload == LlamaStackQuant.name:
        # bounded samples: a few calls each, so the whole arm stays within minutes
        per = {}
        for name in PER_CONFIG:
            sub = WORKLOADS[name](dist, args.layers)
            per[name] = reference_entry(sub, args, dist, min(args.steps, 5), 1)
            release(sub)
        result["per_config"] = per
    assert "cuda_force_b200" not in sys.modules, "the reference arm imported this package"
    return result


def main() -> None:
    parser = argparse.ArgumentParser()
    parser.add_argument("--gpus", type=int, default=1)
    parser.add_argument("--steps", type=int, default=100)
    parser.add_argument("--warmup", type=int, default=5)
    parser.add_argument("--impl", choices=["ours", "reference"], default="ours")
    parser.add_argument("--workload", choices=sorted(WORKLOADS), default=LlamaStackQuant.name)
    parser.add_argument("--e2e-steps", type=int, default=2)
    parser.add_argument("--layers", type=int, default=LLAMA7B_LAYERS,
                        help="stack depth (default 32 = benchmark config 2; smaller only "
                             "for profiling captures)")
    parser.add_argument("--no-cpu-baseline", action="store_true")
    parser.add_argument("--no-per-config", dest="per_config", action="store_false",
                        help="report the headline workload only (default: the headline config "
                             "2 line also carries configs 1, 3, 4 and 5 under per_config)")
    parser.add_argument("--elements", type=int, default=0,
                        help="config 1 workloads: tensor size (default 4096*4096)")
    parser.add_argument("--comm", choices=["auto", "mc", "fused", "ce", "nccl"], default="auto",
                        help="config 5 all-gather: multimem stores through y's NVLink "
                             "multicast address, one TMA store per peer, the copy engines "
                             "behind per-row-group counters, or NCCL (auto: mc where the "
                             "GPUs support multicast, else fused)")
    args = parser.parse_args()
    global COMM_MODE, CONFIG1_ROWS
    COMM_MODE = args.comm
    if args.elements:
        if args.elements % 4096:
            parser.error("--elements must be a multiple of 4096")
        CONFIG1_ROWS = args.elements // 4096
    if args.warmup < 3:
        parser.error("--warmup must be >= 3")

    dist = Dist(args.gpus)
    try:
        result = run_reference(args, dist) if args.impl == "reference" else run_ours(args, dist)
    finally:
        dist.close()
    if result is not None:
        print(json.dumps(result), flush=True)


if __name__ == "__main__":
    main()
