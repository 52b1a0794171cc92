"""bench.py's workload definitions, checked on the CPU.

The roofline fractions and values are algorithmic work ÷ time, so the work per
step must be the figure the benchmark configs define: bytes for the HBM-bound
workloads, FLOPs for the tensor-bound ones. Each workload must also carry every
field the JSON line reports.
"""

from __future__ import annotations

import pytest

import bench


@pytest.fixture(scope="module")
def dist():
    return bench.Dist(1)


def test_llama_stack_bytes(dist):
    wl = bench.LlamaStackQuant(dist)
    assert wl.elems_per_layer * bench.LLAMA7B_LAYERS == 6_476_005_376
    assert bench.BYTES_PER_ELEM_BF16_QUANT * wl.elems_per_layer * 32 == 19_832_766_464


def test_config1_bytes():
    assert (4 + 1 + 4 / 64) * bench.CONFIG1_ROWS * 4096 == 84_934_656


def test_linear_work(dist):
    assert bench.LoraLinear(dist).flops() == 277_025_390_592
    assert bench.W8Decode(dist).bytes() == 49_356_800
    assert bench.W8Prefill(dist).flops() == 371_346_898_944
    # 2MNK + 2·M·r·(K+N) for the 70B MLP shape: 7.774 TFLOP per call in total
    assert bench.W8ColumnSharded(dist).flops() == pytest.approx(7.7739e12, rel=1e-4)


def test_new_workload_bytes(dist):
    assert bench.ResidualRMSNorm(dist).bytes() == 16384 * 4096 * 8 + 4096 * 2
    assert bench.MergeQuant(dist).bytes() == 11008 * 4096 * (2 + 1 + 4 / 64) + 2 * 16 * (11008 + 4096)


@pytest.mark.parametrize("name", sorted(bench.WORKLOADS))
def test_every_workload_reports_the_contract_fields(name, dist):
    wl = bench.WORKLOADS[name](dist, bench.LLAMA7B_LAYERS)
    assert wl.name == name
    assert wl.unit in ("GB/s", "TFLOP/s")
    assert wl.bound in ("hbm", "tensor")
    assert (wl.bound == "hbm") == (wl.unit == "GB/s")
    assert wl.scaling in ("weak", "strong")
    assert isinstance(wl.flush_l2, bool)
    for field in ("metric", "dtype", "kernel"):
        assert isinstance(getattr(wl, field), str) and getattr(wl, field)
    cfg = wl.config()
    assert isinstance(cfg.get("workload"), str) and cfg["workload"]
    assert "l2" in cfg or not wl.flush_l2


def test_reference_arm_imports_nothing_of_the_package(tmp_path):
    # bench.py --impl reference must time the reference's CPU path only: no module of this
    # package may load in that process (its native libraries would show as loaded). Run on
    # the CPU here, with the device redirected to the host.
    import json
    import subprocess
    import sys

    script = tmp_path / "ref_arm.py"
    script.write_text(
        "import sys, torch\n"
        f"sys.path.insert(0, {str(bench.ROOT)!r})\n"
        "sys.argv = ['bench.py', '--impl', 'reference', '--steps', '2', '--warmup', '3',\n"
        "            '--workload', 'config1_quant_f32']\n"
        "import bench\n"
        "bench.Dist.device = property(lambda self: torch.device('cpu'))\n"
        "torch.cuda.set_device = lambda d: None\n"
        "bench.main()\n"
        "assert 'cuda_force_b200' not in sys.modules\n")
    out = subprocess.run([sys.executable, str(script)], capture_output=True, text=True,
                         timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert line["impl"] == "reference"
    assert line["cpu_baseline"]["cores"] >= 1 and line["cpu_baseline"]["cpu_model"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0


def test_headline_line_lists_every_benchmark_config():
    # configs 1 (quantise, dequantise), 3, 4 (decode, prefill) and 5 ride in the config 2 line
    assert set(bench.PER_CONFIG) == {
        "config1_quant_f32", "config1_dequant_f32", "lora_bf16_8192x4096x4096",
        "w8_lora_decode_32x4096x11008", "w8_lora_prefill_4096x4096x11008",
        "w8_lora_70b_colshard_16384x8192x28672"}
    assert all(name in bench.WORKLOADS for name in bench.PER_CONFIG + bench.PER_CONFIG_MULTI)


def test_config5_workloads_at_two_ranks_import_nothing_until_set_up(tmp_path):
    # The reference arm builds every per_config workload at N > 1 too; choosing the
    # multicast exchange (which asks this package about the GPUs) waits for setup().
    import subprocess
    import sys

    script = tmp_path / "two_ranks.py"
    script.write_text(
        "import sys\n"
        f"sys.path.insert(0, {str(bench.ROOT)!r})\n"
        "import bench\n"
        "class D:\n    world, rank, local_rank = 2, 0, 0\n"
        "for cls in (bench.W8ColumnSharded, bench.W8ColumnShardedNccl, bench.W8ColumnShardedPeer):\n"
        "    wl = cls(D())\n"
        "    wl.config()\n"
        "assert 'cuda_force_b200' not in sys.modules\n")
    out = subprocess.run([sys.executable, str(script)], capture_output=True, text=True, timeout=300)
    assert out.returncode == 0, out.stderr[-2000:]
