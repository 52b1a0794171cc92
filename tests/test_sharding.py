"""Host-side multi-GPU logic on CPU ranks (gloo, world size 2).

The column-sharded W8 + LoRA linear is run by two gloo processes with a CPU
stand-in for the per-rank kernel (the dequantise-then-linear composition of the
oracle); the gathered, reassembled output must equal the unsharded product.
Layer and column bookkeeping are checked directly.
"""

from __future__ import annotations

import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cuda_force_b200 import sharding


def free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def cpu_local_op(x, codes, scales, a, b, scale):
    from oracle import linear_ref

    return linear_ref.lora_linear_int8(x, codes, scales, a, b, scale).to(x.dtype)


def make_problem(m=48, k=128, n=96, r=16):
    from oracle import quant_ref

    g = torch.Generator().manual_seed(0)
    x = torch.randn(m, k, generator=g)
    w = torch.randn(n, k, generator=g) * 0.02
    a = torch.randn(k, r, generator=g) * 0.05
    b = torch.randn(r, n, generator=g) * 0.05
    codes, scales = quant_ref.quantize(w.numpy())
    return x, torch.from_numpy(codes).reshape(n, k), torch.from_numpy(scales), a, b


def _worker(rank: int, world: int, port: int, result_path: str) -> None:
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        x, codes, scales, a, b = make_problem()
        n, k = codes.shape
        cols = sharding.column_slice(n, rank, world)
        blocks_per_row = k // 64
        my_codes = codes[cols].contiguous()
        my_scales = scales.reshape(n, blocks_per_row)[cols].reshape(-1).contiguous()
        my_b = b[:, cols].contiguous()
        out = sharding.sharded_lora_linear_int8(x, my_codes, my_scales, a, my_b, 2.0, chunks=3,
                                                local_op=cpu_local_op)
        if rank == 0:
            torch.save(sharding.assemble(out), result_path)
    finally:
        dist.destroy_process_group()


def test_column_sharded_linear_gathers_the_full_product(tmp_path):
    world = 2
    path = str(tmp_path / "y.pt")
    mp.spawn(_worker, args=(world, free_port(), path), nprocs=world, join=True)
    y = torch.load(path)
    x, codes, scales, a, b = make_problem()
    ref = cpu_local_op(x, codes, scales, a, b, 2.0)
    torch.testing.assert_close(y, ref, rtol=1e-5, atol=1e-5)


def test_layer_shard_covers_every_layer_once():
    for world in (1, 2, 4, 8):
        seen = sorted(l for r in range(world) for l in sharding.layer_shard(32, r, world))
        assert seen == list(range(32))
        assert all(len(sharding.layer_shard(32, r, world)) == 32 // world for r in range(world))


def test_column_slices_partition_the_outputs():
    n = 28672
    for world in (1, 2, 4, 8):
        slices = [sharding.column_slice(n, r, world) for r in range(world)]
        assert slices[0].start == 0 and slices[-1].stop == n
        assert all(s.stop == t.start for s, t in zip(slices, slices[1:]))
    with pytest.raises(ValueError):
        sharding.column_slice(100, 0, 3)


def test_row_chunks_and_assemble():
    assert sharding.row_chunks(10, 3) == [slice(0, 4), slice(4, 8), slice(8, 10)]
    g = torch.arange(2 * 3 * 4).reshape(2, 3, 4)
    full = sharding.assemble([g[:, :2], g[:, 2:]])
    assert full.shape == (3, 8)
    assert torch.equal(full[:, :4], g[0]) and torch.equal(full[:, 4:], g[1])
