"""Multi-GPU layouts of the hot path (one process per GPU, torch.distributed).

* Layer-sharded quantisation: independent layers are dealt
  round-robin to ranks; no communication.
* Column-sharded W8 + LoRA linear: rank g owns output
  features [g*N/G, (g+1)*N/G) — its rows of the int8 weight and their scales,
  and the matching columns of the adapter's B — while x and A are replicated.
  Each rank computes its slice y_g = x W_g^T + scale (x A) B_g, and the slices
  are assembled with an all-gather over NVLink. The gather runs on a side
  stream per row chunk so chunk i is exchanged while chunk i+1 is computed.

The reference has no multi-GPU path for these ops (its only NCCL use is a DDP
training example, examples/distributed_train.py:82); the sharding follows the
north-star configuration, not reference code.
"""

from __future__ import annotations

from collections.abc import Callable

import torch
import torch.distributed as dist


def layer_shard(n_layers: int, rank: int, world: int) -> list[int]:
    """Layers quantised by `rank`: l with l % world == rank."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} for world size {world}")
    return list(range(rank, n_layers, world))


def column_slice(n: int, rank: int, world: int) -> slice:
    """Output features owned by `rank` (N must split evenly)."""
    if n % world != 0:
        raise ValueError(f"{n} output features do not split over {world} ranks")
    width = n // world
    return slice(rank * width, (rank + 1) * width)


def row_chunks(m: int, chunks: int) -> list[slice]:
    """Row ranges of the pipelined compute / gather (the last one may be short)."""
    step = -(-m // chunks)
    return [slice(i, min(m, i + step)) for i in range(0, m, step)]


def assemble(gathered: list[torch.Tensor]) -> torch.Tensor:
    """Row chunks of rank-major slices, each [G, rows, N/G] -> y [M, N] (a copy)."""
    parts = [g.permute(1, 0, 2).reshape(g.shape[1], g.shape[0] * g.shape[2]) for g in gathered]
    return torch.cat(parts, dim=0)


def sharded_lora_linear_int8(
    x: torch.Tensor,
    w_codes: torch.Tensor,
    w_scales: torch.Tensor,
    lora_a: torch.Tensor,
    lora_b: torch.Tensor,
    scale: float,
    group: dist.ProcessGroup | None = None,
    chunks: int = 4,
    local_op: Callable[..., torch.Tensor] | None = None,
) -> list[torch.Tensor]:
    """Column-sharded ``lora_linear_int8``.

    ``w_codes`` / ``w_scales`` / ``lora_b`` are this rank's slices ([N/G, K],
    [N/G*K/64], [r, N/G]); ``x`` [M, K] and ``lora_a`` [K, r] are replicated.
    Returns, per row chunk, the gathered rank-major slices [G, rows, N/G] —
    the all-gather writes them in place, so no relayout copy is paid; use
    :func:`assemble` for y [M, N]. ``local_op`` computes one rank's slice
    (default: the sm_100a kernel, ``cuda_force_b200.lora_linear_int8``).
    """
    if local_op is None:
        from cuda_force_b200.ops import lora_linear_int8 as local_op
    world = dist.get_world_size(group) if dist.is_initialized() else 1
    m = x.shape[0]
    width = w_codes.shape[0]
    if world == 1:
        y = local_op(x, w_codes, w_scales, lora_a, lora_b, scale)
        return [y.view(1, m, width)]
    on_cuda = x.is_cuda
    comm = torch.cuda.Stream(device=x.device) if on_cuda else None
    result = []
    for rows in row_chunks(m, chunks):
        y = local_op(x[rows], w_codes, w_scales, lora_a, lora_b, scale)
        flat = torch.empty(world * y.shape[0], width, dtype=y.dtype, device=y.device)
        if on_cuda:
            ready = torch.cuda.Event()
            ready.record()
            comm.wait_event(ready)
            with torch.cuda.stream(comm):
                dist.all_gather_into_tensor(flat, y, group=group)
            y.record_stream(comm)
            flat.record_stream(comm)
        else:
            dist.all_gather_into_tensor(flat, y, group=group)
        result.append(flat.view(world, y.shape[0], width))
    if on_cuda:
        torch.cuda.current_stream(x.device).wait_stream(comm)
    return result
