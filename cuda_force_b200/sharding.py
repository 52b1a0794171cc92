"""Multi-GPU layouts of the hot path (one process per GPU, torch.distributed).

* Layer-sharded quantisation (benchmark config 2): independent layers are dealt
  round-robin to ranks; no communication.
* Column-sharded W8 + LoRA linear (benchmark config 5): rank g owns output
  features [g*N/G, (g+1)*N/G) — its rows of the int8 weight and their scales,
  and the matching columns of the adapter's B — while x and A are replicated.
  Each rank computes its slice y_g = x W_g^T + scale (x A) B_g, and the slices
  are assembled with an all-gather over NVLink. The gather runs on a side
  stream per row chunk so chunk i is exchanged while chunk i+1 is computed.

The reference has no multi-GPU path for these ops (its only NCCL use is a DDP
training example, examples/distributed_train.py:82); the sharding follows the
benchmark configuration, not reference code.
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


class FusedGatherLinear:
    """Column-sharded W8 + LoRA with the all-gather fused into the kernel.

    The output y [M, N] is a symmetric-memory buffer (one per GPU, mapped into
    every rank); each rank's kernel writes its own columns into all G copies
    over NVLink as its tiles complete (``cf_lora_linear_int8_allgather``: the
    epilogue TMA-stores each staged block to the local copy and every peer's),
    so the exchange overlaps the GEMM tile by tile and no relayout is needed.
    A device-side barrier after the launch orders the ranks before y is read.

    ``mode="mc"`` writes through the buffer's NVLink multicast address
    (``cf_lora_linear_int8_allgather_mc``): each 16-byte piece of this rank's
    columns leaves the GPU once and the switch delivers it to every rank's
    copy, instead of one store per peer. It needs multicast support
    (``has_multicast``).

    ``mode="ce"`` moves the exchange to the copy engines
    (``cf_lora_linear_int8_allgather_ce``): the kernel writes only the local
    copy of y and counts finished tiles per row group, and one copy stream per
    peer pushes each finished group over NVLink while the SMs compute the next.
    """

    def __init__(self, m: int, n: int, dtype: torch.dtype, device: torch.device,
                 group: dist.ProcessGroup | None = None, mode: str = "kernel"):
        if mode not in ("kernel", "ce", "mc"):
            raise ValueError(f"unknown exchange mode {mode!r}")
        self.mode = mode
        import torch.distributed._symmetric_memory as symm_mem

        self.group = group if group is not None else dist.group.WORLD
        self.world = dist.get_world_size(self.group)
        self.rank = dist.get_rank(self.group)
        self.y = symm_mem.empty(m, n, dtype=dtype, device=device)
        self.handle = symm_mem.rendezvous(self.y, self.group.group_name)
        peers = [self.handle.get_buffer(r, (m, n), dtype) for r in range(self.world)]
        self._peers = peers  # keep the views alive
        import ctypes

        self._dest = (ctypes.c_void_p * self.world)(*[t.data_ptr() for t in peers])
        self.m, self.n = m, n
        self.mc = 0
        if mode == "mc":
            if not self.has_multicast(device):
                raise RuntimeError("NVLink multicast is not available for this group")
            local = peers[self.rank].data_ptr()
            assert local == self.y.data_ptr()
            # the multicast mapping covers the allocation the way each rank's
            # unicast mapping does, so y sits at the same offset in both
            self.mc = self.handle.multicast_ptr + (local - self.handle.buffer_ptrs[self.rank])

    @staticmethod
    def has_multicast(device: torch.device) -> bool:
        from torch._C._distributed_c10d import _SymmetricMemory

        try:
            return bool(_SymmetricMemory.has_multicast_support(
                torch._C._autograd.DeviceType.CUDA, device.index))
        except Exception:  # noqa: BLE001 - treated as unsupported
            return False

    def __call__(self, x, w_codes, w_scales, lora_a, lora_b, scale: float) -> torch.Tensor:
        import ctypes

        from cuda_force_b200 import _abi

        lib = _abi.load()
        width, k = w_codes.shape
        m = x.shape[0]
        r = lora_a.shape[1]
        rp = 16 if r <= 16 else 32 if r <= 32 else 64
        if rp != r:
            raise ValueError("pad the adapter rank to 16, 32 or 64 first")
        a_layout = _abi.CF_LAYOUT_REF if lora_a.is_contiguous() else _abi.CF_LAYOUT_T
        b_layout = _abi.CF_LAYOUT_REF if lora_b.is_contiguous() else _abi.CF_LAYOUT_T
        dtype = _abi.CF_DTYPE_BF16 if x.dtype == torch.bfloat16 else _abi.CF_DTYPE_F16
        stream = ctypes.c_void_p(torch.cuda.current_stream(x.device).cuda_stream)
        p = lambda t: ctypes.c_void_p(t.data_ptr())  # noqa: E731
        if self.mode == "mc":
            ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
            _abi.check(lib.cf_lora_linear_int8_allgather_mc(
                p(x), p(w_codes), p(w_scales), p(lora_a), a_layout, p(lora_b), b_layout,
                p(self.y), ctypes.c_void_p(self.mc), self.n, self.rank * width, m, k, width, r,
                float(scale), dtype, p(ws), ws_bytes, stream), "cf_lora_linear_int8_allgather_mc")
        elif self.mode == "ce":
            ws_bytes = lib.cf_lora_linear_int8_allgather_ce_workspace_bytes(m, r)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
            _abi.check(lib.cf_lora_linear_int8_allgather_ce(
                p(x), p(w_codes), p(w_scales), p(lora_a), a_layout, p(lora_b), b_layout,
                self.world, self._dest, self.rank, self.n, self.rank * width, m, k, width, r,
                float(scale), dtype, p(ws), ws_bytes, stream), "cf_lora_linear_int8_allgather_ce")
        else:
            ws_bytes = lib.cf_lora_linear_workspace_bytes(m, r)
            ws = torch.empty(ws_bytes, dtype=torch.uint8, device=x.device)
            _abi.check(lib.cf_lora_linear_int8_allgather(
                p(x), p(w_codes), p(w_scales), p(lora_a), a_layout, p(lora_b), b_layout,
                self.world, self._dest, self.rank, self.n, self.rank * width, m, k, width, r,
                float(scale), dtype, p(ws), ws_bytes, stream), "cf_lora_linear_int8_allgather")
        self.handle.barrier()
        return self.y
