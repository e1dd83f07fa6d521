"""Work partitioning across the GPUs of one box (one process per GPU).

The CKKS path shards by independent units: the
feature-major token-shard ciphertexts, their complex pairs and the output
ciphertexts of a linear are independent through every linear, elementwise
op and bootstrap.  Each rank owns a contiguous block of units; the only data
exchange is an all-gather of ciphertext limb buffers at stage boundaries
(torch.distributed: NCCL over NVLink on GPUs, gloo on CPU for tests).
"""

from __future__ import annotations

import torch
import torch.distributed as dist


def shard_range(total: int, world: int, rank: int) -> range:
    """Units [start, stop) of `rank` when `total` units split over `world`
    ranks as evenly as possible (the first total % world ranks get one more)."""

    total, world, rank = int(total), int(world), int(rank)
    if world <= 0 or not 0 <= rank < world:
        raise ValueError(f"rank {rank} outside a world of {world}")
    base, extra = divmod(total, world)
    start = rank * base + min(rank, extra)
    return range(start, start + base + (1 if rank < extra else 0))


def world() -> tuple[int, int]:
    if dist.is_available() and dist.is_initialized():
        return dist.get_rank(), dist.get_world_size()
    return 0, 1


def max_over_ranks(value: float, device: torch.device | str = "cpu") -> float:
    """Maximum of a per-rank scalar (step time) over all ranks."""

    rank, size = world()
    if size == 1:
        return float(value)
    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_units(local: torch.Tensor, total: int) -> torch.Tensor:
    """All-gather every rank's block of units ([n_local, ...] limb buffers,
    n_local from shard_range) into the full [total, ...] tensor on every rank."""

    rank, size = world()
    if size == 1:
        return local
    counts = [len(shard_range(total, size, r)) for r in range(size)]
    if local.shape[0] != counts[rank]:
        raise ValueError(f"rank {rank} holds {local.shape[0]} units, expected {counts[rank]}")
    width = max(counts)
    shape = (width,) + tuple(local.shape[1:])
    padded = torch.zeros(shape, dtype=local.dtype, device=local.device)
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(size)]
    dist.all_gather(parts, padded)
    return torch.cat([p[:c] for p, c in zip(parts, counts)], dim=0)
