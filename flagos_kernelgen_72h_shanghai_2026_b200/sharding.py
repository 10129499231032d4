"""Row sharding of the operator over the GPUs of one node.

Rows (tokens) are independent, so a batch splits into contiguous row slabs,
one per rank, with gamma replicated and no exchange step: nothing crosses
NVLink on the data path. torch.distributed is used only around it — to align
ranks before a timed region and to take the maximum of per-rank device times
after it. The reference has no multi-device code; this is the runner for the
row-sharded benchmark shape (262144 x 7168 over 1/2/4/8 GPUs).
"""
from __future__ import annotations

import torch


def shard_rows(M: int, world: int, rank: int) -> tuple[int, int]:
    """[start, stop) of ``rank``'s contiguous slab: equal slabs, with the
    M % world remainder rows going one each to the last ranks."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of world {world}")
    base, rem = divmod(M, world)
    start = rank * base + max(0, rank - (world - rem))
    stop = start + base + (1 if rank >= world - rem else 0)
    return start, stop


def max_over_ranks(values: list[float], device: torch.device | str = "cpu") -> list[float]:
    """Element-wise maximum of per-rank values (e.g. device times) over the
    default process group; identity without one."""
    import torch.distributed as dist
    t = torch.tensor(values, dtype=torch.float64, device=device)
    if dist.is_available() and dist.is_initialized() and dist.get_world_size() > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return [float(v) for v in t.tolist()]


def gather_rows(local: torch.Tensor, M: int, device: torch.device | str = "cpu") -> torch.Tensor:
    """All-gather every rank's row slab into the full [M, ...] tensor (outside
    any timed region; used for parity checks of a sharded run)."""
    import torch.distributed as dist
    world = dist.get_world_size()
    sizes = [shard_rows(M, world, r) for r in range(world)]
    maxrows = max(b - a for a, b in sizes)
    pad = torch.zeros((maxrows,) + tuple(local.shape[1:]), dtype=local.dtype, device=device)
    pad[: local.shape[0]] = local.to(device)
    parts = [torch.empty_like(pad) for _ in range(world)]
    dist.all_gather(parts, pad)
    return torch.cat([p[: b - a] for p, (a, b) in zip(parts, sizes)], dim=0)
