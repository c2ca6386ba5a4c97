"""Batch sharding of a compiled W8A8 program over ranks (one process per GPU).

Every op on the path is independent per image/row, so a global batch is split into contiguous
shards, each rank runs its shard on its own GPU with replicated weights, and the only exchange is
the final gather of the per-rank outputs (torch.distributed over NCCL on GPUs, or gloo on CPUs).
"""
from __future__ import annotations

import numpy as np


def shard_bounds(n: int, rank: int, world: int) -> tuple[int, int]:
    """[start, stop) of rank's contiguous shard of n rows; the first n % world ranks get one more."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, extra = divmod(int(n), int(world))
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_rows(local: np.ndarray, n_global: int, world: int, group=None) -> np.ndarray:
    """All-gather each rank's output rows (in rank order) into the full [n_global, ...] array on
    every rank.  Shards are padded to the largest shard for the collective and trimmed after."""
    import torch
    import torch.distributed as dist
    sizes = [b - a for a, b in (shard_bounds(n_global, r, world) for r in range(world))]
    width = max(sizes)
    buf = np.zeros((width,) + local.shape[1:], local.dtype)
    buf[: local.shape[0]] = local
    backend = dist.get_backend(group)
    device = "cuda" if backend == "nccl" else "cpu"
    t = torch.from_numpy(buf).to(device)
    parts = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(parts, t, group=group)
    return np.concatenate([p.cpu().numpy()[:s] for p, s in zip(parts, sizes)], axis=0)
