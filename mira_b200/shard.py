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


class _DeviceArray:
    """A device allocation seen through __cuda_array_interface__ (torch wraps it without a copy)."""

    def __init__(self, address: int, shape: tuple, typestr: str = "<f4"):
        self.__cuda_array_interface__ = {"shape": tuple(int(d) for d in shape), "typestr": typestr,
                                         "data": (int(address), False), "version": 2}


class DeviceGather:
    """The final gather of a batch-sharded program, on the GPUs.  Called after a step's kernels are
    queued (CudaExecutable.run_many's `gather` hook), it gathers every rank's output rows, read in
    place from the executable's device output buffer, into one device buffer on rank `dst` over
    NCCL.  The collective is ordered on the library's own stream (torch's NCCL work waits for that
    stream and the stream waits for it), so no host round trip or sync sits between the kernels,
    the gather and rank `dst`'s single device-to-host copy of the whole global batch.  Every rank
    runs the same program at the same batch (equal shards)."""

    def __init__(self, exe, world: int, rank: int, dst: int = 0, group=None):
        import ctypes as C

        import torch

        from . import _lib
        from .device import DeviceBuffer
        outs = [(v, buf, nb) for v, buf, nb in exe.plan.outputs]
        if len(outs) != 1:
            raise ValueError("the device gather handles programs with one output")
        (v, buf, nb), = outs
        shape = tuple(v.type.shape)
        exe.device.activate()
        self.value, self.dst, self.group, self.world = v, int(dst), group, int(world)
        self.local = torch.as_tensor(_DeviceArray(buf.ptr, shape), device="cuda")
        s = C.c_void_p()
        _lib.call("mira_cuda_get_stream", C.byref(s))
        self.stream = torch.cuda.ExternalStream(int(s.value or 0))
        gshape = (world * shape[0],) + shape[1:]
        if rank == self.dst:
            self.buf = DeviceBuffer(world * nb)
            self.parts = [torch.as_tensor(_DeviceArray(self.buf.ptr + r * nb, shape), device="cuda")
                          for r in range(world)]
            self.outputs = [(v, self.buf, world * nb, gshape)]
        else:
            self.buf, self.parts, self.outputs = None, None, []
        self.global_shape = gshape

    def __call__(self) -> None:
        import torch
        import torch.distributed as dist
        with torch.cuda.stream(self.stream):
            dist.gather(self.local, self.parts, dst=self.dst, group=self.group)
