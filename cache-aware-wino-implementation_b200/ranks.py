"""Process-per-GPU plumbing for batch-split runs (no collective on the data path).

The batch N of a layer is split across the ranks (shard(): N / world images
each, contiguous); each rank convolves its shard with its own copy of the
transformed weights.  The only collectives are bookkeeping outside the timed
region: a barrier, the max of per-rank device times, and gathers of sampled
output images to rank 0 for verification.  This replaces the reference's
thread fan-out of tile tasks (multicore_scheduler.py:33-50).  Backend: NCCL
for CUDA tensors, gloo for CPU (tests).
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from datetime import timedelta


@dataclass(frozen=True)
class Rank:
    rank: int
    world: int
    local: int

    @property
    def is_root(self) -> bool:
        return self.rank == 0


def from_env() -> Rank:
    """RANK / WORLD_SIZE / LOCAL_RANK as set by torchrun (single process: 0/1/0)."""
    return Rank(int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
                int(os.environ.get("LOCAL_RANK", "0")))


def shard(global_n: int, r: Rank) -> tuple[int, int]:
    """(first image, image count) of this rank's contiguous shard; shards differ
    by at most one image and cover [0, global_n) exactly once."""
    base, extra = divmod(global_n, r.world)
    first = r.rank * base + min(r.rank, extra)
    return first, base + (1 if r.rank < extra else 0)


def init(r: Rank, backend: str, timeout_s: float = 120.0, device=None) -> None:
    """Joins the process group (a no-op for a single rank).  A short timeout
    turns a rank that never joins, or dies between steps, into an error on the
    others instead of a hang."""
    if r.world <= 1:
        return
    import torch.distributed as dist

    kw = {"timeout": timedelta(seconds=timeout_s)}
    if device is not None and backend == "nccl":
        kw["device_id"] = device
    dist.init_process_group(backend, rank=r.rank, world_size=r.world, **kw)


def barrier(r: Rank) -> None:
    if r.world > 1:
        import torch.distributed as dist

        dist.barrier()


def max_over_ranks(value: float, r: Rank, device=None) -> float:
    if r.world <= 1:
        return float(value)
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_floats(value: float, r: Rank, device=None) -> list[float]:
    if r.world <= 1:
        return [float(value)]
    import torch
    import torch.distributed as dist

    t = torch.tensor([float(value)], dtype=torch.float64, device=device)
    out = [torch.zeros_like(t) for _ in range(r.world)]
    dist.all_gather(out, t)
    return [float(x.item()) for x in out]


def gather_tensor(t, r: Rank) -> list:
    """Every rank's copy of `t` (same shape and dtype on every rank), in rank order.
    Used outside timed regions only, to bring sampled outputs to rank 0 for
    verification; NCCL for CUDA tensors, gloo for CPU tensors."""
    if r.world <= 1:
        return [t]
    import torch
    import torch.distributed as dist

    out = [torch.empty_like(t) for _ in range(r.world)]
    dist.all_gather(out, t.contiguous())
    return out


def finish(r: Rank) -> None:
    if r.world > 1:
        import torch.distributed as dist

        dist.barrier()
        dist.destroy_process_group()
