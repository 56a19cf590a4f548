"""Batch-sharded inference across GPUs (one process per GPU).

The reference trains with DDP over NCCL (experiments/imagenet100/train_vit.py:211-215,
556-566) and reduces per-epoch metrics with ``all_reduce`` (:469-471).  Inference
needs no collective on the data path: images are independent, so each rank runs
its own slice of the global batch; the only exchanges are one gather of the
logits to rank 0 and one MAX-reduction of the per-rank device time.

Everything here works with any ``torch.distributed`` backend: NCCL between
GPUs, gloo for the CPU tests of the bookkeeping.
"""

from __future__ import annotations

import datetime
import os
from dataclasses import dataclass

import torch
import torch.distributed as dist


@dataclass(frozen=True)
class RankContext:
    rank: int
    world: int
    local_rank: int
    device: torch.device

    @property
    def is_main(self) -> bool:
        return self.rank == 0


def init_from_env(backend: str = "nccl", timeout_s: float = 120.0) -> RankContext:
    """Join the process group torchrun describes (RANK / WORLD_SIZE / LOCAL_RANK,
    MASTER_ADDR / MASTER_PORT); a single process needs no group."""
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if backend == "nccl":
        device = torch.device("cuda", local)
        torch.cuda.set_device(device)
    else:
        device = torch.device("cpu")
    if world > 1 and not dist.is_initialized():
        kwargs = {"device_id": device} if backend == "nccl" else {}
        dist.init_process_group(backend, timeout=datetime.timedelta(seconds=timeout_s), **kwargs)
    return RankContext(rank, world, local, device)


def shard_bounds(global_batch: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous, balanced slice [start, stop) of the global batch for `rank`
    (the first global_batch % world ranks take one extra item)."""
    if global_batch < 0 or world < 1 or not 0 <= rank < world:
        raise ValueError("need global_batch >= 0, world >= 1 and 0 <= rank < world")
    base, extra = divmod(global_batch, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


def gather_to_main(local: torch.Tensor, ctx: RankContext, global_batch: int) -> torch.Tensor | None:
    """Concatenate every rank's slice (in rank order) on rank 0; other ranks get None.

    Slices may differ by one row; they are padded to the largest slice for the
    collective and trimmed afterwards."""
    if ctx.world == 1:
        return local
    sizes = [shard_bounds(global_batch, ctx.world, r) for r in range(ctx.world)]
    rows = max(stop - start for start, stop in sizes)
    padded = local.new_zeros((rows,) + tuple(local.shape[1:]))
    padded[: local.shape[0]] = local
    parts = [torch.empty_like(padded) for _ in range(ctx.world)] if ctx.is_main else None
    dist.gather(padded, parts, dst=0)
    if not ctx.is_main:
        return None
    return torch.cat([part[: stop - start] for part, (start, stop) in zip(parts, sizes)])


def max_over_ranks(value: float, ctx: RankContext) -> float:
    """The slowest rank's value (device times are reported as the max)."""
    if ctx.world == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=ctx.device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def barrier(ctx: RankContext) -> None:
    if ctx.world > 1:
        dist.barrier()


def shutdown(ctx: RankContext) -> None:
    if ctx.world > 1 and dist.is_initialized():
        dist.destroy_process_group()
