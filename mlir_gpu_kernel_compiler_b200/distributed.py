"""Row-sharded execution of a plan across the GPUs of one node.

The large-batch programs are row-independent: every output row depends only on
the same input row and on the (replicated) weights.  So the multi-GPU strategy
is plain data parallelism over rows: one process per GPU, rank ``p`` of ``N``
owns rows ``[p*R/N, (p+1)*R/N)``, compiles the same program for ``M = R/N`` rows
and runs it with no cross-GPU traffic in the step.  Only when the caller wants
the whole result on one device does a collective run: ``gather_rows`` is an
NCCL all-gather of the row shards over NVLink (``all_gather_into_tensor``), or
``all_gather`` on backends without it (gloo, used by the CPU tests).
"""
from __future__ import annotations

import torch
import torch.distributed as dist


def shard_bounds(total: int, world: int, rank: int) -> tuple[int, int]:
    """Rows owned by ``rank``: contiguous, as even as possible (earlier ranks take the remainder)."""
    if world < 1 or not 0 <= rank < world:
        raise ValueError(f"bad rank {rank} of {world}")
    base, rem = divmod(total, world)
    lo = rank * base + min(rank, rem)
    return lo, lo + base + (1 if rank < rem else 0)


def shard(t: torch.Tensor, world: int, rank: int) -> torch.Tensor:
    lo, hi = shard_bounds(t.shape[0], world, rank)
    return t[lo:hi]


def gather_rows(local: torch.Tensor, group=None) -> torch.Tensor:
    """Concatenate every rank's row shard (equal shard sizes) on every rank."""
    world = dist.get_world_size(group)
    out = torch.empty((local.shape[0] * world,) + tuple(local.shape[1:]), dtype=local.dtype, device=local.device)
    if dist.get_backend(group) == "nccl":
        dist.all_gather_into_tensor(out, local.contiguous(), group=group)
    else:
        parts = list(out.chunk(world, dim=0))
        dist.all_gather(parts, local.contiguous(), group=group)
    return out


def max_over_ranks(value: float, device=None, group=None) -> float:
    """The slowest rank's time (multi-GPU numbers are max over ranks)."""
    if not dist.is_initialized() or dist.get_world_size(group) == 1:
        return value
    t = torch.tensor([value], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX, group=group)
    return float(t.item())
