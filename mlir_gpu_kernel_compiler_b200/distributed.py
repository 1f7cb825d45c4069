"""Row-sharded execution of a plan across the GPUs of one node.

The large-batch programs are row-independent: every output row depends only on
the same input row and on the (replicated) weights.  So the multi-GPU strategy
is plain data parallelism over rows: one process per GPU, rank ``p`` of ``N``
owns rows ``[p*R/N, (p+1)*R/N)``, compiles the same program for ``M = R/N`` rows
and runs it with no cross-GPU traffic in the step.  When the caller wants the
whole result on one device there are two ways:

* ``gather_rows``: after the step, an NCCL all-gather of the row shards over NVLink
  (``all_gather_into_tensor``), or ``all_gather`` on backends without it (gloo, used
  by the CPU tests);
* ``RowsOnRoot``: no collective at all.  The root rank exports its full-size output
  buffer (CUDA IPC through the runtime's C ABI), every other rank maps it, and each
  rank's program is launched with its own rows of that buffer as the output, so the
  last kernel's epilogue stores its tiles straight into the root's HBM over NVLink
  while the rest of the GEMM is still running.  The only host-visible ordering
  needed is the usual one: a rank's rows are complete when its stream is.
"""
from __future__ import annotations

from typing import Optional

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


class RowsOnRoot:
    """A ``[total, ...]`` tensor on the root rank whose row shards every rank writes directly.

    Collective: every rank of ``group`` constructs it together (root allocates and exports
    its buffer, the others map it).  ``dest`` is what a rank passes as its program's output:
    the root's own tensor slice on the root, a raw peer address elsewhere (programs built
    with ``peer_outputs=True``).  ``full`` is the whole tensor on the root (None elsewhere);
    it holds every rank's rows once all ranks' streams have finished the step (synchronise,
    then ``dist.barrier``).  ``close`` is collective as well: peers unmap first, and the root
    keeps its buffer until they have.
    """

    def __init__(self, shape: tuple, dtype: torch.dtype, device: torch.device, root: int = 0, group=None):
        from . import runtime as rt

        self.group, self.root = group, root
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        self.device = torch.device(device)
        self.shape, self.dtype = tuple(shape), dtype
        self.lo, self.hi = shard_bounds(self.shape[0], self.world, self.rank)
        row_bytes = torch.empty((), dtype=dtype).element_size()
        for d in self.shape[1:]:
            row_bytes *= d
        self.full: Optional[torch.Tensor] = None
        self._mapped: Optional[tuple[int, int]] = None
        cuda = self.device.type == "cuda"
        dev_index = self.device.index if self.device.index is not None else (torch.cuda.current_device() if cuda else 0)
        self._dev = dev_index
        # Failures are collective: every rank learns of one and raises at the same point, so
        # no rank is left waiting in a later collective.
        msg: list = [None]
        if self.rank == root:
            self.full = torch.empty(self.shape, dtype=dtype, device=self.device)
            if cuda:
                torch.cuda.synchronize(self.device)
            try:
                msg[0] = ("ok",) + rt.ipc_export(self.full.data_ptr(), dev_index)
            except Exception as ex:  # noqa: BLE001 - reported to every rank below
                msg[0] = ("error", f"rank {root} could not export its buffer: {ex}")
        dist.broadcast_object_list(msg, src=dist.get_global_rank(group, root) if group else root, group=group)
        err = msg[0][1] if msg[0][0] == "error" else ""
        if self.rank == root:
            self.dest = self.full[self.lo:self.hi]
        elif not err:
            _, handle, offset = msg[0]
            try:
                base = rt.ipc_open(handle, offset, dev_index)
                self._mapped = (base, offset)
                self.dest = base + self.lo * row_bytes
            except Exception as ex:  # noqa: BLE001
                err = f"rank {self.rank} could not map rank {root}'s buffer: {ex}"
        ok = torch.tensor([0 if err else 1], dtype=torch.int32, device=self.device)
        dist.all_reduce(ok, op=dist.ReduceOp.MIN, group=group)
        if not int(ok.item()):
            if self._mapped is not None:
                rt.ipc_close(self._mapped[0], self._mapped[1], dev_index)
                self._mapped = None
            self.full = None
            raise RuntimeError(err or "another rank could not set up the shared output buffer")

    def close(self) -> None:
        from . import runtime as rt

        if self.device.type == "cuda":
            torch.cuda.synchronize(self.device)
        if self._mapped is not None:
            base, offset = self._mapped
            rt.ipc_close(base, offset, self._dev)
            self._mapped = None
        dist.barrier(group=self.group)       # the root frees its buffer only after every peer unmapped it
        self.full = None
