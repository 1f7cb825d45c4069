"""Arena planning for the B200 backend.

The arena layout is part of the plan contract: the reference's planner
(``tensorjit/passes/memory_planner.py:69-119``) places every intermediate that
does not escape to the caller at a 64-byte aligned offset in one arena, using
interval liveness over the straight-line kernel list and a best-fit search over
free ranges.  The B200 runtime allocates that arena once per program in HBM and
binds kernel arguments to ``arena + offset``.

The algorithm below is the same interval best-fit (it has to be: a plan that
is executed with offsets differing from the reference's would not be the same
plan), restated over ``PProgram``.  ``ALIGN`` is raised from 64 to 256 bytes only
when ``align`` is passed explicitly; the default keeps the reference's 64 so the
offsets match it byte for byte, and every offset is still 16-byte aligned as the
128-bit vector paths and TMA need.
"""
from __future__ import annotations

from dataclasses import dataclass, field

from .plan import ITEMSIZE, PNode, PProgram

ALIGN = 64


@dataclass
class Buffer:
    node: PNode
    size: int
    first: int
    last: int
    offset: int = -1


@dataclass
class MemoryPlan:
    buffers: dict[int, Buffer] = field(default_factory=dict)   # node id -> Buffer
    arena_bytes: int = 0
    naive_bytes: int = 0

    @property
    def savings(self) -> float:
        return 1.0 - self.arena_bytes / self.naive_bytes if self.naive_bytes else 0.0

    def offset(self, node: PNode) -> int | None:
        b = self.buffers.get(node.id)
        return None if b is None else b.offset

    def __str__(self) -> str:
        lines = [f"arena {self.arena_bytes} B (naive {self.naive_bytes} B, {self.savings:.0%} saved)"]
        for b in sorted(self.buffers.values(), key=lambda b: b.offset):
            lines.append(f"  [{b.offset:10d}, +{b.size:10d})  k{b.first}..k{b.last}  {b.node.name} {list(b.node.shape)}")
        return "\n".join(lines)


def _aligned(nbytes: int, align: int) -> int:
    return (nbytes + align - 1) // align * align


def plan_memory(program: PProgram, align: int = ALIGN) -> MemoryPlan:
    escaping = {program.resolve(o).id for o in program.outputs}
    bufs: dict[int, Buffer] = {}
    for ki, k in enumerate(program.kernels):
        for o in k.outputs:
            if o.id in escaping:
                continue
            nbytes = o.numel * ITEMSIZE[o.dtype]
            bufs[o.id] = Buffer(o, _aligned(max(nbytes, 1), align), first=ki, last=ki)
        for i in k.inputs:
            src = program.resolve(i)
            if src.id in bufs:
                bufs[src.id].last = ki

    order = sorted(bufs.values(), key=lambda b: (b.first, -b.size))
    live: list[Buffer] = []
    arena = 0
    for b in order:
        live = [x for x in live if x.last >= b.first]
        occupied = sorted((x.offset, x.offset + x.size) for x in live)
        best, best_gap = None, None
        cursor = 0
        for start, end in occupied + [(arena, arena)]:
            gap = start - cursor
            if gap >= b.size and (best_gap is None or gap < best_gap):
                best, best_gap = cursor, gap
            cursor = max(cursor, end)
        if best is None:
            best = cursor
        b.offset = best
        arena = max(arena, b.offset + b.size)
        live.append(b)

    plan = MemoryPlan(bufs, arena_bytes=arena, naive_bytes=sum(b.size for b in bufs.values()))
    verify(plan)
    return plan


def verify(plan: MemoryPlan) -> None:
    """No two buffers that are live at the same kernel may overlap in the arena."""
    bs = sorted(plan.buffers.values(), key=lambda b: b.offset)
    for i, a in enumerate(bs):
        for b in bs[i + 1:]:
            if b.offset >= a.offset + a.size:
                break
            if not (a.last < b.first or b.last < a.first):
                raise AssertionError(f"memory plan conflict: {a.node.name} vs {b.node.name}")
