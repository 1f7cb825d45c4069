"""Row-sharding host logic with world_size-2 gloo process groups on the CPU."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from mlir_gpu_kernel_compiler_b200.distributed import gather_rows, max_over_ranks, shard, shard_bounds


def test_shard_bounds_cover_rows_exactly():
    for total in (1, 7, 512, 131072, 131073):
        for world in (1, 2, 3, 4, 8):
            spans = [shard_bounds(total, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == total
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(h - l for l, h in spans) - min(h - l for l, h in spans) <= 1
    with pytest.raises(ValueError):
        shard_bounds(10, 2, 2)


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        full = torch.arange(24 * 3, dtype=torch.float32).reshape(24, 3)
        mine = shard(full, world, rank) * 2.0          # stand-in for the rank's program on its rows
        got = gather_rows(mine)
        ok = bool(torch.equal(got, full * 2.0))
        slow = max_over_ranks(float(rank + 1))
        q.put((rank, ok, slow))
    finally:
        dist.destroy_process_group()


def test_gather_rows_and_max_over_ranks_gloo():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    assert [r[1] for r in res] == [True, True]
    assert [r[2] for r in res] == [2.0, 2.0]


def _dying_worker(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=5))
    if rank == 1:
        os._exit(0)                                    # leaves between steps, nothing in flight
    try:
        gather_rows(torch.ones(2, 2))
        q.put(("no error", rank))
    except Exception as e:                             # the survivor's collective times out
        q.put(("error", type(e).__name__))


def test_rank_failure_surfaces_as_error_not_hang():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_dying_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    status, _ = q.get(timeout=120)
    for p in procs:
        p.join(timeout=60)
        if p.is_alive():
            p.kill()
    assert status == "error"


def _rows_on_root_worker(rank, world, port, q, mode):
    """RowsOnRoot's set-up on gloo ranks: with fake peer-memory calls (mode "fake") it hands rank
    0 its tensor slice and the other ranks an address inside the exported buffer; when the
    export (mode "no_export", the real call: no driver here) or the mapping (mode "no_map")
    fails, every rank raises at the same point instead of waiting in a later collective."""
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    from datetime import timedelta

    from mlir_gpu_kernel_compiler_b200 import runtime as rt
    from mlir_gpu_kernel_compiler_b200.distributed import RowsOnRoot

    calls = []
    if mode in ("fake", "no_map"):
        rt.ipc_export = lambda ptr, dev: (b"h" * 64, 4096)
    if mode == "fake":
        rt.ipc_open = lambda h, off, dev: (calls.append(("open", h, off)), 1 << 40)[1] + off
        rt.ipc_close = lambda ptr, off, dev: calls.append(("close", ptr, off))
    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=60))
    try:
        try:
            t = RowsOnRoot((10, 4), torch.float32, torch.device("cpu"))
        except RuntimeError as ex:
            q.put((rank, "raised", str(ex)))
            return
        if rank == 0:
            ok = t.full is not None and t.full.shape == (10, 4) and t.dest.data_ptr() == t.full.data_ptr()
        else:
            ok = t.full is None and t.dest == (1 << 40) + 4096 + 5 * 4 * 4 and calls[0] == ("open", b"h" * 64, 4096)
        t.close()
        if rank == 1:
            ok &= calls[-1] == ("close", (1 << 40) + 4096, 4096)
        q.put((rank, "ok", ok))
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("mode", ["fake", "no_export", "no_map"])
def test_rows_on_root_setup_and_collective_failure_gloo(mode):
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rows_on_root_worker, args=(r, world, port, q, mode)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=120) for _ in range(world))
    for p in procs:
        p.join(timeout=60)
    if mode == "fake":
        assert res == [(0, "ok", True), (1, "ok", True)]
    else:
        assert [r[1] for r in res] == ["raised", "raised"], res
        want = "could not export" if mode == "no_export" else "could not map"
        assert any(want in r[2] for r in res), res
