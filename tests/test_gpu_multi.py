"""Row-sharded execution on two GPUs with NCCL (skipped on a machine with fewer than two).

Each of two ranks (one process per GPU) runs the cfg5 program on its own 1024 rows of the seeded
cfg5 inputs (rows [1024 r, 1024 r + 1024)), with the weights replicated and no collective in the
step; ``distributed.gather_rows`` then all-gathers the row shards over NVLink.  Both ranks must
hold the same gathered tensor, rank 0's rows must match the reference ``c`` backend's golden
rows, and rank 1's rows the oracle.
"""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

pytestmark = pytest.mark.gpu


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _rank(rank, world, port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import torch.distributed as dist
    from datetime import timedelta

    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W
    from mlir_gpu_kernel_compiler_b200.distributed import gather_rows
    from oracle import fixtures as FX
    from oracle.plan_oracle import evaluate, normwise_error

    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=timedelta(seconds=120))
    try:
        w = W.WORKLOADS["cfg5"]
        lo, hi = 1024 * rank, 1024 * (rank + 1)
        ins = W.make_inputs(w, device=f"cuda:{rank}", rows=(lo, hi))
        plan = FX.load_plan("cfg5_m1024")
        prog = B200Program(plan, device=f"cuda:{rank}")
        y = prog(*ins)[0]
        prog.check()
        full = gather_rows(y)
        torch.cuda.synchronize()
        sums = torch.tensor([full.float().sum().item(), full.float().abs().sum().item()], device=f"cuda:{rank}",
                            dtype=torch.float64)
        other = sums.clone()
        dist.all_reduce(other, op=dist.ReduceOp.MAX)
        same = bool(torch.equal(other, sums))
        ok_rows = bool(torch.equal(full[lo:hi], y))
        if rank == 0:
            err = FX.check_against_golden(full[:1024], FX.case_expected("cfg5_m1024")[0], 2e-2)
        else:
            sub = [ins[0][:64].float().cpu()] + [t.float().cpu() for t in ins[1:]]
            err = normwise_error(full[1024:1088], evaluate(plan, sub, strict_shapes=False)[0])
        q.put((rank, same, ok_rows, tuple(full.shape), float(err)))
    finally:
        dist.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs two GPUs")
def test_two_rank_shards_and_nccl_gather():
    world, port = 2, _free_port()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    res = sorted(q.get(timeout=600) for _ in range(world))
    for p in procs:
        p.join(timeout=120)
    for rank, same, ok_rows, shape, err in res:
        assert same and ok_rows and shape == (2048, 4096), (rank, same, ok_rows, shape)
        assert err <= 2e-2, (rank, err)
