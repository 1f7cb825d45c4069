"""The five benchmark programs of the B200 backend, as seeded synthetic inputs.

Each workload is one tensorjit program whose fused plan ships as a JSON fixture
(``tests/golden/plans/<plan>.json``, produced by the reference's own tracer and
fusion passes).  This module only knows the argument list of each program and how
to draw its inputs: ``torch.manual_seed(seed)`` on the CPU generator, arguments
created in order, ``randn`` draws for the N(0, s) arguments (scaled by s, then
cast to the program dtype), constants for gains and zero biases.  The CPU
generator makes the inputs identical on every machine.

Algorithmic work per program (the roofline numerators):

* cfg1 MLP 512x768 f32: 2 GEMMs, 2*512*3072*768*2 = 4.832 GFLOP.
* cfg2 RMSNorm(x+r) [16384,4096] + softmax [8192,8192] bf16: reads x, r, s and
  writes both outputs once: 671.1 MB.
* cfg3 gelu(x@w.T+b)+res, 8192x16384x4096 bf16: 1.0995 TFLOP.
* cfg4 pre-norm transformer block B8 x T2048, d1024, 16x64 heads, bf16: 549.8 GFLOP.
* cfg5 MLP 131072x4096 -> 16384 -> 4096 bf16: 35.18 TFLOP (rows split across ranks).
"""
from __future__ import annotations

import math
from dataclasses import dataclass, field

import torch


@dataclass
class Arg:
    name: str
    shape: tuple
    init: str            # "randn" | "ones" | "zeros" | "rand_plus_half"
    scale: float = 1.0


@dataclass
class Workload:
    name: str
    plan: str            # plan fixture name
    dtype: torch.dtype
    seed: int
    args: list[Arg]
    flops: float = 0.0   # algorithmic tensor FLOPs per program
    hbm_bytes: float = 0.0  # algorithmic HBM bytes per program (bandwidth-bound programs)
    row_args: tuple = ()  # indices of arguments sharded by rows across ranks
    rows: int = 0
    description: str = ""
    extra: dict = field(default_factory=dict)


def _mlp_flops(m, d, h):
    return 2.0 * m * h * d * 2


D4 = 1024
WORKLOADS: dict[str, Workload] = {
    "cfg1": Workload(
        "cfg1", "cfg1", torch.float32, 0,
        [Arg("x", (512, 768), "randn"), Arg("g", (768,), "ones"), Arg("w1", (3072, 768), "randn", 0.02),
         Arg("b1", (3072,), "zeros"), Arg("w2", (768, 3072), "randn", 0.02), Arg("b2", (768,), "zeros")],
        flops=_mlp_flops(512, 768, 3072), row_args=(0,), rows=512,
        description="README MLP block, f32: x + linear(gelu(linear(layer_norm(x,g),w1,b1)),w2,b2)"),
    "cfg2": Workload(
        "cfg2", "cfg2", torch.bfloat16, 1,
        [Arg("x", (16384, 4096), "randn"), Arg("r", (16384, 4096), "randn"), Arg("g", (4096,), "ones"),
         Arg("s", (8192, 8192), "randn")],
        hbm_bytes=2.0 * (3 * 16384 * 4096 + 2 * 8192 * 8192), row_args=(0, 1, 3),
        description="rms_norm(x + r, g) and softmax(s), bf16"),
    "cfg3": Workload(
        "cfg3", "cfg3", torch.bfloat16, 2,
        [Arg("x", (8192, 4096), "randn"), Arg("w", (16384, 4096), "randn", 0.02), Arg("b", (16384,), "randn", 0.02),
         Arg("res", (8192, 16384), "randn")],
        flops=2.0 * 8192 * 16384 * 4096, row_args=(0, 3), rows=8192,
        description="gelu(x @ w.T + b) + res, bf16 with f32 accumulate"),
    "cfg4": Workload(
        "cfg4", "cfg4", torch.bfloat16, 3,
        [Arg("x", (16384, D4), "randn"), Arg("g1", (D4,), "ones"), Arg("wq", (D4, D4), "randn", 0.02),
         Arg("wk", (D4, D4), "randn", 0.02), Arg("wv", (D4, D4), "randn", 0.02), Arg("wo", (D4, D4), "randn", 0.02),
         Arg("bo", (D4,), "randn", 0.02), Arg("g2", (D4,), "ones"), Arg("w1", (4 * D4, D4), "randn", 0.02),
         Arg("b1", (4 * D4,), "randn", 0.02), Arg("w2", (D4, 4 * D4), "randn", 0.02), Arg("b2", (D4,), "randn", 0.02)],
        flops=4 * 2.0 * 16384 * D4 * D4 + 2 * 2.0 * 128 * 2048 * 2048 * 64 + 2 * 2.0 * 16384 * D4 * 4 * D4,
        row_args=(0,),
        description="pre-norm transformer block, B8xT2048, d1024, 16 heads x 64, bf16"),
    "cfg5": Workload(
        "cfg5", "cfg5_m131072", torch.bfloat16, 4,
        [Arg("x", (131072, 4096), "randn"), Arg("g", (4096,), "ones"), Arg("w1", (16384, 4096), "randn", 0.02),
         Arg("b1", (16384,), "zeros"), Arg("w2", (4096, 16384), "randn", 0.02), Arg("b2", (4096,), "zeros")],
        flops=_mlp_flops(131072, 4096, 16384), row_args=(0,), rows=131072,
        description="large-batch MLP x + linear(gelu(linear(rms_norm(x,g),w1,b1)),w2,b2), bf16, rows sharded"),
}


def make_inputs(w: Workload, device="cpu", rows: tuple[int, int] | None = None) -> list[torch.Tensor]:
    """Draw the workload's inputs (CPU generator, in argument order), then move them.

    ``rows=(lo, hi)`` returns only that row range of the row-sharded arguments
    (the full tensors are still drawn, so every slice sees the same values).
    """
    g = torch.Generator().manual_seed(w.seed)
    out = []
    for i, a in enumerate(w.args):
        if a.init == "randn":
            t = torch.randn(a.shape, generator=g, dtype=torch.float32)
            if a.scale != 1.0:
                t.mul_(a.scale)
        elif a.init == "ones":
            t = torch.ones(a.shape, dtype=torch.float32)
        elif a.init == "zeros":
            t = torch.zeros(a.shape, dtype=torch.float32)
        elif a.init == "rand_plus_half":
            t = torch.rand(a.shape, generator=g, dtype=torch.float32) + 0.5
        else:  # pragma: no cover
            raise ValueError(a.init)
        if rows is not None and i in w.row_args:
            t = t[rows[0]:rows[1]]
        out.append(t.to(w.dtype).to(device).contiguous())
    return out


def sharded_plan_name(w: Workload, world: int, total: int | None = None) -> str:
    """Plan fixture for one rank's row shard of ``w`` (same program, M = rows / world);
    ``total`` runs a leading row slice of that many rows instead of all of them."""
    if w.name != "cfg5":
        return w.plan
    return f"cfg5_m{(total or w.rows) // world}"


def shard_rows(total: int, world: int, rank: int) -> tuple[int, int]:
    per = total // world
    return rank * per, (rank + 1) * per


def numel(shape) -> int:
    return math.prod(shape) if shape else 1

