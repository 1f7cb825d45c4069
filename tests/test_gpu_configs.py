"""The five benchmark programs at full size on the GPU, against the reference.

Each program's inputs are drawn from its seed (``workloads.make_inputs``).  The
reference ``c`` backend's outputs for the same inputs are pinned in
``tests/golden/<cfg>.golden.npz`` as checksums plus sample rows; the CPU oracle
additionally checks row slices (every program is row-independent except cfg4's
attention, which is checked on its own golden rows).  Tolerance: normwise 1e-4
(f32) / 2e-2 (bf16).
"""
import numpy as np
import pytest
import torch

from mlir_gpu_kernel_compiler_b200 import B200Program
from mlir_gpu_kernel_compiler_b200 import workloads as W
from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu


def _run(plan_name, ins):
    plan = FX.load_plan(plan_name)
    prog = B200Program(plan, device="cuda")
    outs = prog(*[t.cuda() for t in ins])
    torch.cuda.synchronize()
    prog.check()
    return plan, prog, outs


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_config_matches_reference_golden(cfg):
    w = W.WORKLOADS[cfg]
    ins = W.make_inputs(w)
    plan, prog, outs = _run(w.plan, ins)
    tol = FX.TOL[plan.meta["dtype"]]
    exp = FX.case_expected(w.plan)
    assert len(outs) == len(exp)
    for y, e in zip(outs, exp):
        FX.check_against_golden(y, e, tol)
    # oracle on row slices (first, middle, last rows) for the row-independent programs
    if cfg in ("cfg1", "cfg2", "cfg3"):
        rows = w.args[0].shape[0]
        for lo in (0, rows // 2 - 64, rows - 128):
            sl = (lo, lo + 128)
            sub_in = W.make_inputs(w, rows=sl) if cfg != "cfg2" else None
            if cfg == "cfg2":
                continue
            ref = evaluate(plan, sub_in, strict_shapes=False)[0]
            y = outs[0][sl[0]:sl[1]]
            assert normwise_error(y, ref) <= tol


def test_cfg2_rows_against_oracle():
    w = W.WORKLOADS["cfg2"]
    ins = W.make_inputs(w)
    plan, prog, outs = _run(w.plan, ins)
    x, r, g, s = [t.float() for t in ins]
    for lo in (0, 8000, 16384 - 64):
        xs, rs = x[lo:lo + 64], r[lo:lo + 64]
        h = (xs + rs)
        ref = h * torch.rsqrt((h * h).mean(-1, keepdim=True) + 1e-6) * g
        assert normwise_error(outs[0][lo:lo + 64], ref) <= 2e-2
    for lo in (0, 4000, 8192 - 64):
        ref = torch.softmax(s[lo:lo + 64], -1)
        assert normwise_error(outs[1][lo:lo + 64], ref) <= 2e-2


def test_cfg5_full_program_rows_match_reference_and_shard_boundaries():
    w = W.WORKLOADS["cfg5"]
    ins = W.make_inputs(w)
    plan, prog, outs = _run("cfg5_m131072", ins)
    y = outs[0]
    # rows 0..1023 against the reference c backend's own output for those rows
    FX.check_against_golden(y[:1024], FX.case_expected("cfg5_m1024")[0], 2e-2)
    # oracle on slices that straddle every 2/4/8-way shard boundary
    sub_plan = FX.load_plan("cfg5_m1024")
    for b in (16384, 32768, 65536, 98304, 131072 - 64):
        lo = max(0, b - 32)
        sl = (lo, lo + 64)
        sub_in = [ins[0][sl[0]:sl[1]].float()] + [t.float() for t in ins[1:]]
        ref = evaluate(sub_plan, sub_in, strict_shapes=False)[0]
        assert normwise_error(y[sl[0]:sl[1]], ref) <= 2e-2


@pytest.mark.parametrize("world", [2, 4, 8])
def test_cfg5_shard_plans_equal_full_program_rows(world):
    """A rank's shard program (M = R / world) computes exactly the rows the full program does."""
    w = W.WORKLOADS["cfg5"]
    lo, hi = W.shard_rows(w.rows, world, world - 1)
    ins = W.make_inputs(w, rows=(lo, hi))
    plan, prog, outs = _run(W.sharded_plan_name(w, world), ins)
    sub_plan = FX.load_plan("cfg5_m1024")
    for a in (0, (hi - lo) - 64):
        sub_in = [ins[0][a:a + 64].float()] + [t.float() for t in ins[1:]]
        ref = evaluate(sub_plan, sub_in, strict_shapes=False)[0]
        assert normwise_error(outs[0][a:a + 64], ref) <= 2e-2
