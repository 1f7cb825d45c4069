"""The five benchmark programs at full size on the GPU, against the reference.

Each program's inputs are drawn from its seed (``workloads.make_inputs``).  The reference
``c`` backend's outputs for the same inputs are pinned in ``tests/golden``:

* ``<cfg>.golden.npz``: checksums plus sample rows of every output;
* ``<cfg>.dense.npz`` (cfg2, cfg4): per-row checksums of EVERY output row (sum, sum of |y|,
  sum of y^2, position-weighted sum) and whole rows: all of cfg4's batch element 0 (rows
  0..2047, the attention of one batch element end to end) and 256 rows spread over cfg2's
  two outputs.

The CPU oracle additionally checks row slices of the row-independent programs.  Tolerance:
normwise 1e-4 (f32) / 2e-2 (bf16); the row checksums use the same bound relative to the row's
sum of |y|.
"""
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
    dense = FX.case_dense(w.plan)
    if dense is not None:                    # every row, not only the sampled ones
        for i, y in enumerate(outs):
            FX.check_rows_dense(y, dense, i, tol)
    # the oracle on row slices (first, middle, last rows) of the row-independent programs;
    # cfg2's slices take the same rows of both of its outputs (x, r and s are sliced alike)
    if cfg in ("cfg1", "cfg2", "cfg3"):
        rows = w.args[0].shape[0]
        slices = [(0, 128), (rows // 2 - 64, rows // 2 + 64), (rows - 128, rows)]
        if cfg == "cfg2":
            slices.append((8192 - 128, 8192))     # the softmax output's last rows
        for lo, hi in slices:
            sub_in = W.make_inputs(w, rows=(lo, hi))
            refs = evaluate(plan, sub_in, strict_shapes=False)
            for y, ref in zip(outs, refs):
                if ref.shape[0]:
                    assert normwise_error(y[lo:lo + ref.shape[0]], ref) <= tol


def test_cfg4_every_row_of_batch_element_0_matches_the_reference():
    """The transformer block's first batch element (2048 rows: LayerNorm, q/k/v, the fused
    attention over all 16 heads, out-projection, MLP) against the reference c backend's own
    output for those rows, row by row; the per-row checksums cover the other 7 elements."""
    w = W.WORKLOADS["cfg4"]
    plan, prog, outs = _run(w.plan, W.make_inputs(w))
    dense = FX.case_dense(w.plan)
    worst = FX.check_rows_dense(outs[0], dense, 0, 2e-2)
    assert worst["rows"] <= 2e-2
    assert normwise_error(outs[0][:2048], dense["out0_dense"].astype("float32")) <= 2e-2


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
