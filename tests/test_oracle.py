"""The CPU oracle against golden outputs of the reference's own ``c`` backend.

This pins ``oracle/plan_oracle.py`` before any GPU result is compared with it:
every fixture case and every benchmark config is evaluated by the oracle on the
same seeded inputs and must agree with what the reference computed.
"""
import numpy as np
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error, tj_erff

from mlir_gpu_kernel_compiler_b200 import workloads as W


@pytest.mark.parametrize("case", FX.cases("case"))
def test_oracle_matches_reference_c_backend(case):
    plan = FX.load_plan(case)
    ins = FX.case_inputs(case)
    outs = evaluate(plan, ins)
    exp = FX.case_expected(case)
    assert len(outs) == len(exp)
    for y, e in zip(outs, exp):
        FX.check_against_golden(torch.from_numpy(np.ascontiguousarray(y)), e, 1e-5)


@pytest.mark.parametrize("cfg", ["cfg1", "cfg2", "cfg3", "cfg4"])
def test_oracle_matches_reference_on_configs(cfg):
    w = W.WORKLOADS[cfg]
    plan = FX.load_plan(w.plan)
    outs = evaluate(plan, W.make_inputs(w))
    for y, e in zip(outs, FX.case_expected(w.plan)):
        FX.check_against_golden(torch.from_numpy(y), e, 1e-5)
    dense = FX.case_dense(w.plan)
    if dense is not None:
        # every row's checksums, and the whole rows (stored as f16 where that keeps the values
        # normal, hence 1e-3: f16 rounding is at most 2^-11 of a row's largest value)
        for i, y in enumerate(outs):
            worst = FX.check_rows_dense(torch.from_numpy(y), dense, i, 1e-3)
            assert max(v for k, v in worst.items() if k != "rows") <= 1e-5


def test_oracle_matches_reference_on_cfg5_slice():
    w = W.WORKLOADS["cfg5"]
    plan = FX.load_plan("cfg5_m1024")
    outs = evaluate(plan, W.make_inputs(w, rows=(0, 1024)))
    for y, e in zip(outs, FX.case_expected("cfg5_m1024")):
        FX.check_against_golden(torch.from_numpy(y), e, 1e-5)


def test_tj_erff_bound():
    import math

    x = np.linspace(-6, 6, 20001, dtype=np.float32)
    ref = np.array([math.erf(float(v)) for v in x])
    # A&S 7.1.26 is accurate to 1.5e-7 in exact arithmetic; f32 evaluation adds a few ulp
    assert np.abs(tj_erff(x).astype(np.float64) - ref).max() < 6e-7


def test_normwise_error_metric():
    ref = np.array([1.0, -2.0, 4.0], np.float32)
    assert normwise_error(ref, ref) == 0.0
    assert abs(normwise_error(ref + np.float32(0.04), ref) - 0.01) < 1e-6
    assert normwise_error(np.array([np.nan, 0, 0], np.float32), ref) == float("inf")
