"""The checked kernel build on the GPU (``TENSORJIT_B200_CHECKED=1`` / ``checked=True``).

In the checked build every generated global load and store goes through a bounded view of its
operand, the GEMM and attention templates check their TMA tile coordinates and TMEM columns,
and a violation is reported as TJ_STATUS_BOUNDS in the program's status words (the access is
skipped) -- the stand-in for a memory checker, which is not available on these machines.  The
counterpart in the reference is its debug build and the native runtime's argument checks
(``tensorjit/backends/cuda_driver.py:86-87``, ``csrc/runtime.cpp:53-68,89-90``).

Every fixture plan and the full-size transformer block and fused GEMM run here under the
checked build: no kernel may report a violation, and the results must still match the
reference's golden outputs.
"""
import pytest
import torch

from mlir_gpu_kernel_compiler_b200 import workloads as W
from oracle import fixtures as FX

pytestmark = pytest.mark.gpu


def _checked_program(plan):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    prog = B200Program(plan, device="cuda", checked=True)
    assert prog.checked and all(("status", None) in ks.args for ks in prog.kernel_sources)
    return prog


@pytest.mark.parametrize("case", FX.cases("case"))
def test_fixture_runs_clean_under_the_checked_build(case):
    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    prog = _checked_program(plan)
    outs = prog(*ins)
    torch.cuda.synchronize()
    assert prog.native.check_status() == (0, 0)           # no bounds violation, no timeout
    tol = FX.TOL[plan.meta["dtype"]]
    for i, (y, e) in enumerate(zip(outs, FX.case_expected(case))):
        FX.check_against_golden(y, e, FX.allowed_error(case, i, tol))


@pytest.mark.parametrize("cfg", ["cfg3", "cfg4"])
def test_full_size_config_runs_clean_under_the_checked_build(cfg):
    w = W.WORKLOADS[cfg]
    plan = FX.load_plan(w.plan)
    prog = _checked_program(plan)
    outs = prog(*[t.cuda() for t in W.make_inputs(w)])
    torch.cuda.synchronize()
    assert prog.native.check_status() == (0, 0)
    for y, e in zip(outs, FX.case_expected(w.plan)):
        FX.check_against_golden(y, e, 2e-2)
