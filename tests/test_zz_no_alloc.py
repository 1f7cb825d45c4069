"""The allocation-free f32 linear entry point, checked against the regular path.

``tj_b200_linear_f32_noalloc`` exists for callers that cannot call cudaMalloc -- code
running inside a host application that owns all device memory and only hands out input
and output buffers, or a path where an allocation could block or fail.  It computes the
same 3xTF32 linear layer as a compiled program run through ``tj_b200_run``, but keeps
its TF32 hi/lo operand copies in a static device array instead of a runtime-allocated
workspace.  This file is collected last on purpose: a failure here leaves every other
test already run.  It must also pass on its own in a fresh process.
"""
import ctypes

import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu

CASE = "linear_nobias_ragged__f32"      # C[200, 300] = A[200, 136] @ B[300, 136]^T


def _noalloc(lib, a, b, c):
    m, k = a.shape
    n = b.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tj_b200_linear_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream)


def test_noalloc_linear_matches_the_regular_entry_point_on_two_calls():
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import runtime as rt

    lib = rt.library()
    plan = FX.load_plan(CASE)
    a0, b0 = [t.cuda() for t in FX.case_inputs(CASE)]
    prog = B200Program(plan)                               # regular path: tj_b200_run, arena workspace
    inputs = [(a0, b0), (a0 * -0.5 + 1.0, b0 * 2.0 - 0.25)]  # second call: new data in the shared scratch
    for a, b in inputs:
        ref = prog(a, b)[0]
        c = torch.full((a.shape[0], b.shape[0]), float("nan"), device="cuda")
        assert _noalloc(lib, a, b, c) == rt.TJ_OK, lib.tj_b200_last_error()
        torch.cuda.synchronize()
        assert normwise_error(c, ref) <= 1e-4                  # the f32 tolerance of every f32 test
        assert normwise_error(c, evaluate(plan, [a.cpu(), b.cpu()])[0]) <= 1e-4


def test_noalloc_linear_allocates_nothing_and_rejects_oversized_calls():
    from mlir_gpu_kernel_compiler_b200 import runtime as rt

    lib = rt.library()
    a, b = [t.cuda() for t in FX.case_inputs(CASE)]
    c = torch.empty(a.shape[0], b.shape[0], device="cuda")
    assert _noalloc(lib, a, b, c) == rt.TJ_OK            # first call on this device: set-up
    torch.cuda.synchronize()
    free_before = torch.cuda.mem_get_info()[0]
    for _ in range(3):
        assert _noalloc(lib, a, b, c) == rt.TJ_OK
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free_before    # no device memory taken by the calls
    # M*K beyond the static scratch (2^21 elements per operand) is refused, not truncated
    big = torch.empty(2049, 1024, device="cuda")
    w = torch.empty(64, 1024, device="cuda")
    out = torch.empty(2049, 64, device="cuda")
    assert _noalloc(lib, big, w, out) == rt.TJ_ERR_INVALID
    assert b"static scratch" in lib.tj_b200_last_error()
    # K must keep 16-byte rows
    assert lib.tj_b200_linear_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), 200, 300, 135,
                                          None) == rt.TJ_ERR_INVALID
