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
import subprocess
import sys
import textwrap
from pathlib import Path

import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parents[1]
CASE = "linear_nobias_ragged__f32"      # C[200, 300] = A[200, 136] @ B[300, 136]^T


def _noalloc(lib, a, b, c):
    m, k = a.shape
    n = b.shape[0]
    stream = torch.cuda.current_stream().cuda_stream
    return lib.tj_b200_linear_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), m, n, k, stream)


def _status(lib):
    code, where = ctypes.c_int32(-7), ctypes.c_int32(-7)
    rc = lib.tj_b200_linear_f32_noalloc_status(ctypes.byref(code), ctypes.byref(where),
                                               torch.cuda.current_stream().cuda_stream)
    return rc, code.value, where.value


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
    assert _status(lib) == (rt.TJ_OK, 0, 0)                # no bounded wait ran out


@pytest.mark.parametrize("m,n,k", [(2048, 2048, 1024),   # 512 output tiles: 3-4 per CTA, both TMEM buffers
                                   (200, 301, 136)])     # N % 4 != 0: the scalar epilogue stores
def test_noalloc_linear_persistent_and_ragged_shapes(m, n, k):
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import runtime as rt
    from mlir_gpu_kernel_compiler_b200.autotune import plain_gemm_plan

    lib = rt.library()
    plan = plain_gemm_plan(m, n, k, "f32")
    prog = B200Program(plan)
    g = torch.Generator(device="cuda").manual_seed(11)
    for rep in range(2):
        a = torch.randn((m, k), generator=g, device="cuda")
        b = torch.randn((n, k), generator=g, device="cuda") * (0.05 if rep else 1.0)
        c = torch.full((m, n), float("nan"), device="cuda")
        assert _noalloc(lib, a, b, c) == rt.TJ_OK, lib.tj_b200_last_error()
        ref = prog(a, b)[0]
        torch.cuda.synchronize()
        assert normwise_error(c, ref) <= 1e-4
        assert normwise_error(c, evaluate(plan, [a.cpu(), b.cpu()])[0]) <= 1e-4
    assert _status(lib) == (rt.TJ_OK, 0, 0)


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
    assert _status(lib)[0] == rt.TJ_OK
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


_STALL_CHILD = textwrap.dedent("""
    import ctypes, sys
    import torch
    sys.path.insert(0, sys.argv[2])
    from mlir_gpu_kernel_compiler_b200 import runtime as rt
    lib = rt.library(sys.argv[1])            # the failure-path test build of the library
    a = torch.randn(256, 128, device="cuda")
    b = torch.randn(192, 128, device="cuda")
    c = torch.zeros(256, 192, device="cuda")
    s = torch.cuda.current_stream().cuda_stream
    assert lib.tj_b200_linear_f32_noalloc(a.data_ptr(), b.data_ptr(), c.data_ptr(), 256, 192, 128, s) == 0
    code, where = ctypes.c_int32(), ctypes.c_int32()
    rc = lib.tj_b200_linear_f32_noalloc_status(ctypes.byref(code), ctypes.byref(where), s)
    rc2 = lib.tj_b200_linear_f32_noalloc_status(ctypes.byref(ctypes.c_int32()), ctypes.byref(ctypes.c_int32()), s)
    torch.cuda.synchronize()
    ok = bool(torch.allclose(a @ b.T, (a.double() @ b.double().T).float(), atol=1e-2))   # context still usable
    print("RESULT", rc, code.value, where.value, rc2, ok)
""")


def test_noalloc_bounded_wait_timeout_is_reported_by_the_status_read():
    """A test build whose producer never fills the first pipeline stage, with the wait limit
    lowered to 20 ms: the call returns TJ_OK (it is asynchronous), the status read then reports
    the timeout and its wait site, the read clears it, and the context stays usable.  Run in a
    child process so the test build's own static scratch never meets the product library's."""
    from mlir_gpu_kernel_compiler_b200 import runtime as rt
    from mlir_gpu_kernel_compiler_b200 import toolchain

    lib = toolchain.build_runtime(extra_flags=toolchain.STALL_TEST_FLAGS, variant="stalltest")
    r = subprocess.run([sys.executable, "-c", _STALL_CHILD, str(lib), str(ROOT)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr[-2000:]
    line = [x for x in r.stdout.splitlines() if x.startswith("RESULT")][-1].split()
    rc, code, where, rc2, ok = int(line[1]), int(line[2]), int(line[3]), int(line[4]), line[5] == "True"
    assert rc == rt.TJ_ERR_DEVICE_STATUS and code == 1 and where in (1, 2, 3, 4)
    assert rc2 == rt.TJ_OK                                 # the read cleared the words
    assert ok
