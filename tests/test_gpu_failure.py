"""Failure detection on the GPU without a fault: a bounded wait that runs out.

A test build of the tcgen05 GEMM (``-DTJ_TEST_STALL_FIRST_LOAD``) never fills its
first pipeline stage, so the MMA warp's wait on that stage cannot complete.  With
the wait limit lowered to 20 ms (``-DTJ_WAIT_NS``), every CTA must give up, record
(TIMEOUT, kernel*16 + site) in the program's status words, let its in-flight copies
land, free TMEM and return.  The host reads the status, and the context must stay
usable: the normal build of the same program then runs and matches the oracle.
"""
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu


def test_bounded_wait_timeout_reports_status_and_context_survives():
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200.runtime import RuntimeError_

    case = "gemm_tc_aligned__bf16"
    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    bad = B200Program(plan, use_graph=False, nvcc_flags=("-DTJ_TEST_STALL_FIRST_LOAD", "-DTJ_WAIT_NS=20000000ull"))
    outs = [torch.empty(s, dtype=d, device="cuda") for s, d in bad.output_specs()]
    bad.run_into(ins, outs)
    torch.cuda.synchronize()
    code, where = bad.native.check_status()
    assert code == 1                       # TJ_STATUS_WAIT_TIMEOUT
    assert where // 16 == 0 and where % 16 in (1, 2, 3, 4)
    # the words were cleared by the read
    assert bad.native.check_status() == (0, 0)
    # B200Program.check() raises on a recorded failure
    bad.run_into(ins, outs)
    with pytest.raises(RuntimeError_):
        bad.check()
    bad.close()
    # the context is still healthy
    good = B200Program(plan)
    y = good(*ins)[0]
    good.check()
    ref = evaluate(plan, [t.cpu() for t in ins], round_stored=True)[0]
    assert normwise_error(y, ref) <= 2e-2


def test_cta_pair_bounded_wait_timeout_reports_status_and_context_survives():
    """The same for the CTA-pair GEMM (cta_group::2, 2-CTA clusters): neither CTA fills its
    first stage, so the leader's MMA wait runs out; the abort reaches the peer CTA through
    distributed shared memory, both leave through the final cluster barrier after a bounded
    grace period for their copies, and the context stays usable."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200.autotune import parse_tile, plain_gemm_plan

    plan = plain_gemm_plan(512, 512, 512)
    tiles = {0: parse_tile("256:4:16:1").as_dict()}
    g = torch.Generator(device="cuda").manual_seed(5)
    a = torch.randn((512, 512), generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn((512, 512), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    bad = B200Program(plan, use_graph=False, tiles=tiles,
                      nvcc_flags=("-DTJ_TEST_STALL_FIRST_LOAD", "-DTJ_WAIT_NS=20000000ull"))
    assert bad.kernel_sources[0].cluster == (2, 1, 1) and bad.kernel_sources[0].info["pair"]
    out = torch.empty((512, 512), dtype=torch.bfloat16, device="cuda")
    bad.run_into([a, b], [out])
    torch.cuda.synchronize()
    code, where = bad.native.check_status()
    assert code == 1 and where // 16 == 0 and where % 16 in (1, 2, 3, 4)
    bad.close()
    good = B200Program(plan, tiles=tiles)
    y = good(a, b)[0]
    good.check()
    assert normwise_error(y, a.float() @ b.float().T) <= 1e-2


def test_attention_bounded_wait_timeout_reports_status_and_context_survives():
    """The same for the fused attention kernel: its test build never loads the first K/V
    block, so the MMA warps (and then every other role) must give up, report, drain and
    return."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    case = "attention_core__bf16"
    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    bad = B200Program(plan, use_graph=False, nvcc_flags=("-DTJ_TEST_STALL_FIRST_LOAD", "-DTJ_WAIT_NS=20000000ull"))
    assert [ks.family for ks in bad.kernel_sources] == ["attention"]
    outs = [torch.empty(s, dtype=d, device="cuda") for s, d in bad.output_specs()]
    bad.run_into(ins, outs)
    torch.cuda.synchronize()
    code, where = bad.native.check_status()
    assert code == 1 and where // 16 == 0  # TJ_STATUS_WAIT_TIMEOUT in plan kernel 0
    bad.close()
    good = B200Program(plan)
    y = good(*ins)[0]
    good.check()
    ref = evaluate(plan, [t.cpu() for t in ins])[0]
    assert normwise_error(y, ref) <= 2e-2
