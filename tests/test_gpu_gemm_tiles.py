"""Every tensor-core GEMM tile shape against the reference, not only the one the
tuner picks: ``TENSORJIT_B200_TILE=BN:STAGES:GROUP_M:PAIR`` forces the tile of
each bf16/f16 matmul, including the CTA-pair (``cta_group::2``, 256-row tile)
kernel, which runs only when the override asks for it.  Outputs must match the
reference ``c`` backend's golden outputs and the bf16-storage oracle exactly as
in the fixture parity suite (cuda_backend.py:299-429 is the path replaced)."""
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu

CASES = ["gemm_tc_aligned__bf16", "gemm_tc_aligned__f16", "gemm_tc_ragged__bf16", "gemm_tc_multiwave__bf16",
         "gemm_tc_batched_tb__bf16", "cuda_mlp__bf16", "linear_tb__bf16"]
# (BN, STAGES, GROUP_M, PAIR): the pair kernel at both widths, and single-CTA tiles of
# every width with shallow and deep pipelines
TILES = ["256:4:16:1", "128:6:8:1", "256:3:16:0", "128:6:4:0", "64:8:16:0"]


@pytest.mark.parametrize("tile", TILES)
@pytest.mark.parametrize("case", CASES)
def test_forced_tile_matches_reference(case, tile, monkeypatch):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    monkeypatch.setenv("TENSORJIT_B200_TILE", tile)
    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    prog = B200Program(plan, device="cuda")
    gemms = [ks for ks in prog.kernel_sources if ks.family == "gemm_tc"]
    assert gemms, "the case must run a tensor-core GEMM"
    bn, _, _, pair = (int(x) for x in tile.split(":"))
    for ks in gemms:   # every case has a K-major B, which the pair kernel needs
        assert (ks.info["BN"], ks.info["pair"]) == (bn, bool(pair))
        assert ks.cluster == ((2, 1, 1) if pair else (1, 1, 1))
    outs = prog(*ins)
    torch.cuda.synchronize()
    prog.check()
    dt = plan.meta["dtype"]
    tol = FX.TOL[dt]
    cpu_ins = [t.cpu() for t in ins]
    ref = evaluate(plan, cpu_ins)
    emul = evaluate(plan, cpu_ins, round_stored=True)
    for i, (y, e, r, m) in enumerate(zip(outs, FX.case_expected(case), ref, emul)):
        assert normwise_error(y, m) <= tol
        FX.check_against_golden(y, e, FX.allowed_error(case, i, tol))
        assert normwise_error(y, r) <= FX.allowed_error(case, i, tol)



@pytest.mark.parametrize("tile", ["256:5:16:1", "256:6:8:1", "128:8:16:1", "256:4:16:0"])
@pytest.mark.parametrize("M,N,K", [(2000, 4000, 1000), (4096, 2048, 4096)])
def test_persistent_tiles_against_torch_fp32(tile, M, N, K):
    """More tiles than CTA pairs (every pair runs several tiles through both TMEM
    accumulator buffers) with ragged M, N and K, against a plain PyTorch fp32 GEMM."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200.autotune import parse_tile, plain_gemm_plan

    cfg = parse_tile(tile)
    prog = B200Program(plain_gemm_plan(M, N, K), device="cuda", tiles={0: cfg.as_dict()})
    (ks,) = prog.kernel_sources
    tiles = -(-M // (256 if cfg.PAIR else 128)) * -(-N // cfg.BN)
    assert ks.info["pair"] == cfg.PAIR and tiles > ks.grid[0] // (2 if cfg.PAIR else 1)
    g = torch.Generator(device="cuda").manual_seed(M + N + K)
    a = torch.randn((M, K), generator=g, device="cuda").to(torch.bfloat16)
    b = (torch.randn((N, K), generator=g, device="cuda") * 0.05).to(torch.bfloat16)
    y = prog(a, b)[0]
    torch.cuda.synchronize()
    prog.check()
    ref = a.float() @ b.float().T
    assert y.dtype == torch.bfloat16 and y.shape == (M, N)
    assert normwise_error(y, ref) <= 1e-2


def test_library_comparison_tool_runs():
    from mlir_gpu_kernel_compiler_b200.autotune import compare_with_library, parse_tile

    res = compare_with_library(1024, 1024, 512, [parse_tile("256:4:16:1"), parse_tile("256:4:16:0")], rounds=1,
                               seconds=0.05)
    assert set(res) == {"256:4:16:1", "256:4:16:0", "library"}
    assert all(r["ms"] > 0 for r in res.values())
