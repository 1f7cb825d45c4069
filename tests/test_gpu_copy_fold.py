"""A transpose copy kernel folded into the GEMM that reads it (``fuse.fold_copies_into_gemm``),
on the GPU: the GEMM reads its A operand, or its K-major B, from the transpose's source through a
rank-3..5 tensor map (``heads_scores``: both, each with two batch dims; ``heads_attention_probs``:
also an N-major B), or, for operands that go through a pack / split launch (f32), that launch
gathers them from the source.

Against the unfused program (copy kernel, then the GEMM on the copy) and, at the transformer
config's head-merge size, against a PyTorch fp32 reference.  The fused and unfused GEMMs read the
same values in the same k order, so where both run the single-CTA kernel the outputs must be the
same bits; the unfused GEMM may run CTA-pair tiles at large sizes, then 1e-3 normwise.
"""
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import normwise_error

pytestmark = pytest.mark.gpu


def _compare(plan, ins):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    fused = B200Program(plan, device="cuda")
    plain = B200Program(plan, device="cuda", fuse_kernels=False)
    fams = [k.family for k in fused.kernel_sources]
    assert "copy" not in fams
    assert (any(k.info.get("a_strided") or k.info.get("b_strided") for k in fused.kernel_sources)
            or any(f in k.attrs for k in fused.xplan.kernels for f in ("a_gather", "b_gather")))
    assert "copy" in [k.family for k in plain.kernel_sources]
    y1, y0 = fused(*ins), plain(*ins)
    torch.cuda.synchronize()
    fused.check()
    plain.check()
    same_kernel = not any(k.info.get("pair") for k in plain.kernel_sources)
    return y1, y0, same_kernel


@pytest.mark.parametrize("case", ["merge_heads_linear__bf16", "merge_heads_linear__f16", "merge_heads_linear__f32",
                                  "transpose_bmm__bf16", "heads_scores__bf16", "heads_attention_probs__bf16"])
def test_folded_copy_matches_unfused_program(case):
    """``heads_attention_probs``: an attention whose probabilities are returned too, so it is not
    fused; its q / k / v head splits (v as the N-major B of P·V) and its head merge are folded.
    ``merge_heads_linear__f32``: the 3xTF32 split launch gathers A from the source (1e-4)."""
    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    ys1, ys0, same_kernel = _compare(plan, ins)
    for y1, y0, exp in zip(ys1, ys0, FX.case_expected(case)):
        assert torch.equal(y1, y0) if same_kernel else normwise_error(y1, y0) <= 1e-3
        tol = 1e-4 if case.endswith("__f32") else 2e-2
        assert FX.check_against_golden(y1, exp, tol) <= tol


@pytest.mark.parametrize("shape", [(8, 16, 2048, 64, 1024), (3, 4, 384, 64, 256)])
def test_folded_head_merge_at_size(shape):
    """Many 128-row tiles per batch element and several batch elements per GEMM (the transformer
    config's output projection: x[8, 16, 2048, 64] -> [16384, 1024] @ w[1024, 1024]ᵀ)."""
    B, H, S, D, N = shape
    plan = FX.merge_heads_plan(B, H, S, D, N)
    g = torch.Generator(device="cuda").manual_seed(5)
    x = torch.randn((B, H, S, D), generator=g, device="cuda").to(torch.bfloat16)
    w = (torch.randn((N, H * D), generator=g, device="cuda") * 0.03).to(torch.bfloat16)
    b = (torch.randn((N,), generator=g, device="cuda") * 0.1).to(torch.bfloat16)
    ys1, ys0, same_kernel = _compare(plan, [x, w, b])
    y1, y0 = ys1[0], ys0[0]
    assert torch.equal(y1, y0) if same_kernel else normwise_error(y1, y0) <= 1e-3
    ref = x.float().permute(0, 2, 1, 3).reshape(B * S, H * D) @ w.float().t() + b.float()
    assert normwise_error(y1, ref) <= 2e-2
