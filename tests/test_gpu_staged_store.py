"""Staged epilogue stores against the per-row stores, on one GPU.

First, the plain-store epilogue of programs built for peer outputs (``peer_outputs=True``, used when
a row shard's output is another GPU's memory) against the ordinary program on one GPU.

Those GEMMs stage each warp's 32-row block in shared memory, as the TMA-store path does, and
write it back with plain coalesced 16-byte stores (two 32-column chunks as 128-byte row
segments, a lone chunk as 64-byte ones).  The stored values are the same, so the output must be
the same bits, for ragged row counts, column counts that end inside a chunk, batched and
broadcast GEMMs, single-CTA and CTA-pair tiles.  Second, the last-tile staging of f32 outputs and
split-K partial sums through the idle pipeline memory.
"""
import pytest
import torch

from oracle import fixtures as FX

pytestmark = pytest.mark.gpu

CASES = ["attention_heads__bf16", "attention_probs_escape__bf16", "block_tail__bf16", "bmm_broadcast__bf16",
         "cuda_mlp__bf16", "cuda_wmma__f16", "gemm_tc_aligned__bf16", "gemm_tc_batched_tb__bf16",
         "gemm_tc_multiwave__bf16", "gemm_tc_nn_batched__bf16", "linear_tb__bf16", "matmul_epi_64x64x64__bf16",
         "transformer_block__bf16"]


def _both(case: str):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    plan = FX.load_plan(case)
    ins = [t.cuda() for t in FX.case_inputs(case)]
    regular = B200Program(plan, device="cuda")
    peer = B200Program(plan, device="cuda", peer_outputs=True)
    assert any(ks.info.get("staged_store") for ks in peer.kernel_sources)
    assert not any(ks.info.get("tma_store") for ks in peer.kernel_sources)
    a, b = regular(*ins), peer(*ins)
    torch.cuda.synchronize()
    regular.check()
    peer.check()
    return a, b


@pytest.mark.parametrize("case", CASES)
def test_staged_plain_stores_match_the_ordinary_program(case):
    a, b = _both(case)
    for x, y in zip(a, b):
        assert torch.equal(x, y), case


@pytest.mark.parametrize("case", ["gemm_tc_multiwave__bf16", "block_tail__bf16", "gemm_tc_aligned__bf16"])
def test_staged_plain_stores_on_cta_pairs(case, monkeypatch):
    monkeypatch.setenv("TENSORJIT_B200_TILE", "256:5:16:1")
    a, b = _both(case)
    for x, y in zip(a, b):
        assert torch.equal(x, y), case


def test_staged_plain_stores_cfg5_shard():
    """The cfg5 row-shard program (CTA-pair GEMMs, 1024 rows) with plain stores: bit-identical
    to the ordinary program and within tolerance of the reference's golden rows."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W

    w = W.WORKLOADS["cfg5"]
    ins = W.make_inputs(w, device="cuda", rows=(0, 1024))
    plan = FX.load_plan("cfg5_m1024")
    y0 = B200Program(plan, device="cuda")(*ins)[0]
    peer = B200Program(plan, device="cuda", peer_outputs=True)
    assert [ks.info.get("pair") for ks in peer.kernel_sources if ks.family == "gemm_tc"] == [True, True]
    y1 = peer(*ins)[0]
    torch.cuda.synchronize()
    peer.check()
    assert torch.equal(y0, y1)
    assert FX.check_against_golden(y1, FX.case_expected("cfg5_m1024")[0], 2e-2) <= 2e-2


F32_CASES = ["block_tail__f32", "bmm_broadcast__f32", "cuda_mlp__f32", "gemm_tc_aligned__f32",
             "gemm_tc_batched_tb__f32", "gemm_tc_nn_batched__f32", "linear_tb__f32", "matmul_epi_64x64x64__f32",
             "transformer_block__f32", "cfg1"]


@pytest.mark.parametrize("case", F32_CASES)
def test_last_tile_staged_f32_stores_are_bit_identical(case, monkeypatch):
    """f32 outputs and split-K partial sums of a CTA's last tile go through the idle pipeline
    memory and out as whole row segments; the values are the same, so the outputs must be the
    same bits as with the per-row stores (``TENSORJIT_B200_STAGE_LAST=0``).  By default only the
    partial sums are staged; ``all`` stages the f32 outputs with an epilogue as well."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W

    if case == "cfg1":
        plan, ins = FX.load_plan("cfg1"), [t.cuda() for t in W.make_inputs(W.WORKLOADS["cfg1"])]
    else:
        plan, ins = FX.load_plan(case), [t.cuda() for t in FX.case_inputs(case)]
    outs = {}
    for flag in ("0", "1", "all"):
        monkeypatch.setenv("TENSORJIT_B200_STAGE_LAST", flag)
        prog = B200Program(plan, device="cuda")
        staged = [k for k in prog.kernel_sources if k.info.get("stage_last")]
        assert (not staged) if flag == "0" else all(k.info["ksplit"] > 1 or flag == "all" for k in staged)
        if flag == "all":
            assert staged
        outs[flag] = prog(*ins)
        torch.cuda.synchronize()
        prog.check()
    for flag in ("1", "all"):
        for a, b in zip(outs["0"], outs[flag]):
            assert torch.equal(a, b), (case, flag)
