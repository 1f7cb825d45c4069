"""Host-side logic without a GPU: plan serialisation, the arena planner against
the reference planner's offsets, code generation and sm_100a compilation,
launch geometry, and the tensorjit registration hook."""
import json
import math

import pytest

from mlir_gpu_kernel_compiler_b200.codegen import generate
from mlir_gpu_kernel_compiler_b200.memory import plan_memory
from mlir_gpu_kernel_compiler_b200.plan import PProgram
from oracle import fixtures as FX

ALL = FX.cases("case") + FX.cases("plan")


@pytest.mark.parametrize("name", ALL)
def test_plan_roundtrip_and_arena_matches_reference(name):
    p = FX.load_plan(name)
    q = PProgram.from_json(p.to_json())
    assert [k.kind for k in q.kernels] == [k.kind for k in p.kernels]
    assert [[n.id for n in k.nodes] for k in q.kernels] == [[n.id for n in k.nodes] for k in p.kernels]
    mp = plan_memory(p)
    assert mp.arena_bytes == p.meta["reference_arena_bytes"]
    ref = {int(k): v for k, v in p.meta["reference_offsets"].items()}
    assert {nid: b.offset for nid, b in mp.buffers.items()} == ref
    assert all(b.offset % 64 == 0 for b in mp.buffers.values())


def test_planner_never_overlaps_live_buffers():
    mp = plan_memory(FX.load_plan("cfg4"))
    bs = list(mp.buffers.values())
    for i, a in enumerate(bs):
        for b in bs[i + 1:]:
            live = not (a.last < b.first or b.last < a.first)
            over = not (a.offset + a.size <= b.offset or b.offset + b.size <= a.offset)
            assert not (live and over)
    assert mp.savings > 0.1


def test_launch_geometry_and_kernel_families():
    """tests/test_cuda_backend.py:60-65: plan kinds and launch grids of the MLP case."""
    p = FX.load_plan("cuda_mlp__f32")
    assert [k.kind for k in p.kernels] == ["row", "matmul", "matmul"]
    ks = generate(p)
    # f32 matmuls with a K-major B run as 3xTF32: two operand-split launches + the tcgen05 GEMM
    assert [k.family for k in ks] == ["row", "split", "split", "gemm_tc", "split", "split", "gemm_tc"]
    assert [k.info["index"] for k in ks] == [0, 1, 1, 1, 2, 2, 2]
    assert all(k.info.get("tf32x3") for k in ks if k.family == "gemm_tc")
    # one row group per row, 256-thread CTAs
    assert ks[0].block[0] == 256 and ks[0].grid[0] * ks[0].info["rpc"] >= 64
    p16 = FX.load_plan("cuda_mlp__bf16")
    ks16 = generate(p16)
    assert [k.family for k in ks16] == ["row", "gemm_tc", "gemm_tc"]
    for k in ks16[1:]:
        assert k.block[0] in (192, 320) and len(k.tmaps) in (2, 3) and k.grid[0] <= 148


def test_tensor_core_path_only_for_half_precision_with_aligned_pitch():
    """tests/test_cuda_backend.py:50-57 analogue: tcgen05 for bf16/f16 when TMA pitches allow."""
    fam = lambda n: [k.family for k in generate(FX.load_plan(n)) if k.family.startswith("gemm")]
    assert fam("cuda_wmma__f16") == ["gemm_tc"]
    assert fam("cuda_wmma__bf16") == ["gemm_tc"]
    assert fam("cuda_wmma__f32") == ["gemm_tc"]                 # f32, K-major B: 3xTF32
    assert fam("gemm_tc_nn_batched__f32") == ["gemm_simt"]      # f32 with an N-major B
    assert fam("matmul_epi_7x13x5__bf16") == ["gemm_simt"]       # K % 8 != 0
    assert fam("matmul_epi_33x128x65__bf16") == ["gemm_simt"]    # N-major B with N % 8 != 0
    assert fam("gemm_tc_nn_batched__bf16") == ["gemm_tc"]


def test_vectorised_paths_selected():
    cfg2 = generate(FX.load_plan("cfg2"))
    assert all(k.family == "row" and k.info["vec"] == 8 for k in cfg2)
    cfg4 = generate(FX.load_plan("cfg4"))
    copies = [k for k in cfg4 if k.family == "copy"]
    assert len(copies) == 4 and all(k.info["vec"] == 8 for k in copies)
    assert [k.family for k in cfg4].count("gemm_tc") == 8


def test_param_block_layout():
    for name in ("cfg3", "cfg1", "cfg4"):
        for k in generate(FX.load_plan(name)):
            n = len(k.args)
            if k.tmaps:
                assert k.tmaps[0].param_offset == math.ceil(8 * n / 64) * 64
                assert k.param_bytes == k.tmaps[-1].param_offset + 128
            else:
                assert k.param_bytes == 8 * n


@pytest.mark.parametrize("name", ["cuda_mlp__bf16", "cfg4", "rows_odd__f32", "transpose_2d__bf16",
                                  "gemm_tc_nn_batched__bf16", "empty_rows__f32"])
def test_kernels_compile_for_sm100a(name):
    from mlir_gpu_kernel_compiler_b200.toolchain import compile_cubins

    ks = generate(FX.load_plan(name))
    imgs = compile_cubins([(k.symbol, k.source) for k in ks])
    assert all(img[:4] == b"\x7fELF" for img in imgs)


def test_corrupt_cubin_cache_entry_is_rebuilt(tmp_path, monkeypatch):
    from mlir_gpu_kernel_compiler_b200 import toolchain

    monkeypatch.setenv("TENSORJIT_B200_CACHE_DIR", str(tmp_path))
    ks = generate(FX.load_plan("unary_gelu__f32"))[0]
    img = toolchain.compile_cubin(ks.source, ks.symbol)
    key = toolchain.source_key(ks.source)
    (tmp_path / f"{key}.cubin").write_bytes(b"garbage")
    img2 = toolchain.compile_cubin(ks.source, ks.symbol)
    assert img2[:4] == b"\x7fELF" and len(img2) == len(img)


def test_unsupported_kernel_kind_raises():
    p = FX.load_plan("unary_gelu__f32")
    p.kernels[0].kind = "scan"
    with pytest.raises(NotImplementedError):
        generate(p)


def test_autotune_space_and_cost_model():
    from mlir_gpu_kernel_compiler_b200 import autotune as AT

    c = AT.candidates(16384, False)
    assert {x.BN for x in c} >= {64, 128, 256}
    best = AT.pick(8192, 16384, 4096, 1, False)
    assert best.BN == 256
    small = AT.pick(128, 64, 64, 1, True)
    assert small.BN == 64
    tiles = AT.tiles_for_plan(FX.load_plan("cfg5_m131072"))
    assert set(tiles) == {1, 2}


def test_output_pool_reuses_only_dropped_buffers():
    """tests/test_backends.py:190-206 semantics, on host tensors."""
    import torch

    from mlir_gpu_kernel_compiler_b200.program import OutputPool

    p = OutputPool()
    a = p.take((4, 4), torch.float32, "cpu")
    view = a[:2]
    b = p.take((4, 4), torch.float32, "cpu")
    assert a.data_ptr() != b.data_ptr()
    del view
    c = p.take((4, 4), torch.float32, "cpu")
    assert c.data_ptr() not in (a.data_ptr(), b.data_ptr())
    pa = a.data_ptr()
    del a
    d = p.take((4, 4), torch.float32, "cpu")
    assert d.data_ptr() == pa


def test_bf16_storage_emulation_in_oracle():
    from oracle.plan_oracle import evaluate, normwise_error

    plan = FX.load_plan("cuda_mlp__bf16")
    ins = FX.case_inputs("cuda_mlp__bf16")
    a = evaluate(plan, ins)[0]
    b = evaluate(plan, ins, round_stored=True)[0]
    assert 0 < normwise_error(b, a) < 1e-2


def test_x3_workspace_follows_the_planned_arena():
    from mlir_gpu_kernel_compiler_b200.program import B200Program

    prog = B200Program(FX.load_plan("cfg1"))
    assert prog.ws_base >= prog.plan.arena_bytes and prog.ws_base % 256 == 0
    a_bytes = 512 * 3072 * 4        # the larger A operand (h1) of the second GEMM
    assert prog.workspace_bytes >= 2 * a_bytes
    scratch = [v for (kind, v), L in zip(prog._args, [None] * len(prog._args)) if kind == 1 and v >= prog.ws_base]
    assert scratch and max(scratch) < prog.arena_bytes
