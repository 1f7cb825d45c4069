"""Host-side logic without a GPU: plan serialisation, the arena planner against
the reference planner's offsets, code generation and sm_100a compilation,
launch geometry, and the tensorjit registration hook."""
import math

import numpy as np

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
    # f32 matmuls with a K-major B run as 3xTF32: one launch splitting both operands + the tcgen05 GEMM
    assert [k.family for k in ks] == ["row", "split", "gemm_tc", "split", "gemm_tc"]
    assert [k.info["index"] for k in ks] == [0, 1, 1, 2, 2]
    assert all(k.info.get("tf32x3") for k in ks if k.family == "gemm_tc")
    # one row group per row, 256-thread CTAs
    assert ks[0].block[0] == 256 and ks[0].grid[0] * ks[0].info["rpc"] >= 64
    p16 = FX.load_plan("cuda_mlp__bf16")
    ks16 = generate(p16)
    assert [k.family for k in ks16] == ["row", "gemm_tc", "gemm_tc"]
    for k in ks16[1:]:
        assert k.block[0] in (192, 320) and len(k.tmaps) in (2, 3) and k.grid[0] <= 148


def test_every_matmul_runs_on_the_tensor_cores():
    """tests/test_cuda_backend.py:50-57 analogue (which matmuls reach the tensor cores): on B200
    all of them do.  Operands the tensor maps can read in place go straight to the tcgen05
    GEMM; a pitch that breaks the 16-byte TMA rule, or f32 / N-major operands on the 3xTF32
    path, get one pack / split launch first."""
    fam = lambda n: [k.family for k in generate(FX.load_plan(n)) if k.family in ("gemm_tc", "split")]
    assert fam("cuda_wmma__f16") == ["gemm_tc"]
    assert fam("cuda_wmma__bf16") == ["gemm_tc"]
    assert fam("cuda_wmma__f32") == ["split", "gemm_tc"]        # f32, K-major B: 3xTF32
    assert fam("gemm_tc_nn_batched__f32") == ["split", "gemm_tc"]   # f32 N-major B: transposed by the split
    assert fam("matmul_epi_7x13x5__bf16") == ["split", "gemm_tc"]   # K % 8 != 0: both packed
    assert fam("matmul_epi_33x128x65__bf16") == ["split", "gemm_tc"]  # N-major B with N % 8 != 0: B packed
    assert fam("gemm_tc_nn_batched__bf16") == ["gemm_tc"]       # N-major B read in place
    for case in FX.cases("case") + FX.cases("config"):
        for k in generate(FX.load_plan(case)):
            assert k.family in ("ewise", "copy", "row", "split", "gemm_tc", "attention"), (case, k.family)


def test_pack_prepass_layout():
    """The packed operands are K-major with the padded pitch, and the GEMM's tensor maps read
    them (not the plan's buffers) with that pitch."""
    from mlir_gpu_kernel_compiler_b200.codegen.gemm import gemm_form

    p = FX.load_plan("matmul_epi_7x13x5__bf16")          # A[7,13] @ B[13,5]: K = 13
    mm = [k for k in p.kernels if k.kind == "matmul"][0]
    f = gemm_form(mm)
    assert (f.mode, f.pack_a, f.pack_b, f.pitch, f.b_mn) == ("f16", True, True, 16, False)
    pk, g = generate(p)
    assert pk.args[1] == ("scratch", 0) and pk.args[4][0] == "scratch"
    assert pk.info["scratch_bytes"] == g.info["scratch_bytes"] > 0
    ta, tb = g.tmaps[0], g.tmaps[1]
    assert ta.dims == [13, 7] and ta.strides == [16 * 2] and tb.dims == [13, 5] and tb.strides == [16 * 2]
    n_in, n_out = len(mm.inputs), len(mm.outputs)
    assert g.args[ta.arg] == ("scratch", 0) and g.args[tb.arg] == pk.args[4]
    assert g.info["packed"] == ["a", "b"]
    # an N-major f32 B is transposed by the split into K-major hi / lo copies
    p2 = FX.load_plan("gemm_tc_nn_batched__f32")
    sp, g2 = generate(p2)
    assert "tile[tx][y]" in sp.source and g2.info["tf32x3"] and g2.tmaps[1].dims == [192, 6 * 64]


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


def test_pair_tiles_in_search_space_and_plain_gemm_plan(monkeypatch):
    from mlir_gpu_kernel_compiler_b200 import autotune as AT

    assert any(c.PAIR for c in AT.candidates(16384, False))
    assert not any(c.PAIR for c in AT.candidates(16384, True))      # N-major B: one CTA only
    monkeypatch.setenv("TENSORJIT_B200_PAIR", "0")
    assert not any(c.PAIR for c in AT.candidates(16384, False))
    monkeypatch.delenv("TENSORJIT_B200_PAIR")
    assert AT.parse_tile("256:5:16:1") == AT.TileConfig(256, 5, 16, True)
    assert AT.parse_tile("128:6") == AT.TileConfig(128, 6, 16, False)
    plan = AT.plain_gemm_plan(512, 1024, 256)
    ks = generate(plan, tiles={0: AT.parse_tile("256:5:16:1").as_dict()})
    assert [k.family for k in ks] == ["gemm_tc"]
    assert ks[0].cluster == (2, 1, 1) and ks[0].info["pair"] and ks[0].info["stages"] == 5
    assert ks[0].grid[0] == 2 * (512 // 256) * (1024 // 256)
    # shared memory of the deepest pair pipeline stays under the 227 KB opt-in limit
    deep = generate(AT.plain_gemm_plan(8192, 16384, 4096), tiles={0: AT.parse_tile("256:6:16:1").as_dict()})[0]
    assert deep.smem <= 232448


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


# -- attention fusion (fuse.py) ----------------------------------------------------------
def _fused(name):
    from mlir_gpu_kernel_compiler_b200.fuse import fuse_attention

    p = FX.load_plan(name)
    return p, fuse_attention(p)


@pytest.mark.parametrize("name,before,after", [
    ("attention_core__bf16", 3, 1), ("attention_ragged__bf16", 3, 1), ("attention_ragged__f16", 3, 1),
    ("attention_short__f16", 3, 1), ("attention_heads__bf16", 11, 5), ("cfg4", 16, 10)])
def test_attention_chains_fuse_and_fold_their_transposes(name, before, after):
    p, f = _fused(name)
    assert len(p.kernels) == before and len(f.kernels) == after
    att = [k for k in f.kernels if k.kind == "attention"]
    assert len(att) == 1
    a = att[0].attrs
    assert a["d"] == a["dv"] == 64 and a["scale"] > 0
    # no intermediate of the chain (scores, probabilities, folded copies) keeps arena storage
    mp = plan_memory(f)
    kept = {b.node.op for b in mp.buffers.values() if b.node is not att[0].outputs[0]}
    assert not kept & {"div", "exp", "max", "sum", "transpose"}
    assert mp.arena_bytes <= plan_memory(p).arena_bytes
    # the original plan is left untouched
    assert len(FX.load_plan(name).kernels) == len(p.kernels)


def test_cfg4_attention_reads_and_writes_the_head_split_layout():
    p, f = _fused("cfg4")
    a = [k for k in f.kernels if k.kind == "attention"][0].attrs
    # [8, 2048, 16, 64] matmul output viewed as [8, 16, 2048, 64]: (b, h, s, d) strides
    for name in ("q", "k", "v"):
        assert a[name][1] == (2048 * 16 * 64, 64, 16 * 64, 1)
    assert a["out"][0].op == "transpose" and a["out"][1] == (2048 * 16 * 64, 64, 16 * 64, 1)
    assert a["batch"] == (8, 16) and a["sq"] == a["sk"] == 2048 and a["scale"] == 0.125


def test_attention_not_fused_when_probabilities_escape(monkeypatch):
    p, f = _fused("attention_probs_escape__bf16")
    assert [k.kind for k in f.kernels] == ["matmul", "row", "matmul"]
    from mlir_gpu_kernel_compiler_b200.fuse import fuse

    monkeypatch.setenv("TENSORJIT_B200_FUSE", "0")
    p2 = FX.load_plan("attention_core__bf16")
    assert fuse(p2) is p2


def test_attention_not_fused_for_other_row_kernels():
    from mlir_gpu_kernel_compiler_b200.fuse import fuse_attention

    p = FX.load_plan("attention_core__bf16")
    row = p.kernels[1]
    ex = [n for n in row.nodes if n.op == "exp"][0]
    ex.op = "tanh"                     # not a softmax any more
    assert [k.kind for k in fuse_attention(p).kernels] == ["matmul", "row", "matmul"]


def test_attention_tensor_maps_and_launch_geometry():
    _, f = _fused("cfg4")
    ks = [k for k in generate(f) if k.family == "attention"][0]
    assert ks.grid == (128 * 8, 1, 1) and ks.block == (640, 1, 1)
    assert ks.smem <= 232448 and len(ks.tmaps) == 3
    for t in ks.tmaps:
        # head dim innermost, then heads, sequence, batch -- strides increasing, 16-byte multiples
        assert t.dims == [64, 16, 2048, 8] and t.box == [64, 1, 128, 1]
        assert t.strides == sorted(t.strides) and all(s % 16 == 0 for s in t.strides)
    _, f = _fused("attention_ragged__bf16")
    ks = [k for k in generate(f) if k.family == "attention"][0]
    assert ks.grid == (3, 1, 1)
    assert [t.dims for t in ks.tmaps] == [[64, 200, 3], [64, 300, 3], [64, 300, 3]]


@pytest.mark.parametrize("name", ["attention_core__bf16", "attention_ragged__f16", "attention_heads__bf16"])
def test_fused_attention_compiles_for_sm100a(name):
    from mlir_gpu_kernel_compiler_b200.toolchain import compile_cubins

    _, f = _fused(name)
    ks = generate(f)
    assert any(k.family == "attention" for k in ks)
    imgs = compile_cubins([(k.symbol, k.source) for k in ks])
    assert all(img[:4] == b"\x7fELF" for img in imgs)


@pytest.mark.parametrize("knobs,header,threads,kv_rows", [("SPLIT=1", "attention_split_sm100.cuh", 640, 128),
                                                          ("ROW=1,STAGES=6", "attention_row_sm100.cuh", 384, 64),
                                                          ("F2=1", "attention_sm100.cuh", 640, 128)])
def test_attention_kernel_variants_generate_and_compile(knobs, header, threads, kv_rows, monkeypatch):
    """The split-row and one-thread-per-row attention kernels (``TENSORJIT_B200_ATTN``) build for
    sm_100a with their own launch shape and K/V tensor-map boxes."""
    from mlir_gpu_kernel_compiler_b200.toolchain import compile_cubins

    monkeypatch.setenv("TENSORJIT_B200_ATTN", knobs)
    _, f = _fused("attention_ragged__f16")
    (k,) = [k for k in generate(f) if k.family == "attention"]
    assert f'#include "{header}"' in k.source and k.block == (threads, 1, 1)
    assert k.tmaps[0].box[-2 if len(k.tmaps[0].box) > 2 else 1] == 128
    assert all(kv_rows in t.box for t in k.tmaps[1:])
    assert compile_cubins([(k.symbol, k.source)])[0][:4] == b"\x7fELF"


def _ex2_poly_f32(x):
    """numpy float32 restatement of ex2_poly (csrc/kernels/attention_sm100.cuh)."""
    x = np.maximum(np.asarray(x, np.float32), np.float32(-126.0))
    magic = np.float32(12582912.0)
    t = (x + magic).astype(np.float32)
    f = (x - (t - magic)).astype(np.float32)
    c3, c2, c1, c0 = (np.float32(v) for v in (0.05522261559963226, 0.24261537194252014, 0.6932516098022461,
                                              0.9999275803565979))
    p = ((c3 * f + c2) * f + c1) * f + c0
    bits = p.view(np.int32) + (t.view(np.int32) << np.int32(23))
    return bits.view(np.float32)


def test_polynomial_exp2_is_below_half_an_ulp_of_bf16_and_f16():
    x = np.concatenate([np.linspace(-30.0, 8.0, 400001), -np.logspace(-6, 1.5, 2000)]).astype(np.float32)
    y = _ex2_poly_f32(x).astype(np.float64)
    ref = np.exp2(x.astype(np.float64))
    rel = np.abs(y / ref - 1.0)
    assert rel.max() < 1e-4          # bf16 half-ulp 2^-9, f16 half-ulp 2^-12 = 2.4e-4
    # masked keys (-inf) and far-below-range arguments vanish after rounding to half precision
    tiny = _ex2_poly_f32(np.array([-np.inf, -200.0, -127.0], np.float32))
    assert np.all(tiny < 2.0 ** -125) and np.all(tiny >= 0)


def test_x3_gemm_with_few_tiles_is_split_over_k():
    """cfg1's second GEMM (512 x 768, K = 3072) has 24 output tiles of 128 x 128: six K slices
    write partial sums into the workspace and a finalize launch adds them and applies the
    epilogue; the first (K = 768, 96 tiles) fills one wave unsplit."""
    ks = generate(FX.load_plan("cfg1"))
    assert [k.family for k in ks] == ["row", "split", "gemm_tc", "split", "gemm_tc", "ewise"]
    g1, g2, fin = ks[2], ks[4], ks[5]
    assert (g1.info["BN"], g1.info["ksplit"], g1.grid[0]) == (128, 1, 96)
    assert (g2.info["BN"], g2.info["ksplit"], g2.grid[0]) == (128, 6, 144) and "KSPLIT = 6" in g2.source
    assert fin.info["ksplit"] == 6 and fin.args == g2.args and fin.info["index"] == g2.info["index"] == 2
    # ragged N: scalar partial stores; 1 x 3 tiles of 128 x 64, K = 2048 -> eight slices
    ks = generate(FX.load_plan("linear_splitk_ragged__f32"))
    g = [k for k in ks if k.family == "gemm_tc"][0]
    assert g.info["ksplit"] == 8 and "row[j + u] = acc[c + u]" in g.source


def test_gemms_sharing_a_become_one_launch():
    from mlir_gpu_kernel_compiler_b200.fuse import fuse

    p = fuse(FX.load_plan("shared_a_projections__bf16"))
    assert [k.kind for k in p.kernels] == ["matmul_multi"]
    k = p.kernels[0]
    assert [n for _b, _o, n in k.attrs["parts"]] == [256, 512, 256] and len(k.outputs) == 3
    ks = generate(p)[0]
    assert ks.family == "gemm_tc" and ks.info["segments"] == 3 and ks.info["N"] == 1024
    assert len(ks.tmaps) == 4 and [t.dims[1] for t in ks.tmaps[1:]] == [256, 512, 256]
    # on a CTA pair (M = 300 >= one 256-row tile): each CTA loads 128 rows of every B tile;
    # 2 row tiles x 4 column tiles of 256 -> 8 clusters
    assert ks.info["pair"] and ks.cluster == (2, 1, 1) and ks.grid[0] == 16
    assert all(t.box[1] == 128 for t in ks.tmaps[1:]) and "gemm_sm100_pair<Cfg>" in ks.source
    single = generate(p, tiles={0: {"BN": 256, "STAGES": 4, "GROUP_M": 16, "PAIR": False}})[0]
    assert not single.info["pair"] and single.cluster == (1, 1, 1) and single.tmaps[1].box[1] == 256
    # cfg4: the q, k, v projections (same LayerNorm output) -> one launch; with the attention chain
    # and the residual add folded as well, 16 plan kernels -> 7
    p4 = fuse(FX.load_plan("cfg4"))
    assert [k.kind for k in p4.kernels] == ["row", "matmul_multi", "attention", "matmul", "row", "matmul",
                                           "matmul"]
    # a GEMM with an epilogue, or N not a multiple of the 256-column tile, is left alone
    p5 = fuse(FX.load_plan("attention_heads__bf16"))
    assert "matmul_multi" not in [k.kind for k in p5.kernels]


def test_fast_gelu_for_half_precision_outputs_tracks_erf_gelu():
    """numpy float32 restatement of tj_gelu_fast (csrc/kernels/tj_common.cuh) against the
    exact erf GELU: relative error below half an ulp of bf16 (2^-9) wherever the output is
    not negligible, the negative tail included; saturation to x / -0 for large |x|."""
    import math

    c = [np.float32(v) for v in (2.2976467609405518, 0.10939675569534302, -0.0014235572889447212,
                                 1.303200679103611e-05)]

    def gelu_fast(x):
        x = x.astype(np.float32)
        y = x * x
        p = ((c[3] * y + c[2]) * y + c[1]) * y + c[0]
        with np.errstate(over="ignore"):
            return (x / (np.float32(1.0) + np.exp2(-(x * p)))).astype(np.float32)

    x = np.linspace(-12.0, 12.0, 60001).astype(np.float32)
    y = gelu_fast(x).astype(np.float64)
    ref = np.array([0.5 * v * (1.0 + math.erf(v / math.sqrt(2.0))) for v in x.astype(np.float64)])
    assert np.abs(y - ref).max() < 1.7e-4
    big = np.abs(ref) > 1e-6
    assert (np.abs(y - ref)[big] / np.abs(ref[big])).max() < 1.4e-3 < 2.0 ** -9
    pos = x > 0                                            # below half an f16 ulp there
    assert (np.abs(y - ref)[pos] / np.abs(ref[pos])).max() < 3.9e-4 < 2.0 ** -11
    # the exponent polynomial is increasing, so Phi is monotone and saturates correctly
    xs = np.linspace(0.0, 40.0, 100001).astype(np.float32)
    g = xs * (((c[3] * xs * xs + c[2]) * xs * xs + c[1]) * xs * xs + c[0])
    assert np.all(np.diff(g) > 0)
    assert list(gelu_fast(np.array([-1e30, -50.0, 50.0, 1e30], np.float32))) == [0.0, 0.0, 50.0, 1e30]
    # used only where every stored value is half precision
    from mlir_gpu_kernel_compiler_b200.codegen.common import EXPR, EXPR_FAST

    assert "fast" in EXPR_FAST["gelu"] and "erff" not in EXPR_FAST["gelu"] and EXPR["gelu"] == "tj_gelu({0})"


def test_compile_batch_with_repeated_source(tmp_path, monkeypatch):
    """A batch naming one kernel source twice (the fused and the plan-as-given program often
    share kernels) compiles it once; both entries get the same cubin, the cache holds no
    temporary files."""
    from mlir_gpu_kernel_compiler_b200 import toolchain as TC

    monkeypatch.setenv("TENSORJIT_B200_CACHE_DIR", str(tmp_path))
    src = 'extern "C" __global__ void tj_probe(float* p) { p[threadIdx.x] += 1.0f; }\n'
    a, b, c = TC.compile_cubins([("x", src), ("y", src), ("z", src.replace("1.0f", "2.0f"))])
    assert a == b and a[:4] == b"\x7fELF" and c != a
    suffixes = [p.suffix for p in tmp_path.iterdir()]
    assert suffixes.count(".cubin") == 2 and ".tmp" not in suffixes


def test_checked_build_bounds_checks_every_kernel_family():
    """TENSORJIT_B200_CHECKED: every generated kernel gets the status words and declares its
    global operands as bounded views (element counts baked in); the GEMM and attention
    templates receive the operand extents their coordinate checks use.  The normal build
    contains none of it."""
    from mlir_gpu_kernel_compiler_b200.fuse import fuse

    seen = set()
    for case in ("cuda_rows__f32", "ew_chain_8x33__bf16", "cfg1", "matmul_epi_7x13x5__bf16",
                 "linear_splitk_ragged__f32", "attention_heads__bf16", "shared_a_projections__bf16",
                 "matmul_epi_1x1x1__f32"):
        plan = fuse(FX.load_plan(case))
        plain = generate(plan)
        chk = generate(plan, checked=True)
        assert [k.symbol for k in plain] == [k.symbol for k in chk]
        for k0, k1 in zip(plain, chk):
            seen.add(k1.family)
            assert "tj_view" not in k0.source and "tj_status" not in k0.source
            assert ("status", None) in k1.args
            if k1.family in ("ewise", "copy", "row", "split"):
                assert "tj_view<" in k1.source or "tj_check(" in k1.source, (case, k1.symbol)
            if k1.family == "gemm_tc":
                assert "A_MATS" in k1.source
            if k1.family == "attention":
                assert "O_NUMEL" in k1.source
            k1.finalize_params()
            assert k1.param_bytes >= 8 * len(k1.args)
    assert {"ewise", "row", "split", "gemm_tc", "attention"} <= seen


def test_residual_add_after_a_gemm_joins_its_epilogue():
    """The elementwise kernel after the MLP's down projection (the residual add, planned on its
    own because x1 also feeds the LayerNorm) is evaluated in that GEMM's epilogue; a kernel that
    is not only post-processing the GEMM output is left alone."""
    from mlir_gpu_kernel_compiler_b200.fuse import absorb_elementwise_epilogues, fuse

    for case in ("block_tail__f32", "block_tail__bf16", "cfg4"):
        p = FX.load_plan(case)
        f = fuse(p)
        assert f.meta.get("absorbed_epilogues") == 1
        last = f.kernels[-1]
        assert last.kind == "matmul" and [o.id for o in last.outputs] == [p.resolve(p.outputs[0]).id]
        assert len(f.kernels) == len(p.kernels) - 1 - (len(p.kernels) - 8 if case == "cfg4" else 0)
        assert generate(f)[-1].info["kind"] == "matmul"      # the GEMM (or its split-K finalize) is last
    # the GEMM output also escapes as a graph output: nothing to absorb
    assert absorb_elementwise_epilogues(FX.load_plan("cuda_mlp__bf16")).meta.get("absorbed_epilogues") is None


def test_every_kernel_waits_for_its_predecessor_before_touching_memory():
    """Programmatic dependent launch: a kernel may start while the previous one of the program
    finishes, so each one must wait (griddepcontrol.wait) before its first global access.  The
    generated kernels do it first thing; the GEMM and attention templates right after their
    set-up (barrier init, TMEM allocation), before their roles start."""
    from mlir_gpu_kernel_compiler_b200.fuse import fuse
    from mlir_gpu_kernel_compiler_b200.toolchain import KDIR

    import re

    early_seen = 0
    for case in FX.cases("case") + FX.cases("config"):
        for k in generate(fuse(FX.load_plan(case))):
            if k.family in ("gemm_tc", "attention"):
                continue
            body = k.source.split("Params prm) {", 1)[1]
            if not k.info.get("early_segments"):
                assert body.lstrip().startswith("tj_pdl_launch_dependents();\n  tj_pdl_wait();"), (case, k.symbol)
                continue
            # a pre-pass may touch the segments that are program inputs before its wait, no others
            assert k.family == "split" and body.lstrip().startswith("tj_pdl_launch_dependents();"), (case, k.symbol)
            pre = body[:body.index("tj_pdl_wait();")]
            loops = pre[pre.index("for ("):]
            segs = {int(i) // 3 for i in re.findall(r"prm\.p\[(\d+)\]", loops)}
            segs |= {int(i) for i in re.findall(r"\b(?:src|hi|lo)(\d+)\[", loops)}
            inputs = {j for j in range(len(k.args) // 3) if k.args[3 * j][0] == "node"
                      and k.args[3 * j][1].op == "input"}
            assert segs and segs <= inputs, (case, k.symbol, segs, inputs)
            early_seen += 1
    assert early_seen > 0
    for hdr in ("gemm_sm100.cuh", "gemm_sm100_pair.cuh", "attention_sm100.cuh", "attention_split_sm100.cuh",
                "attention_row_sm100.cuh", "attention_quad_sm100.cuh"):
        src = (KDIR / hdr).read_text()
        setup_end = src.index("const uint32_t tmem_base = *tmem_slot;")
        assert src.index("tj_pdl_wait();", setup_end) < src.index("if (warp == 0)", setup_end), hdr


def test_peer_output_programs_store_without_tma():
    """A program whose output rows may be a peer GPU's memory (``peer_outputs``) keeps every GEMM
    epilogue on plain 16-byte stores: no output tensor map, same kernels otherwise."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    plan = FX.load_plan("cfg5_m1024")
    normal = [k for k in generate(plan) if k.family == "gemm_tc"]
    peer = [k for k in generate(plan, tma_store=False) if k.family == "gemm_tc"]
    assert any(k.info["tma_store"] for k in normal)
    assert not any(k.info["tma_store"] for k in peer)
    assert [len(k.tmaps) for k in peer] == [len(k.tmaps) - int(k.info["tma_store"]) for k in normal]
    assert "TMA_STORE = false" in peer[-1].source
    assert all(k.info["staged_store"] for k in peer) and not any(k.info["staged_store"] for k in normal)
    prog = B200Program(plan, device="cuda", peer_outputs=False)
    with pytest.raises(ValueError, match="peer_outputs"):
        prog.run_into([], [1 << 40])


def test_3xtf32_operand_forwarding(monkeypatch):
    """cfg1: the LayerNorm writes its output as the first GEMM's TF32 hi / lo A operand, and the
    first GEMM's GELU epilogue writes h as the second GEMM's; the split launches keep only the
    weights (program inputs, split before the wait).  Forwarding stops where the operand has
    another reader or is a program output."""
    plan = FX.load_plan("cfg1")
    assert not any(k.info.get("forwarded_outputs") for k in generate(plan))     # off by default
    monkeypatch.setenv("TENSORJIT_B200_FORWARD", "1")
    ks = generate(plan)
    row, sp1, g1, sp2, g2 = ks[:5]
    assert [k.family for k in ks] == ["row", "split", "gemm_tc", "split", "gemm_tc", "ewise"]
    assert row.info["forwarded_outputs"] and g1.info["forwarded_outputs"]
    assert g1.info["x3_forwarded"] == ["a"] and g2.info["x3_forwarded"] == ["a"]
    for sp in (sp1, sp2):       # one segment each, the weight, handled before the wait
        assert len(sp.args) == 3 and sp.args[0][1].op == "input" and sp.info["early_segments"] == 1
    # the row kernel's output argument is the first GEMM's A hi copy, the GEMM's h argument the second's
    assert ("scratch", g1.info["scratch_base"] + g1.info["x3_vec"]["a"][1]) in row.args
    assert ("scratch", g2.info["scratch_base"] + g2.info["x3_vec"]["a"][1]) in g1.args
    assert "tj_tf32_hi" in row.source and "tj_tf32_hi" in g1.source
    # the hi -> lo distance in the stores equals the consumer's layout
    a_hi, a_lo = g1.info["x3_vec"]["a"][1:]
    assert f"+ {(a_lo - a_hi) // 4}L" in row.source
    # a program output is never forwarded: the plan with x_ln also returned keeps its split
    from mlir_gpu_kernel_compiler_b200.codegen import _split_forwarding

    first = generate(plan)
    fwd, skip = _split_forwarding(plan, first)
    xln = plan.kernels[0].outputs[0]
    assert xln.id in fwd and skip == {1: {"a"}, 2: {"a"}}
    plan.outputs.append(xln)
    fwd2, skip2 = _split_forwarding(plan, first)
    assert xln.id not in fwd2 and 1 not in skip2


def test_pdl_chosen_per_program(monkeypatch):
    """Programmatic dependent launch: on for latency-bound programs (short estimated run time),
    off for programs of long persistent GEMMs, where it cost clock under the power cap;
    TENSORJIT_B200_PDL forces either way, and the constructor argument overrides the estimate."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    monkeypatch.delenv("TENSORJIT_B200_PDL", raising=False)
    assert B200Program(FX.load_plan("cfg4"), device="cuda").pdl
    assert B200Program(FX.load_plan("cfg1"), device="cuda").pdl
    big = B200Program(FX.load_plan("cfg5_m131072"), device="cuda")
    assert not big.pdl and big.estimated_ms() > 10
    assert B200Program(FX.load_plan("cfg5_m131072"), device="cuda", pdl=True).pdl
    monkeypatch.setenv("TENSORJIT_B200_PDL", "1")
    assert B200Program(FX.load_plan("cfg5_m131072"), device="cuda").pdl
    monkeypatch.setenv("TENSORJIT_B200_PDL", "0")
    assert not B200Program(FX.load_plan("cfg4"), device="cuda").pdl


def test_transpose_copy_folded_into_gemm_operand():
    """A transpose copy kernel that only feeds a bf16/f16 GEMM's A operand disappears: the GEMM
    reads A from the transpose's source through a tensor map whose dims are ordered by stride,
    with the 64-column k-block and the 128-row tile as the only box extents above 1."""
    from mlir_gpu_kernel_compiler_b200.fuse import fuse, strided_a_layout

    f = fuse(FX.load_plan("merge_heads_linear__bf16"))
    assert [k.kind for k in f.kernels] == ["matmul"] and f.meta["folded_copies"] == 1
    (g,) = generate(f)
    assert g.info["a_strided"] and not g.info["pair"] and "A_RANK = 4" in g.source
    tm = g.tmaps[0]
    assert tm.dims == [64, 256, 4, 2] and tm.box == [64, 128, 1, 1]        # d, s, h, b of x[2, 4, 256, 64]
    assert tm.strides == sorted(tm.strides) == [64 * 2, 256 * 64 * 2, 4 * 256 * 64 * 2]
    assert g.args[tm.arg][1].op == "input"                                  # the source x, not the transpose
    # batch-dim transpose before a batched matmul: rank 3, the batch coordinate from the GEMM's batch
    (g2,) = generate(fuse(FX.load_plan("transpose_bmm__bf16")))
    assert g2.tmaps[0].dims == [128, 4, 256] and g2.tmaps[0].box == [64, 1, 128] and "A_RANK = 3" in g2.source
    # unfused attention scores: A (q) and the K-major B (k) both read from the projection outputs,
    # each through a rank-4 map with two batch dims (head, batch) split from the batch index
    hs = fuse(FX.load_plan("heads_scores__bf16"))
    assert [k.kind for k in hs.kernels] == ["matmul"] * 3 and hs.meta["folded_copies"] == 2
    g3 = generate(hs)[-1]
    assert g3.info["a_strided"] and g3.info["b_strided"] and "A_RANK = 4" in g3.source and "B_RANK = 4" in g3.source
    assert g3.tmaps[0].dims == g3.tmaps[1].dims == [64, 4, 256, 2] and g3.tmaps[1].box[2] == g3.info["BN"]
    assert "c[1] = static_cast<int>(ab % 4L);" in g3.source and "c[3] = static_cast<int>(bb / 4L);" in g3.source
    # an unfused attention (probabilities returned): all four copies folded, v as the N-major B of
    # P·V read in 64 x 64 chunks (n first) from the v projection's output
    ha = fuse(FX.load_plan("heads_attention_probs__bf16"))
    assert [k.kind for k in ha.kernels] == ["matmul"] * 4 + ["row", "matmul", "matmul"]
    assert ha.meta["folded_copies"] == 4
    pv = [g for g in generate(ha) if g.family == "gemm_tc"][-2]
    assert pv.info["b_strided"] and "B_FOLDED = true" in pv.source and pv.tmaps[1].box == [64, 1, 64, 1]
    # f32 (3xTF32): the split launch gathers A from the transpose's source instead of a tensor map
    f32 = fuse(FX.load_plan("merge_heads_linear__f32"))
    assert [k.kind for k in f32.kernels] == ["matmul"] and "a_gather" in f32.kernels[0].attrs
    sp = generate(f32)[0]
    assert sp.family == "split" and sp.args[0][1].op == "input"
    assert "(kk % 64L) + (kk / 64L) * 16384L + (r % 256L) * 64L + (r / 256L) * 65536L" in sp.source
    # kept as a copy: a 128-row tile that would straddle two batch elements (seq 200), a K block
    # that would straddle two heads (head dim 32)
    for shape in ((2, 4, 200, 64, 128), (2, 8, 256, 32, 128)):
        p = FX.merge_heads_plan(*shape)
        assert [k.kind for k in fuse(p).kernels] == ["copy", "matmul"], shape
    ok = FX.merge_heads_plan(8, 16, 2048, 64, 1024)                            # the transformer config's merge
    assert strided_a_layout(ok, ok.kernels[1], set()) is not None
    # the transpose is also a program output: kept
    esc = FX.load_plan("merge_heads_linear__bf16")
    esc.outputs.append(esc.kernels[0].outputs[0])
    assert [k.kind for k in fuse(esc).kernels] == ["copy", "matmul"]


def test_folded_transpose_gemm_fits_on_one_cta():
    """The transformer config's head merge + output projection: its tuned tile is a CTA pair,
    which a folded transpose cannot use; the single-CTA kernel then keeps the stages that fit."""
    from mlir_gpu_kernel_compiler_b200 import B200Program

    p = B200Program(FX.merge_heads_plan(8, 16, 2048, 64, 1024), device="cuda")
    (k,) = p.kernel_sources
    assert k.info["a_strided"] and not k.info["pair"] and k.smem <= 232448 and k.info["stages"] >= 2
