"""Every operand form of a plan matmul on the tcgen05 GEMM, against an fp64 PyTorch matmul.

A matmul whose operands the tensor maps can read in place (16-byte row pitch) runs the
kernel directly; the others get a pack (bf16/f16) or split (3xTF32) launch that copies them
K-major with a padded pitch, transposing an N-major B.  These shapes cover each path: odd K,
N-major B with odd N, f32 N-major, batch broadcast, a single element, K < 8, and K == 0
(epilogue only).  Tolerances: 1e-4 normwise for f32 operands (3xTF32 keeps ~21 mantissa bits
per product), 2e-2 for bf16/f16 (the output is rounded to the half type).
"""
import pytest
import torch

from oracle import fixtures as FX
from oracle.plan_oracle import evaluate, normwise_error

pytestmark = pytest.mark.gpu

TORCH = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}


def matmul_plan(a_shape, b_shape, dtype, trans_b):
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    M = a_shape[-2]
    N = b_shape[-2] if trans_b else b_shape[-1]
    batch = list(torch.broadcast_shapes(tuple(a_shape[:-2]), tuple(b_shape[:-2])))
    nodes = [{"id": 0, "op": "input", "name": "a", "inputs": [], "shape": list(a_shape), "dtype": dtype, "attrs": {}},
             {"id": 1, "op": "input", "name": "b", "inputs": [], "shape": list(b_shape), "dtype": dtype, "attrs": {}},
             {"id": 2, "op": "matmul", "name": "y", "inputs": [0, 1], "shape": batch + [M, N], "dtype": dtype,
              "attrs": {"trans_b": trans_b}}]
    return PProgram.from_dict({
        "format": "tensorjit-plan/1", "name": "mm", "nodes": nodes, "inputs": [0, 1], "outputs": [2],
        "aliases": {}, "meta": {"dtype": dtype},
        "kernels": [{"kind": "matmul", "nodes": [2], "anchor": 2, "inputs": [0, 1], "outputs": [2],
                     "iter_shape": batch + [M, N]}]})


CASES = [
    # (a shape, b shape, trans_b, dtypes)
    ((7, 13), (13, 5), False, ("bf16", "f16", "f32")),          # K % 8 != 0, N-major B with odd N
    ((1, 1), (1, 1), False, ("bf16", "f32")),                   # one element
    ((33, 65), (129, 65), True, ("bf16", "f32")),               # K-major B, odd K
    ((3, 130, 72), (72, 200), False, ("f32",)),                 # batched, f32 N-major B
    ((2, 3, 200, 136), (3, 136, 96), False, ("f32", "bf16")),   # broadcast batch of B
    ((300, 4), (260, 4), True, ("bf16", "f32")),                # K < 8: one padded k-block
    ((513, 1000), (1000, 333), False, ("bf16", "f32")),         # several tiles, ragged everything
]


@pytest.mark.parametrize("a_shape,b_shape,trans_b,dtypes", CASES)
def test_matmul_form_matches_fp64(a_shape, b_shape, trans_b, dtypes):
    from mlir_gpu_kernel_compiler_b200 import B200Program

    g = torch.Generator(device="cuda").manual_seed(3)
    for dt in dtypes:
        a = torch.randn(a_shape, generator=g, device="cuda").to(TORCH[dt])
        b = torch.randn(b_shape, generator=g, device="cuda").to(TORCH[dt])
        prog = B200Program(matmul_plan(a_shape, b_shape, dt, trans_b))
        # pack / split pre-pass, the tcgen05 GEMM, and the finalize launch of a split-K GEMM
        assert [k.family for k in prog.kernel_sources if k.family != "split"][0] == "gemm_tc"
        assert all(k.family in ("split", "gemm_tc", "ewise") for k in prog.kernel_sources)
        y = prog(a, b)[0]
        prog.check()
        bb = b.double().transpose(-1, -2) if trans_b else b.double()
        ref = a.double() @ bb
        err = normwise_error(y, ref)
        assert err <= (1e-4 if dt == "f32" else 2e-2), (dt, err)
        if dt == "f32":      # the oracle restatement agrees too
            assert normwise_error(y, evaluate(prog.pplan, [a.cpu(), b.cpu()])[0]) <= 1e-4


def test_matmul_with_empty_k_is_its_epilogue():
    """K == 0: every dot product is empty, so y = gelu(0 + bias) row by row."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    nodes = [{"id": 0, "op": "input", "name": "a", "inputs": [], "shape": [6, 0], "dtype": "f32", "attrs": {}},
             {"id": 1, "op": "input", "name": "b", "inputs": [], "shape": [0, 5], "dtype": "f32", "attrs": {}},
             {"id": 2, "op": "input", "name": "c", "inputs": [], "shape": [5], "dtype": "f32", "attrs": {}},
             {"id": 3, "op": "matmul", "name": "m", "inputs": [0, 1], "shape": [6, 5], "dtype": "f32",
              "attrs": {"trans_b": False}},
             {"id": 4, "op": "add", "name": "s", "inputs": [3, 2], "shape": [6, 5], "dtype": "f32", "attrs": {}},
             {"id": 5, "op": "gelu", "name": "y", "inputs": [4], "shape": [6, 5], "dtype": "f32", "attrs": {}}]
    plan = PProgram.from_dict({
        "format": "tensorjit-plan/1", "name": "mm0", "nodes": nodes, "inputs": [0, 1, 2], "outputs": [5],
        "aliases": {}, "meta": {},
        "kernels": [{"kind": "matmul", "nodes": [3, 4, 5], "anchor": 3, "inputs": [0, 1, 2], "outputs": [5],
                     "iter_shape": [6, 5]}]})
    prog = B200Program(plan)
    assert [k.family for k in prog.kernel_sources] == ["ewise"]
    c = torch.randn(5, device="cuda")
    y = prog(torch.empty(6, 0, device="cuda"), torch.empty(0, 5, device="cuda"), c)[0]
    prog.check()
    ref = torch.nn.functional.gelu(c).expand(6, 5)
    assert normwise_error(y, ref) <= 1e-4


@pytest.mark.parametrize("case", ["cfg1", "cuda_mlp__f32", "transformer_block__f32", "block_tail__f32"])
def test_forwarded_3xtf32_operands_are_bit_identical(case, monkeypatch):
    """Producers that write a 3xTF32 GEMM's hi / lo operand copies themselves compute the same
    split as the split launch, so the program's outputs are the same bits with forwarding off
    (the default) and on (``TENSORJIT_B200_FORWARD=1``)."""
    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W

    if case == "cfg1":
        plan, ins = FX.load_plan("cfg1"), [t.cuda() for t in W.make_inputs(W.WORKLOADS["cfg1"])]
    else:
        plan, ins = FX.load_plan(case), [t.cuda() for t in FX.case_inputs(case)]
    outs = {}
    for flag in ("0", "1"):
        monkeypatch.setenv("TENSORJIT_B200_FORWARD", flag)
        prog = B200Program(plan, device="cuda")
        assert any(k.info.get("forwarded_outputs") for k in prog.kernel_sources) == (flag == "1")
        outs[flag] = prog(*ins)
        torch.cuda.synchronize()
        prog.check()
    for a, b in zip(outs["0"], outs["1"]):
        assert torch.equal(a, b), case
