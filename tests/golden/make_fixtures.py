"""Generate the golden fixtures of the B200 backend from the reference itself.

Run in a container where the reference tensorjit sources are importable:

    CC=/usr/bin/gcc CXX=/usr/bin/g++ python tests/golden/make_fixtures.py --ref <path-to-tensorjit-checkout>

For every case it writes

* ``plans/<case>.json``  the fused kernel plan that the reference's tracer,
  cleanup passes, ``fuse`` and ``row_fuse`` produce for the ``cuda`` backend
  (``tensorjit/compiler.py:37-42``; the B200 backend registers with the same
  ``ROW_FUSION_MAX_N = 8192``, so the plan is identical), plus the reference
  memory planner's arena size and offsets (``memory_planner.py:69-119``);
* ``<case>.npz``  seeded inputs and the outputs of the reference's own ``c``
  backend (``c_backend.compile_program`` run through its native runtime) on the
  f32 upcast of those inputs.  For the five benchmark configs only checksums and
  sample rows of the outputs are kept (the tensors themselves are regenerated
  from their seeds by ``mlir_gpu_kernel_compiler_b200.workloads``).

The cases mirror the reference's own tests (``tests/test_backends.py``,
``tests/test_cuda_backend.py``, ``tests/test_runtime_and_planner.py``) plus edge
cases for the B200 kernels (ragged GEMM tiles, long rows, empty tensors).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
import time
from pathlib import Path

import numpy as np
import torch

HERE = Path(__file__).resolve().parent
REPO = HERE.parents[1]
sys.path.insert(0, str(REPO))

from mlir_gpu_kernel_compiler_b200 import workloads as W  # noqa: E402
from mlir_gpu_kernel_compiler_b200.plan import from_tensorjit  # noqa: E402
from oracle import reference_checkout  # noqa: E402


def cases(tj):
    """name -> (fn, [shapes], input recipe, dtypes to emit)."""
    F32, BF16, F16 = "f32", "bf16", "f16"
    C = {}

    def add(name, fn, shapes, recipe="randn", dtypes=(F32, BF16)):
        C[name] = (fn, shapes, recipe, dtypes)

    # tests/test_backends.py:39-47
    for shape in [(17,), (8, 33), (2, 3, 5)]:
        add("ew_chain_" + "x".join(map(str, shape)),
            lambda a, b: tj.exp(tj.relu(a * 2.0 + b)) / (1.0 + tj.sigmoid(a)) - tj.tanh(b),
            [shape, (shape[-1],)])
    # tests/test_backends.py:50-58 (x = rand + 0.5)
    for op in ["gelu", "silu", "log", "sqrt", "rsqrt", "abs", "sigmoid"]:
        add(f"unary_{op}", getattr(tj, op), [(64,)], recipe="rand_plus_half", dtypes=(F32,))
    # tests/test_backends.py:61-66
    add("where_max_pow", lambda a, b: tj.where(a, tj.maximum(a, b), tj.minimum(a, b)) + tj.abs(a) ** 2.0,
        [(40,), (40,)], dtypes=(F32,))
    # tests/test_backends.py:68-74
    for m, k, n in [(1, 1, 1), (7, 13, 5), (64, 64, 64), (33, 128, 65)]:
        add(f"matmul_epi_{m}x{k}x{n}", lambda x, y, z: tj.gelu(tj.matmul(x, y) + z), [(m, k), (k, n), (n,)])
    # tests/test_backends.py:77-82
    add("bmm_broadcast", lambda x, y: tj.relu(tj.matmul(x, y)), [(2, 3, 8, 16), (3, 16, 8)])
    # tests/test_backends.py:85-90
    add("linear_tb", tj.linear, [(10, 32), (48, 32), (48,)])
    # tests/test_backends.py:93-103
    for n in [1, 17, 100, 1000]:
        add(f"reductions_{n}", lambda t: (tj.sum(t), tj.max(t), tj.mean(t, keepdim=True)), [(6, n)])
    # tests/test_backends.py:106-111
    add("reduce_axis1", lambda t: tj.sum(t, axis=1), [(4, 5, 6)])
    # tests/test_backends.py:114-123
    add("softmax_ln_rms", lambda t, w, c: (tj.softmax(t), tj.layer_norm(t, w, c), tj.rms_norm(t, w)),
        [(9, 70), (70,), (70,)])
    # tests/test_backends.py:126-131
    add("transpose_reshape", lambda t: tj.exp(tj.permute(t, 2, 0, 1)).reshape(5, 12) + 1.0, [(3, 4, 5)])

    # tests/test_backends.py:134-163
    def block(x, ln_g, w1, b1, w2, b2, wq, wk):
        h = tj.layer_norm(x, ln_g)
        q, k = tj.linear(h, wq), tj.linear(h, wk)
        scores = tj.softmax(tj.matmul(q, k.T) * (1.0 / 8.0))
        mlp = tj.linear(tj.gelu(tj.linear(h, w1, b1)), w2, b2)
        return x + mlp, scores

    add("transformer_block", block, [(12, 32), (32,), (64, 32), (64,), (32, 64), (32,), (32, 32), (32, 32)])
    # tests/test_runtime_and_planner.py:80-85
    add("reshape_const_outputs", lambda t: (tj.exp(t).reshape(5, 12), tj.sum(t * 0.0 + 2.0)), [(3, 4, 5)],
        dtypes=(F32,))

    # tests/test_cuda_backend.py:20-28 (CASES)
    add("cuda_mlp", lambda x, g, w1, b1, w2, b2: x + tj.linear(tj.gelu(tj.linear(tj.layer_norm(x, g), w1, b1)), w2, b2),
        [(64, 128), (128,), (256, 128), (256,), (128, 256), (128,)])
    add("cuda_rows", lambda x, w: (tj.softmax(x), tj.rms_norm(x, w), tj.sum(x * x), tj.max(x, keepdim=True)),
        [(8, 100), (100,)])
    add("cuda_bmm", lambda a, b: tj.relu(tj.matmul(a, b)).sum(axis=2), [(2, 3, 8, 16), (3, 16, 8)])
    add("cuda_pointwise", lambda a, b: tj.where(a, tj.maximum(a, b), tj.minimum(a, b)) + tj.exp(a) ** 2.0,
        [(4, 5, 6), (6,)])
    add("cuda_movement", lambda t: tj.exp(tj.permute(t, 2, 0, 1)).reshape(5, 12) + 1.0, [(3, 4, 5)])
    add("cuda_wmma", lambda x, w, b: tj.gelu(tj.linear(x, w, b)), [(64, 128), (256, 128), (256,)],
        dtypes=(F32, BF16, F16))

    # B200 edge cases: tensor-core tiles (aligned and ragged), long/short rows, empty input
    add("gemm_tc_aligned", lambda x, w, b, r: tj.gelu(tj.linear(x, w, b)) + r,
        [(256, 512), (512, 512), (512,), (256, 512)], dtypes=(BF16, F16, F32))
    add("gemm_tc_ragged", lambda x, w, b: tj.gelu(tj.linear(x, w, b)), [(200, 136), (300, 136), (300,)],
        dtypes=(BF16, F32))
    add("gemm_tc_nn_batched", lambda s, v: tj.matmul(s, v), [(2, 3, 256, 192), (2, 3, 192, 64)], dtypes=(BF16, F32))
    add("gemm_tc_batched_tb", lambda q, k: tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125,
        [(2, 2, 256, 64), (2, 2, 384, 64)], dtypes=(BF16, F32))
    add("gemm_tc_multiwave", lambda x, w: tj.linear(x, w), [(2048, 1024), (2304, 1024)], dtypes=(BF16,))
    add("rows_long", lambda x, r, g: (tj.rms_norm(x + r, g), tj.softmax(x)), [(16, 8192), (16, 8192), (8192,)])
    add("rows_too_long", lambda x: tj.softmax(x), [(3, 8200)])
    add("rows_odd", lambda x, g, b: tj.layer_norm(x, g, b), [(37, 333), (333,), (333,)])
    add("empty_rows", lambda x, b: tj.gelu(x + b), [(0, 16), (16,)], dtypes=(F32,))
    add("transpose_2d", lambda x: tj.permute(x, 1, 0) * 2.0, [(67, 129)])
    add("linear_nobias_ragged", lambda x, w: tj.linear(x, w), [(200, 136), (300, 136)], dtypes=(F32,))
    # three bare GEMMs reading the same A (a q/k/v-style projection): one GEMM over the concatenated N
    add("shared_a_projections", lambda x, w1, w2, w3: (tj.linear(x, w1), tj.linear(x, w2), tj.linear(x, w3)),
        [(300, 128), (256, 128), (512, 128), (256, 128)], dtypes=(BF16,))
    # few output tiles and a long K: the 3xTF32 GEMM is split over K (ragged N: scalar partial stores)
    add("linear_splitk_ragged", lambda x, w, b: tj.gelu(tj.linear(x, w, b)), [(100, 2048), (130, 2048), (130,)],
        dtypes=(F32,))
    # attention core (QK^T * scale -> softmax -> PV), the pattern of the transformer config
    add("attention_core", lambda q, k, v: tj.matmul(tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125), v),
        [(2, 4, 256, 64), (2, 4, 256, 64), (2, 4, 256, 64)], dtypes=(BF16,))
    add("attention_probs_escape",
        lambda q, k, v: (lambda p_: (tj.matmul(p_, v), p_))(tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125)),
        [(1, 2, 128, 64), (1, 2, 384, 64), (1, 2, 384, 64)], dtypes=(BF16,))
    # ragged query/key lengths (partial 128-row tiles and a masked last key block), scale as a divide
    add("attention_ragged", lambda q, k, v: tj.matmul(tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) / 8.0), v),
        [(3, 200, 64), (3, 300, 64), (3, 300, 64)], dtypes=(BF16, F16))
    # no scale, fewer queries and keys than one tile
    add("attention_short", lambda q, k, v: tj.matmul(tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2))), v),
        [(2, 2, 40, 64), (2, 2, 72, 64), (2, 2, 72, 64)], dtypes=(F16,))

    # head split / merge around the attention (the transformer config's layout, small)
    def mha(x, wq, wk, wv, wo):
        def heads(t):
            return tj.permute(tj.reshape(t, (2, 256, 4, 64)), 0, 2, 1, 3)

        # projections scaled by 1/sqrt(fan-in) so that q, k, v ~ N(0, 1) and the scores stay O(1)
        q, k, v = (heads(tj.linear(x, w) * 0.08838834764831845) for w in (wq, wk, wv))
        s = tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125)
        return tj.linear(tj.reshape(tj.permute(tj.matmul(s, v), 0, 2, 1, 3), (512, 256)), wo) * 0.0625

    add("attention_heads", mha, [(512, 128), (256, 128), (256, 128), (256, 128), (128, 256)], dtypes=(BF16,))

    # a transpose kernel feeding a plain GEMM's A operand (folded into the GEMM's operand
    # addressing): the head merge before an output projection, and a batch-dim transpose
    # before a batched matmul with an N-major B
    add("merge_heads_linear", lambda x, w, b: tj.linear(tj.reshape(tj.permute(x, 0, 2, 1, 3), (512, 256)), w, b),
        [(2, 4, 256, 64), (128, 256), (128,)], dtypes=(BF16, F16, F32))
    add("transpose_bmm", lambda x, w: tj.gelu(tj.matmul(tj.permute(x, 1, 0, 2), w)),
        [(256, 4, 128), (4, 128, 192)], dtypes=(BF16,))

    # unfused attention scores (no softmax follows): both GEMM operands come from head-split
    # transposes of projection outputs, A and the K-major B (trans_b) each with two batch dims
    def heads_scores(x, wq, wk):
        def heads(t):
            return tj.permute(tj.reshape(t, (2, 256, 4, 64)), 0, 2, 1, 3)

        q, k = heads(tj.linear(x, wq) * 0.0625), heads(tj.linear(x, wk) * 0.0625)
        return tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125

    add("heads_scores", heads_scores, [(512, 256), (256, 256), (256, 256)], dtypes=(BF16,))

    # an attention whose probabilities are also returned (so it is not fused): the q / k / v head
    # splits, the N-major v of P·V and the head merge before the output projection are all copies
    # that the GEMMs reading them fold away
    def heads_attention_probs(x, wq, wk, wv, wo):
        def heads(t):
            return tj.permute(tj.reshape(t, (2, 256, 4, 64)), 0, 2, 1, 3)

        q, k, v = (heads(tj.linear(x, w) * 0.0625) for w in (wq, wk, wv))
        p_ = tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125)
        o = tj.linear(tj.reshape(tj.permute(tj.matmul(p_, v), 0, 2, 1, 3), (512, 256)), wo) * 0.0625
        return o, p_

    add("heads_attention_probs", heads_attention_probs,
        [(512, 256), (256, 256), (256, 256), (256, 256), (256, 256)], dtypes=(BF16,))

    # a pre-norm block's tail: the residual add after the MLP is planned as its own elementwise
    # kernel (x1 also feeds the LayerNorm), which the B200 backend folds into the GEMM epilogue
    def block_tail(x, r, wo, g, w1, b1, w2, b2):
        x1 = r + tj.linear(x, wo) * 0.0883883461
        return x1 + tj.linear(tj.gelu(tj.linear(tj.layer_norm(x1, g), w1, b1) * 0.0883883461), w2, b2) * 0.0441941738

    add("block_tail", block_tail, [(300, 128), (300, 128), (128, 128), (128,), (512, 128), (512,), (128, 512), (128,)],
        dtypes=(F32, BF16))
    return C


def config_fns(tj):
    def mlp_ln(x, g, w1, b1, w2, b2):
        return x + tj.linear(tj.gelu(tj.linear(tj.layer_norm(x, g), w1, b1)), w2, b2)

    def rms_softmax(x, r, g, s):
        return tj.rms_norm(x + r, g), tj.softmax(s)

    def gemm_epi(x, w, b, res):
        return tj.gelu(tj.linear(x, w, b)) + res

    def block(x, g1, wq, wk, wv, wo, bo, g2, w1, b1, w2, b2):
        h = tj.layer_norm(x, g1)

        def heads(t):
            return tj.permute(tj.reshape(t, (8, 2048, 16, 64)), 0, 2, 1, 3)

        q, k, v = heads(tj.linear(h, wq)), heads(tj.linear(h, wk)), heads(tj.linear(h, wv))
        s = tj.softmax(tj.matmul(q, tj.transpose(k, -1, -2)) * 0.125)
        o = tj.reshape(tj.permute(tj.matmul(s, v), 0, 2, 1, 3), (16384, 1024))
        x1 = x + tj.linear(o, wo, bo)
        return x1 + tj.linear(tj.gelu(tj.linear(tj.layer_norm(x1, g2), w1, b1)), w2, b2)

    def mlp_rms(x, g, w1, b1, w2, b2):
        return x + tj.linear(tj.gelu(tj.linear(tj.rms_norm(x, g), w1, b1)), w2, b2)

    return {"cfg1": mlp_ln, "cfg2": rms_softmax, "cfg3": gemm_epi, "cfg4": block, "cfg5": mlp_rms}


def _inputs(shapes, recipe, seed=0):
    g = torch.Generator().manual_seed(seed)
    out = []
    for s in shapes:
        if recipe == "rand_plus_half":
            out.append(torch.rand(s, generator=g) + 0.5)
        else:
            out.append(torch.randn(s, generator=g))
    return out


def _plan_json(tj_mod, program, name, meta):
    from tensorjit.passes.memory_planner import plan_memory

    p = from_tensorjit(program)
    mp = plan_memory(program)
    ids = {}
    # map reference Node ids -> plan node ids through names (unique per graph)
    by_name = {n.name: n.id for n in p.nodes}
    for b in mp.buffers.values():
        ids[str(by_name[b.node.name])] = b.offset
    p.meta = dict(meta, reference_arena_bytes=mp.arena_bytes, reference_offsets=ids)
    p.name = name
    return p


def _run_c(tj_mod, fn, shapes, inputs_f32):
    """The reference ``c`` backend (f32) on f32 inputs, through its native runtime."""
    import tensorjit.compiler as C
    from tensorjit.ir import TensorType

    g = tj_mod.trace(fn, [TensorType(tuple(s)) for s in shapes])
    cp = C.compile_graph(g, "c", device="cpu", tune=False)
    outs = cp(*inputs_f32)
    return [o.detach().clone().float().numpy() for o in outs]


def _sample_rows(a: np.ndarray, k: int = 2) -> tuple[np.ndarray, np.ndarray]:
    m = a.reshape(-1, a.shape[-1]) if a.ndim >= 2 else a.reshape(1, -1)
    R = m.shape[0]
    idx = sorted(set([*range(min(k, R)), *range(max(R // 2 - k // 2, 0), min(R // 2 + (k + 1) // 2, R)),
                      *range(max(R - k, 0), R)]))
    return np.asarray(idx, dtype=np.int64), m[idx].astype(np.float32)


SMALL = 1 << 16   # arrays up to this many elements are stored whole


def _summary(i: int, o: np.ndarray) -> dict:
    """Checksums and sample rows of a large output (inputs are regenerated from their seed)."""
    ridx, rows = _sample_rows(o)
    return {
        f"out{i}_rows_idx": ridx,
        f"out{i}_rows": rows,
        f"out{i}_sum": np.float64(o.astype(np.float64).sum()),
        f"out{i}_abssum": np.float64(np.abs(o.astype(np.float64)).sum()),
        f"out{i}_absmax": np.float64(np.abs(o).max()) if o.size else np.float64(0),
        f"out{i}_shape": np.asarray(o.shape, dtype=np.int64),
    }


DENSE_CONFIGS = ("cfg2", "cfg4")


def row_checksums(o: np.ndarray) -> dict:
    """Per-row checksums of an output viewed as [rows, last dim], in f64: the sum, the sum of
    |y|, the sum of y^2, and the position-weighted sum (j + 1) / n * y_j (which also catches
    a permutation within the row)."""
    m = o.reshape(-1, o.shape[-1]).astype(np.float64)
    w = (np.arange(m.shape[1], dtype=np.float64) + 1.0) / m.shape[1]
    return {"sum": m.sum(1), "abssum": np.abs(m).sum(1), "sumsq": (m * m).sum(1), "wsum": m @ w}


def _dense(cname: str, outs: list[np.ndarray]) -> dict:
    """Dense golden data of a full-size config: per-row checksums of every output row, plus
    whole rows -- cfg4: all of batch element 0 (rows 0..2047 of y, stored as f16); cfg2: 192 rows
    of the RMSNorm output spread over its 16384 (f16) and 64 rows of the softmax (f32: its
    values lie below f16's normal range)."""
    arrays = {}
    for i, o in enumerate(outs):
        for k, v in row_checksums(o).items():
            arrays[f"out{i}_row_{k}"] = v
    if cname == "cfg4":
        arrays["out0_dense_idx"] = np.arange(2048, dtype=np.int64)
        arrays["out0_dense"] = outs[0][:2048].astype(np.float16)
    elif cname == "cfg2":
        i0 = np.unique(np.linspace(0, outs[0].shape[0] - 1, 192).round().astype(np.int64))
        i1 = np.unique(np.linspace(0, outs[1].shape[0] - 1, 64).round().astype(np.int64))
        arrays.update(out0_dense_idx=i0, out0_dense=outs[0][i0].astype(np.float16),
                      out1_dense_idx=i1, out1_dense=outs[1][i1].astype(np.float32))
    return arrays


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=str(reference_checkout()))
    ap.add_argument("--only", nargs="*", default=None)
    ap.add_argument("--skip-configs", action="store_true")
    ap.add_argument("--configs-only", action="store_true")
    ap.add_argument("--dense-only", action="store_true",
                    help="only (re)write <cfg>.dense.npz of the configs in DENSE_CONFIGS (or --only)")
    a = ap.parse_args()
    sys.path.insert(0, a.ref)
    os.environ.setdefault("TENSORJIT_NO_AUTOTUNE", "1")
    os.environ.setdefault("TENSORJIT_CACHE_DIR", tempfile.mkdtemp(prefix="tjref_"))
    import tensorjit as tj
    import tensorjit.compiler as C
    from tensorjit.ir import DType, TensorType

    dt = {"f32": DType.f32, "bf16": DType.bf16, "f16": DType.f16}
    (HERE / "plans").mkdir(exist_ok=True)
    index = {}
    idx_path = HERE / "index.json"
    if idx_path.exists() and (a.only or a.skip_configs or a.configs_only or a.dense_only):
        index = json.loads(idx_path.read_text())     # partial run: keep the other entries

    if a.dense_only:
        fns = config_fns(tj)
        for cname in (a.only or DENSE_CONFIGS):
            w = W.WORKLOADS[cname]
            ins = [t.float() for t in W.make_inputs(w)]
            outs = _run_c(tj, fns[cname], [tuple(t.shape) for t in ins], ins)
            np.savez_compressed(HERE / f"{w.plan}.dense.npz", **_dense(cname, outs))
            index[w.plan]["dense"] = f"{w.plan}.dense.npz"
            print(f"  dense {w.plan}: {[o.shape for o in outs]}")
        idx_path.write_text(json.dumps(index, indent=1, sort_keys=True))
        return

    if not a.configs_only:
        for name, (fn, shapes, recipe, dtypes) in cases(tj).items():
            if a.only and name not in a.only:
                continue
            ins = _inputs(shapes, recipe)
            for d in dtypes:
                ins_d = [t.to({"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16}[d]) for t in ins]
                ins_f32 = [t.float() for t in ins_d]          # exact upcast
                g = tj.trace(fn, [TensorType(tuple(s), dt[d]) for s in shapes])
                prog = C.lower(g, "cuda")
                case = f"{name}__{d}"
                p = _plan_json(tj, prog, case, {"dtype": d, "shapes": [list(s) for s in shapes], "recipe": recipe})
                (HERE / "plans" / f"{case}.json").write_text(p.to_json(indent=None))
                outs = _run_c(tj, fn, shapes, ins_f32)
                arrays = {}
                if sum(t.numel() for t in ins_f32) <= SMALL:
                    arrays.update({f"in{i}": t.numpy() for i, t in enumerate(ins_f32)})
                for i, o in enumerate(outs):
                    if o.size <= SMALL:
                        arrays[f"out{i}"] = o
                    else:
                        arrays.update(_summary(i, o))
                np.savez_compressed(HERE / f"{case}.npz", **arrays)
                index[case] = {"plan": f"plans/{case}.json", "data": f"{case}.npz", "dtype": d,
                               "kernels": [k.kind for k in p.kernels], "n_out": len(outs)}
                print(f"{case:36s} {len(p.kernels)} kernels {[k.kind for k in p.kernels]}")

    if not a.skip_configs:
        fns = config_fns(tj)
        for cname, w in W.WORKLOADS.items():
            if a.only and cname not in a.only:
                continue
            fn = fns[cname]
            dname = {torch.float32: "f32", torch.bfloat16: "bf16"}[w.dtype]
            ms = [w.args[0].shape[0]]
            if cname == "cfg5":
                ms = [131072, 65536, 32768, 16384, 1024]
            for m in ms:
                shapes = [tuple(ar.shape) for ar in w.args]
                for i in w.row_args:
                    shapes[i] = (m,) + tuple(shapes[i][1:])
                pname = w.plan if cname != "cfg5" else f"cfg5_m{m}"
                g = tj.trace(fn, [TensorType(s, dt[dname]) for s in shapes])
                prog = C.lower(g, "cuda")
                p = _plan_json(tj, prog, pname, {"dtype": dname, "shapes": [list(s) for s in shapes],
                                                 "workload": cname})
                (HERE / "plans" / f"{pname}.json").write_text(p.to_json(indent=None))
                print(f"{pname:36s} {len(p.kernels)} kernels {[k.kind for k in p.kernels]} "
                      f"arena {p.meta['reference_arena_bytes']}")
                index[pname] = {"plan": f"plans/{pname}.json", "dtype": dname,
                                "kernels": [k.kind for k in p.kernels], "workload": cname}
            # golden outputs of the reference c backend on the seeded inputs
            if cname == "cfg5":
                m = 1024
                ins = [t.float() for t in W.make_inputs(w, rows=(0, m))]
                shapes = [tuple(t.shape) for t in ins]
                gname = "cfg5_m1024"
            else:
                ins = [t.float() for t in W.make_inputs(w)]
                shapes = [tuple(t.shape) for t in ins]
                gname = w.plan
            t0 = time.time()
            outs = _run_c(tj, fn, shapes, ins)
            el = time.time() - t0
            arrays = {}
            for i, o in enumerate(outs):
                arrays.update(_summary(i, o))
            np.savez_compressed(HERE / f"{gname}.golden.npz", **arrays)
            index[gname]["golden"] = f"{gname}.golden.npz"
            if cname in DENSE_CONFIGS:
                np.savez_compressed(HERE / f"{gname}.dense.npz", **_dense(cname, outs))
                index[gname]["dense"] = f"{gname}.dense.npz"
            index[gname]["c_backend_seconds_here"] = round(el, 3)
            print(f"  golden {gname}: c backend {el:.2f}s")

    idx_path.write_text(json.dumps(index, indent=1, sort_keys=True))


if __name__ == "__main__":
    main()
