"""Golden-fixture access for the parity checks — TEST INFRASTRUCTURE ONLY.

Fixtures live in ``tests/golden`` and are written by ``tests/golden/make_fixtures.py``
from the reference itself: ``plans/<case>.json`` is the fused kernel plan, and
``<case>.npz`` holds the seeded inputs (small cases) and the outputs of the
reference ``c`` backend, either whole or, for large outputs, as checksums plus
sample rows.  Inputs that are not stored are regenerated here exactly as the
generator drew them.
"""
from __future__ import annotations

import json
from functools import lru_cache
from pathlib import Path

import numpy as np
import torch

REPO = Path(__file__).resolve().parents[1]
GOLDEN = REPO / "tests" / "golden"
TORCH_DTYPE = {"f32": torch.float32, "bf16": torch.bfloat16, "f16": torch.float16, "i32": torch.int32}
TOL = {"f32": 1e-4, "bf16": 2e-2, "f16": 2e-2}


@lru_cache(maxsize=None)
def index() -> dict:
    return json.loads((GOLDEN / "index.json").read_text())


def cases(kind: str = "case") -> list[str]:
    idx = index()
    if kind == "case":
        return sorted(k for k, v in idx.items() if "data" in v)
    return sorted(k for k, v in idx.items() if "workload" in v)


def load_plan(name: str):
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    return PProgram.load(GOLDEN / index()[name]["plan"])


def case_inputs(name: str) -> list[torch.Tensor]:
    """Inputs of a test case in the plan's dtype (CPU tensors)."""
    plan = load_plan(name)
    meta = plan.meta
    data = np.load(GOLDEN / index()[name]["data"])
    dt = TORCH_DTYPE[meta["dtype"]]
    if "in0" in data.files:
        return [torch.from_numpy(data[f"in{i}"]).to(dt) for i in range(len(meta["shapes"]))]
    g = torch.Generator().manual_seed(0)
    out = []
    for s in meta["shapes"]:
        if meta.get("recipe") == "rand_plus_half":
            t = torch.rand(tuple(s), generator=g) + 0.5
        else:
            t = torch.randn(tuple(s), generator=g)
        out.append(t.to(dt))
    return out


def case_expected(name: str) -> list[dict]:
    """Per output: {"full": array} or {"rows_idx", "rows", "sum", "abssum", "absmax", "shape"}."""
    entry = index()[name]
    fname = entry.get("data") or entry.get("golden")
    data = np.load(GOLDEN / fname)
    outs = []
    i = 0
    while True:
        if f"out{i}" in data.files:
            outs.append({"full": data[f"out{i}"]})
        elif f"out{i}_rows" in data.files:
            outs.append({k[len(f"out{i}_"):]: data[k] for k in data.files if k.startswith(f"out{i}_")})
        else:
            break
        i += 1
    return outs


def check_against_golden(y, exp: dict, tol: float) -> float:
    """Normwise error of output ``y`` against one golden entry; raises if above ``tol``."""
    from oracle.plan_oracle import normwise_error

    y = y.detach().to("cpu", torch.float32).numpy() if isinstance(y, torch.Tensor) else np.asarray(y, np.float32)
    if "full" in exp:
        err = normwise_error(y, exp["full"].reshape(y.shape))
    else:
        assert tuple(y.shape) == tuple(int(s) for s in exp["shape"]), (y.shape, exp["shape"])
        m = y.reshape(-1, y.shape[-1]) if y.ndim >= 2 else y.reshape(1, -1)
        rows = m[exp["rows_idx"]]
        scale = float(exp["absmax"]) or 1.0
        err = float(np.abs(rows.astype(np.float64) - exp["rows"]).max() / scale) if rows.size else 0.0
        # checksum of the whole output: mean absolute value must agree to the same tolerance
        n = max(y.size, 1)
        abs_mean = float(np.abs(y.astype(np.float64)).sum()) / n
        ref_abs_mean = float(exp["abssum"]) / n
        err = max(err, abs(abs_mean - ref_abs_mean) / scale)
    if not err <= tol:
        raise AssertionError(f"normwise error {err:.3e} > tol {tol:.1e}")
    return err


def case_dense(name: str) -> dict | None:
    """Dense golden data of a full-size config (per-row checksums of every output row and whole
    rows; written by ``tests/golden/make_fixtures.py``), or None if the config has none."""
    entry = index()[name]
    if "dense" not in entry:
        return None
    data = np.load(GOLDEN / entry["dense"])
    return {k: data[k] for k in data.files}


def check_rows_dense(y, dense: dict, i: int, tol: float) -> dict:
    """Output ``i`` against the dense golden data, row by row.

    * whole rows (``out{i}_dense_idx`` / ``out{i}_dense``): normwise error per row ≤ tol;
    * every row: with S = Σ|ref| over the row, |Σy − Σref| ≤ tol·S, |Σ|y| − Σ|ref|| ≤ tol·S,
      |Σ(j+1)/n·y − the same of ref| ≤ tol·S (a permuted row fails) and
      |Σy² − Σref²| ≤ 2·tol·Σref² (a row with the right sum but the wrong spread fails).
    These are the normwise tolerance applied to row-level L1 / L2 measures.  Returns the worst
    value of each measure."""
    y = y.detach().to("cpu", torch.float32).numpy() if isinstance(y, torch.Tensor) else np.asarray(y, np.float32)
    m = y.reshape(-1, y.shape[-1]).astype(np.float64)
    worst = {}
    if f"out{i}_dense" in dense:
        idx = dense[f"out{i}_dense_idx"]
        ref = dense[f"out{i}_dense"].astype(np.float64)
        got = m[idx]
        scale = np.maximum(np.abs(ref).max(1), 1e-30)
        e = np.abs(got - ref).max(1) / scale
        worst["rows"] = float(e.max())
        if not worst["rows"] <= tol:
            raise AssertionError(f"out{i} row {int(idx[e.argmax()])}: normwise error {e.max():.3e} > {tol:.1e}")
    w = (np.arange(m.shape[1], dtype=np.float64) + 1.0) / m.shape[1]
    S = np.maximum(dense[f"out{i}_row_abssum"], 1e-30)
    checks = {"sum": (np.abs(m.sum(1) - dense[f"out{i}_row_sum"]) / S, tol),
              "abssum": (np.abs(np.abs(m).sum(1) - dense[f"out{i}_row_abssum"]) / S, tol),
              "wsum": (np.abs(m @ w - dense[f"out{i}_row_wsum"]) / S, tol),
              "sumsq": (np.abs((m * m).sum(1) - dense[f"out{i}_row_sumsq"])
                        / np.maximum(dense[f"out{i}_row_sumsq"], 1e-30), 2 * tol)}
    if m.shape[0] != S.shape[0]:
        raise AssertionError(f"out{i}: {m.shape[0]} rows, golden has {S.shape[0]}")
    for k, (e, t) in checks.items():
        worst[k] = float(e.max())
        if not worst[k] <= t:
            raise AssertionError(f"out{i} row {int(e.argmax())}: row {k} differs by {e.max():.3e} (> {t:.1e})")
    return worst


# Half-precision outputs whose distance from the f32 reference exceeds the 2e-2 tolerance
# because of the plan's own bf16 storage, not the GPU: (case, output index) -> (error of the
# bf16-storage oracle against the f32 reference, bound the GPU output must meet).  The GPU
# output must still match the bf16-storage oracle within 2e-2.
#   transformer_block__bf16 output 1 (the attention probabilities): the weights are N(0, 1),
#   so the scores reach the hundreds and their bf16 rounding (stored between the QK^T matmul
#   and the softmax, as the plan says) moves the probabilities by 3.04e-2 on its own.
BF16_STORAGE_EXCEPTIONS = {("transformer_block__bf16", 1): (3.04e-2, 3.5e-2)}


def allowed_error(case: str, out_index: int, tol: float) -> float:
    """The bound an output of ``case`` must meet against the f32 reference."""
    ent = BF16_STORAGE_EXCEPTIONS.get((case, out_index))
    return ent[1] if ent else tol


def merge_heads_plan(batch: int, heads: int, seq: int, dh: int, n: int, dtype: str = "bf16"):
    """The reference's plan of linear(reshape(permute(x, 0, 2, 1, 3), (batch*seq, heads*dh)), w, b)
    (fixture merge_heads_linear) with other sizes: a transpose copy kernel, then the GEMM."""
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    d = load_plan("merge_heads_linear__bf16").to_dict()
    shapes = {0: [batch, heads, seq, dh], 1: [n, heads * dh], 2: [n], 3: [batch, seq, heads, dh],
              4: [batch * seq, heads * dh], 5: [batch * seq, n], 6: [batch * seq, n]}
    for nd in d["nodes"]:
        nd["shape"] = shapes[nd["id"]]
        nd["dtype"] = dtype
        if nd["op"] == "reshape":
            nd["attrs"]["shape"] = shapes[4]
    d["kernels"][0]["iter_shape"] = shapes[3]
    d["kernels"][1]["iter_shape"] = shapes[5]
    d["aliases"] = {"4": [3, shapes[4]]}
    d["meta"] = dict(d.get("meta", {}), dtype=dtype)
    return PProgram.from_dict(d)
