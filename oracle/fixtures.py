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
