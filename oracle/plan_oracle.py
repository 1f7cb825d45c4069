"""CPU oracle for the B200 backend — TEST INFRASTRUCTURE ONLY.

Only ``tests/``, ``__graft_entry__.smoke()`` and ``bench.py``'s CPU-baseline leg may
import this module, and only as the checker.  The product path
(``mlir_gpu_kernel_compiler_b200``) never imports it and has no CPU fallback.

What it restates: the arithmetic of tensorjit's ``c`` backend
(``tensorjit/backends/c_backend.py``), which is the oracle named by the build's
north star.  That backend is f32-only (``c_backend.py:77-80``): every load is an
f32 value, every node is evaluated in f32 with the expressions of ``C_EXPR``
(``tensorjit/backends/common.py:65-85``), scalar constants are f32 literals
(``common.py:113-119``), reductions accumulate in f32 and ``mean`` divides the sum
by ``float(N)`` (``c_backend.py:174-176``), ``max`` starts at ``-INFINITY`` and uses
``fmaxf`` (``c_backend.py:169-172``), GELU uses the vectorisable Abramowitz & Stegun
7.1.26 ``tj_erff`` with |x| clamped at 4 (``c_backend.py:44-56``), and matmuls
accumulate ``A[b,i,k]*B[b,k,j]`` (or ``B[b,j,k]`` with ``trans_b``) in f32
(``c_backend.py:186-304``).  Fusion only regroups these per-node expressions into
kernels, so evaluating the optimised graph node by node in f32 gives the
``c`` backend's values up to summation order.

For bf16/f16 plans the oracle evaluates the same graph on the exact f32 upcast
of the inputs, with f32 intermediates — i.e. what the ``c`` backend computes for
the f32 trace of the same function on the upcast inputs.

Pinned against the reference: ``tests/test_oracle.py`` checks this module
against golden outputs produced by running the reference's own ``c`` backend
(``tests/golden/make_fixtures.py``), case by case.
"""
from __future__ import annotations

import numpy as np

F32 = np.float32


def tj_erff(x: np.ndarray) -> np.ndarray:
    """Abramowitz & Stegun 7.1.26 erf, f32, as ``tj_erff`` in ``c_backend.py:44-56``."""
    x = x.astype(F32, copy=False)
    sign = np.where(x < F32(0), F32(-1), F32(1)).astype(F32)
    a = np.abs(x)
    a = np.minimum(a, F32(4.0))
    t = F32(1) / (F32(1) + F32(0.3275911) * a)
    poly = ((((F32(1.061405429) * t - F32(1.453152027)) * t) + F32(1.421413741)) * t - F32(0.284496736)) * t + F32(0.254829592)
    y = F32(1) - poly * t * np.exp(-a * a)
    return (sign * y).astype(F32)


def _f(x):
    return np.asarray(x, dtype=F32)


# C_EXPR, common.py:65-85 (with the tj_erff GELU of the C prelude)
UNARY = {
    "neg": lambda x: -x,
    "exp": lambda x: np.exp(x),
    "log": lambda x: np.log(x),
    "sqrt": lambda x: np.sqrt(x),
    "rsqrt": lambda x: F32(1) / np.sqrt(x),
    "tanh": lambda x: np.tanh(x),
    "relu": lambda x: np.fmax(x, F32(0)),
    "sigmoid": lambda x: F32(1) / (F32(1) + np.exp(-x)),
    "gelu": lambda x: F32(0.5) * x * (F32(1) + tj_erff(x * F32(0.70710678118654752))),
    "silu": lambda x: x / (F32(1) + np.exp(-x)),
    "abs": lambda x: np.abs(x),
}
BINARY = {
    "add": lambda a, b: a + b,
    "sub": lambda a, b: a - b,
    "mul": lambda a, b: a * b,
    "div": lambda a, b: a / b,
    "pow": lambda a, b: np.power(a, b),
    "maximum": lambda a, b: np.fmax(a, b),
    "minimum": lambda a, b: np.fmin(a, b),
}


def _reduce(op: str, x: np.ndarray, keepdim: bool) -> np.ndarray:
    n = x.shape[-1]
    if op == "max":
        r = np.fmax.reduce(x, axis=-1, initial=-np.inf).astype(F32) if n else np.full(x.shape[:-1], -np.inf, F32)
    else:
        r = np.add.reduce(x, axis=-1, dtype=F32)
        if op == "mean":
            r = (r / F32(float(n))).astype(F32)
    return r[..., None] if keepdim else r


def _matmul(a: np.ndarray, b: np.ndarray, trans_b: bool) -> np.ndarray:
    if trans_b:
        b = np.swapaxes(b, -1, -2)
    return np.matmul(a, b, dtype=F32)


def evaluate(plan, inputs, outputs_only: bool = True, strict_shapes: bool = True, round_stored: bool = False):
    """Evaluate ``plan`` (a ``PProgram``) on ``inputs`` (arrays in graph-input order).

    Returns the graph outputs as f32 numpy arrays (or, with ``outputs_only=False``,
    the dict node id -> value of everything computed).  ``strict_shapes=False``
    lets a row-independent plan run on a leading-dimension slice of its row
    inputs (used for the large configs, whose rows are independent).

    ``round_stored=True`` additionally rounds every value a kernel writes to
    memory (each kernel output) to its plan dtype (bf16/f16, round to nearest
    even), while values inside a kernel stay f32 — the storage behaviour of a
    GPU backend that keeps the plan's dtypes in HBM.  With it off (the default)
    the oracle is the reference ``c`` backend: f32 everywhere.
    """
    stored = {o.id: o.dtype for k in plan.kernels for o in k.outputs} if round_stored else {}
    if len(inputs) != len(plan.inputs):
        raise TypeError(f"expected {len(plan.inputs)} inputs, got {len(inputs)}")
    env: dict[int, np.ndarray] = {}
    for node, x in zip(plan.inputs, inputs):
        x = _to_f32(x)
        if strict_shapes and tuple(x.shape) != tuple(node.shape):
            raise ValueError(f"{node.name}: expected {node.shape}, got {tuple(x.shape)}")
        env[node.id] = x

    def val(n):
        if n.id in env:
            return env[n.id]
        if n.op == "const":
            v = np.full(n.shape, F32(n.attrs["value"]), dtype=F32)
            env[n.id] = v
            return v
        raise KeyError(f"{n.name} not computed yet")

    for n in plan.nodes:
        if n.op in ("input", "const") or n.id in env:
            continue
        ins = [val(i) for i in n.inputs]
        if n.op in UNARY:
            with np.errstate(all="ignore"):
                r = UNARY[n.op](ins[0])
        elif n.op in BINARY:
            with np.errstate(all="ignore"):
                r = BINARY[n.op](ins[0], ins[1])
        elif n.op == "where":
            r = np.where(ins[0] != F32(0), ins[1], ins[2])
        elif n.op in ("sum", "max", "mean"):
            r = _reduce(n.op, ins[0], bool(n.attrs.get("keepdim", False)))
        elif n.op == "matmul":
            r = _matmul(ins[0], ins[1], bool(n.attrs.get("trans_b", False)))
        elif n.op == "reshape":
            r = ins[0].reshape(n.shape)
        elif n.op == "transpose":
            r = np.ascontiguousarray(np.transpose(ins[0], n.attrs["perm"]))
        elif n.op == "broadcast_to":
            r = np.broadcast_to(ins[0], n.shape).copy()
        else:
            raise NotImplementedError(n.op)
        r = np.asarray(r, dtype=F32)
        if strict_shapes and tuple(r.shape) != tuple(n.shape):
            r = np.broadcast_to(r, n.shape).astype(F32)
        if stored.get(n.id) in ("bf16", "f16"):
            r = _round_to(r, stored[n.id])
        env[n.id] = r

    outs = [val(plan.resolve(o)).reshape(o.shape) if strict_shapes else val(plan.resolve(o)) for o in plan.outputs]
    return outs if outputs_only else env


def _round_to(x: np.ndarray, dtype: str) -> np.ndarray:
    import torch

    t = torch.from_numpy(np.ascontiguousarray(x))
    return t.to(torch.bfloat16 if dtype == "bf16" else torch.float16).float().numpy()


def _to_f32(x) -> np.ndarray:
    try:
        import torch

        if isinstance(x, torch.Tensor):
            return x.detach().to("cpu", torch.float32).numpy()
    except ImportError:  # pragma: no cover
        pass
    return np.asarray(x, dtype=F32)


def normwise_error(y, ref) -> float:
    """``max|y - ref| / max|ref|`` over the whole output (the parity metric)."""
    y = _to_f32(y).astype(np.float64)
    ref = _to_f32(ref).astype(np.float64)
    if y.shape != ref.shape:
        raise ValueError(f"shape mismatch {y.shape} vs {ref.shape}")
    if ref.size == 0:
        return 0.0
    finite = np.isfinite(ref)
    if not np.array_equal(finite, np.isfinite(y)):
        return float("inf")
    if not finite.any():
        return 0.0
    d = np.abs(y[finite] - ref[finite]).max()
    scale = np.abs(ref[finite]).max()
    return float(d / scale) if scale > 0 else float(d)
