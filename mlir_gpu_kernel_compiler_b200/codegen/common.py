"""Shared pieces of the sm_100a code generator: op expressions, C types,
kernel-source records and index arithmetic.

The generator emits one small CUDA translation unit per plan kernel: a
parameter-block struct, the kernel entry point, and the fused pointwise DAG
written out as straight-line f32 code.  The heavy lifting (vector memory
access, reductions, the tcgen05 GEMM pipeline) lives in the hand-written
headers under ``csrc/kernels``; the generated part only binds sizes, strides
and the DAG as compile-time constants.
"""
from __future__ import annotations

import contextlib
import contextvars
import math
from dataclasses import dataclass, field
from typing import Optional

from ..plan import PKernel, PNode

# Checked build (TENSORJIT_B200_CHECKED=1): generators declare global operands as bounded views
# (``tj_view`` in tj_common.cuh, compiled with -DTJ_CHECKED) and give every kernel a status
# argument, so an out-of-range element index is reported instead of touching memory.
_CHECKED = contextvars.ContextVar("tj_checked", default=False)
BOUNDS_SITE = 15          # status "where" = plan kernel index * 16 + BOUNDS_SITE


def checked() -> bool:
    return _CHECKED.get()


@contextlib.contextmanager
def checked_build(on: bool = True):
    token = _CHECKED.set(bool(on))
    try:
        yield
    finally:
        _CHECKED.reset(token)


# Programs whose outputs may live in another GPU's memory (rows stored over NVLink into a peer's
# buffer) keep every epilogue on plain 16-byte stores instead of TMA stores.
_TMA_STORE = contextvars.ContextVar("tj_tma_store", default=True)


def tma_store_allowed() -> bool:
    return _TMA_STORE.get()


@contextlib.contextmanager
def store_mode(tma_store: bool = True):
    token = _TMA_STORE.set(bool(tma_store))
    try:
        yield
    finally:
        _TMA_STORE.reset(token)


# 3xTF32 operand forwarding: an f32 intermediate whose only reader is a 3xTF32 GEMM is written by
# its producer directly as that GEMM's TF32 hi / lo copies in the workspace, so the GEMM's split
# launch keeps only the operands that are program inputs.  ``split_out``: node id -> elements from
# the hi copy to the lo copy; ``split_skip``: plan kernel index -> operands ("a" / "b") whose
# split its producer already wrote.
_SPLIT_OUT = contextvars.ContextVar("tj_split_out", default=None)
_SPLIT_SKIP = contextvars.ContextVar("tj_split_skip", default=None)


def split_out() -> dict:
    return _SPLIT_OUT.get() or {}


def split_skip(kernel_id: int) -> set:
    return (_SPLIT_SKIP.get() or {}).get(kernel_id, set())


@contextlib.contextmanager
def split_forwarding(out: dict, skip: dict):
    t1, t2 = _SPLIT_OUT.set(dict(out)), _SPLIT_SKIP.set(dict(skip))
    try:
        yield
    finally:
        _SPLIT_SKIP.reset(t2)
        _SPLIT_OUT.reset(t1)


def split_store_lines(ptr: str, off: str, src: str, n: int, delta: int) -> list[str]:
    """Store the ``n`` f32 values ``src[0..n)`` at ``ptr + off`` as their TF32 split: hi (13 low
    mantissa bits cleared, as the split launch computes it) there, lo = value - hi ``delta``
    elements further on; 16-byte stores for n a multiple of 4, else scalar."""
    L = [f"{{ float sh[{n}], sl[{n}];",
         "  #pragma unroll",
         f"  for (int q = 0; q < {n}; ++q) {{ sh[q] = tj_tf32_hi({src}[q]); sl[q] = {src}[q] - sh[q]; }}"]
    if n % 4 == 0:
        for c in range(0, n, 4):
            L.append(f"  tj_store_vec({ptr} + ({off}) + {c}, sh + {c}); "
                     f"tj_store_vec({ptr} + ({off}) + {delta + c}L, sl + {c});")
    else:
        for c in range(n):
            L.append(f"  {ptr}[({off}) + {c}] = sh[{c}]; {ptr}[({off}) + {delta + c}L] = sl[{c}];")
    L.append("}")
    return L


def ptr_decl(name: str, ctype: str, idx: int, numel: int, const: bool, kernel_id: int = 0,
             status: str = "tj_status") -> str:
    """Declaration of kernel argument ``idx`` as ``name``: a restrict pointer, or in a checked
    build a ``tj_view`` over its ``numel`` elements that reports (TJ_STATUS_BOUNDS,
    kernel_id * 16 + 15, argument idx) through ``status``."""
    t = f"const {ctype}" if const else ctype
    if not checked():
        return f"{t}* __restrict__ {name} = ({t}*)prm.p[{idx}];"
    return (f"const tj_view<{t}> {name}{{({t}*)prm.p[{idx}], {numel}L, {status}, "
            f"{kernel_id * 16 + BOUNDS_SITE}, {idx}}};")


def status_decl(idx: int) -> str:
    """``tj_status``: the program's status words (argument ``idx``), declared in checked builds."""
    return f"int* const tj_status = (int*)prm.p[{idx}];" if checked() else ""

CTYPE = {"f32": "float", "f16": "__half", "bf16": "__nv_bfloat16", "i32": "int"}
ITEM = {"f32": 4, "f16": 2, "bf16": 2, "i32": 4}
NUM_SMS = 148

# CUDA expression per op (tensorjit/backends/common.py:65-88).  The helper
# functions are defined in csrc/kernels/tj_common.cuh with the same formulas.
EXPR = {
    "neg": "(-{0})",
    "exp": "expf({0})",
    "log": "logf({0})",
    "sqrt": "sqrtf({0})",
    "rsqrt": "tj_rsqrt({0})",
    "tanh": "tanhf({0})",
    "relu": "tj_relu({0})",
    "sigmoid": "tj_sigmoid({0})",
    "gelu": "tj_gelu({0})",
    "silu": "tj_silu({0})",
    "abs": "fabsf({0})",
    "add": "({0} + {1})",
    "sub": "({0} - {1})",
    "mul": "({0} * {1})",
    "div": "({0} / {1})",
    "pow": "powf({0}, {1})",
    "maximum": "fmaxf({0}, {1})",
    "minimum": "fminf({0}, {1})",
    "where": "tj_where({0}, {1}, {2})",
}


# Half-precision programs round every stored value to bf16/f16 (relative step
# 2^-8 / 2^-11), so their kernels use approximations at or below that rounding:
# __expf (ex2.approx based, rel. error ~1e-6 for the arguments seen here), __fdividef
# (rcp.approx * a) and tj_gelu_fast (Phi as a logistic of a fitted odd polynomial:
# relative error <= 3.8e-4 for x >= 0, <= 1.4e-3 for x < 0 where |GELU| <= 0.17,
# absolute <= 1.7e-4; normwise 2.3e-5 on N(0, 1.5^2) inputs).  f32 programs keep the
# IEEE-accurate library functions and erf as the reference computes it.
EXPR_FAST = dict(EXPR, exp="__expf({0})", sigmoid="tj_sigmoid_fast({0})", silu="tj_silu_fast({0})",
                 gelu="tj_gelu_fast({0})",
                 div="__fdividef({0}, {1})")


def fast_math_for(dtypes) -> bool:
    """Approximate exp/div only when every value the kernel stores is half precision."""
    ds = set(dtypes)
    return bool(ds) and ds <= {"bf16", "f16"}


def literal(v: float) -> str:
    """f32 literal for a scalar constant (``common.py:113-119``)."""
    v = float(v)
    if v != v:
        return "__int_as_float(0x7fffffff)"
    if v == float("inf"):
        return "__int_as_float(0x7f800000)"
    if v == float("-inf"):
        return "__int_as_float(0xff800000)"
    return f"{v!r}f"


def is_scalar_const(n: PNode) -> bool:
    return n.op == "const" and n.shape == ()


def expr(node: PNode, operand: dict[int, str], fast: bool = False) -> str:
    """Expression of one elementwise node given operand names (scalar consts inline)."""
    args = []
    for i in node.inputs:
        if is_scalar_const(i):
            args.append(literal(i.attrs["value"]))
        elif i.op == "const":
            args.append(literal(i.attrs["value"]))   # shaped const: every element has the value
        else:
            args.append(operand[i.id])
    if node.op in ("transpose", "broadcast_to"):
        return args[0]
    return (EXPR_FAST if fast else EXPR)[node.op].format(*args)


@dataclass
class TMapSpec:
    arg: int                  # index into the kernel's argument list
    dtype: str                # plan dtype
    dims: list[int]           # innermost first (elements)
    strides: list[int]        # bytes, dims 1..rank-1
    box: list[int]
    swizzle: int              # CUtensorMapSwizzle
    param_offset: int = 0
    l2_promotion: int = 2     # CU_TENSOR_MAP_L2_PROMOTION_L2_128B


TMAP_DTYPE = {"f16": 6, "f32": 7, "bf16": 9}


@dataclass
class KernelSource:
    symbol: str
    family: str                         # ewise | copy | row | split | gemm_tc | attention
    source: str
    grid: tuple
    block: tuple
    args: list                          # list of ("node", PNode) | ("status", None)
    smem: int = 0
    cluster: tuple = (1, 1, 1)
    tmaps: list = field(default_factory=list)
    param_bytes: int = 0
    info: dict = field(default_factory=dict)

    def finalize_params(self) -> None:
        """Lay the parameter block out exactly as nvcc lays out the generated struct:
        pointers first, then 64-byte aligned CUtensorMaps."""
        n = len(self.args)
        if self.tmaps:
            off = (8 * n + 63) // 64 * 64
            for t in self.tmaps:
                t.param_offset = off
                off += 128
            self.param_bytes = off
        else:
            self.param_bytes = 8 * n


def params_struct(nptr: int, ntmap: int) -> str:
    lines = ["struct Params {", f"  void* p[{max(nptr, 1)}];"]
    if ntmap:
        lines.append(f"  CUtensorMap tm[{ntmap}];")
    lines.append("};")
    return "\n".join(lines)


def prod(xs) -> int:
    return math.prod(xs) if xs else 1


def coalesce(shape: tuple, stride_sets: list[tuple]) -> tuple[tuple, list[tuple]]:
    """Merge adjacent iteration dims whenever every operand's strides allow it
    (``stride[d] == stride[d+1] * shape[d+1]``), and drop size-1 dims.  Fewer
    dims means cheaper index decomposition in the generated loops."""
    dims = [(s, [st[d] for st in stride_sets]) for d, s in enumerate(shape) if s != 1]
    if not dims:
        return (), [() for _ in stride_sets]
    out = [dims[0]]
    for s, sts in dims[1:]:
        ps, psts = out[-1]
        if all(a == b * s for a, b in zip(psts, sts)):
            out[-1] = (ps * s, sts)
        else:
            out.append((s, sts))
    new_shape = tuple(s for s, _ in out)
    new_strides = [tuple(sts[i] for _, sts in out) for i in range(len(stride_sets))]
    return new_shape, new_strides


def offset_expr(idx_vars: list[str], strides: tuple) -> str:
    terms = []
    for v, s in zip(idx_vars, strides):
        if s == 0:
            continue
        terms.append(v if s == 1 else f"{v} * {s}L")
    return " + ".join(terms) if terms else "0L"


def decompose_stmts(linear: str, shape: tuple, prefix: str) -> tuple[list[str], list[str]]:
    """Split a linear index over ``shape`` into per-dim indices (compile-time divisors)."""
    stmts, names = [], []
    rem = linear
    cs = []
    acc = 1
    for s in reversed(shape):
        cs.append(acc)
        acc *= s
    cs = list(reversed(cs))
    for d, (s, st) in enumerate(zip(shape, cs)):
        name = f"{prefix}{d}"
        names.append(name)
        if d == 0 and len(shape) > 1:
            stmts.append(f"const long {name} = ({rem}) / {st}L;")
            stmts.append(f"const long {prefix}r{d} = ({rem}) - {name} * {st}L;")
            rem = f"{prefix}r{d}"
        elif d == len(shape) - 1:
            stmts.append(f"const long {name} = {rem};")
        else:
            stmts.append(f"const long {name} = ({rem}) / {st}L;")
            stmts.append(f"const long {prefix}r{d} = ({rem}) - {name} * {st}L;")
            rem = f"{prefix}r{d}"
    return stmts, names


HEADER = '#include "tj_common.cuh"\n'
# first statements of every generated kernel without a template prologue: let the program's next
# kernel launch early, then wait for the previous one (programmatic dependent launch)
PDL = "  tj_pdl_launch_dependents();\n  tj_pdl_wait();"


def node_var(n: PNode) -> str:
    return f"v{n.id}"


def kernel_io(k: PKernel) -> tuple[list[PNode], list[PNode]]:
    return list(k.inputs), list(k.outputs)


def pick_vec(dtypes: list[str]) -> int:
    """Elements per 16-byte access for the widest dtype among the operands."""
    return 16 // max(ITEM[d] for d in dtypes)


def find_consumer(n: PNode, nodes: list[PNode]) -> Optional[PNode]:
    for c in nodes:
        if any(i is n for i in c.inputs):
            return c
    return None
