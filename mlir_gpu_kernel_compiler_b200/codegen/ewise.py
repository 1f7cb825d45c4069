"""Elementwise / copy kernels: the flattened fused DAG as a vectorised grid-stride loop.

Plan semantics (``tensorjit/backends/cuda_backend.py:142-160``): iterate over
``k.iter_shape``; read every kernel input through its access strides (broadcast
dims have stride 0, a transpose reads with permuted strides,
``common.py:18-35``); evaluate the DAG in f32; store every escaping node.

B200 mapping: adjacent dims are coalesced, and when the innermost dim of every
operand is unit-stride (or broadcast) the loop moves 16 bytes per operand per
access (8 bf16 / 4 f32), two vectors per thread in flight, grid sized to the
148 SMs.  Anything else (a transpose that moves the innermost dim, i32) takes
the scalar path with compile-time index decomposition.
"""
from __future__ import annotations

from ..plan import PKernel, access_strides, contiguous_strides, first_consumer
from .common import (PDL, CTYPE, HEADER, NUM_SMS, KernelSource, checked, coalesce, decompose_stmts, expr, fast_math_for,
                     offset_expr, params_struct, pick_vec, prod, ptr_decl, status_decl)

THREADS = 256
UNROLL = 2


def gen_elementwise(k: PKernel, symbol: str, kernel_id: int = 0) -> KernelSource:
    shape = tuple(k.iter_shape)
    numel = prod(shape)
    ins, outs = list(k.inputs), list(k.outputs)
    in_strides = [access_strides(n, first_consumer(n, k.nodes, k.nodes[0]), shape) for n in ins]
    out_strides = contiguous_strides(shape)
    cshape, cstr = coalesce(shape, in_strides + [out_strides])
    cin = cstr[: len(ins)]
    dtypes = [n.dtype for n in ins + outs]
    VEC = pick_vec(dtypes)
    vec_ok = (
        numel > 0 and len(cshape) > 0 and "i32" not in dtypes and VEC > 1
        and cshape[-1] % VEC == 0
        and all(st[-1] in (0, 1) for st in cin)
        and all(s % VEC == 0 for st in cin for s in st[:-1])
    )
    if not vec_ok:
        VEC = 1

    chk = checked()
    L = [HEADER, params_struct(len(ins) + len(outs) + (1 if chk else 0), 0),
         f'extern "C" __global__ void __launch_bounds__({THREADS}) {symbol}(const __grid_constant__ Params prm) {{', PDL]
    if chk:
        L.append("  " + status_decl(len(ins) + len(outs)))
    for j, n in enumerate(ins):
        L.append("  " + ptr_decl(f"in{j}", CTYPE[n.dtype], j, n.numel, True, kernel_id))
    for j, o in enumerate(outs):
        L.append("  " + ptr_decl(f"out{j}", CTYPE[o.dtype], len(ins) + j, o.numel, False, kernel_id))
    names = {n.id: f"x{j}" for j, n in enumerate(ins)}
    fast = fast_math_for([o.dtype for o in outs])
    nvec = numel // VEC
    need_idx = any(st != out_cs for st, out_cs in zip(cin, [cstr[-1]] * len(cin)))

    def body(vexpr: str, tag: str) -> tuple[list[str], list[str]]:
        """(load lines, compute+store lines) for the vector at index ``vexpr``."""
        loads, comp = [], []
        loads.append(f"const long e{tag} = ({vexpr}) * {VEC}L;")
        if need_idx and cshape:
            st, idx = decompose_stmts(f"e{tag}", cshape, f"i{tag}_")
            loads += st
        else:
            idx = None
        for j, n in enumerate(ins):
            off = offset_expr(idx, cin[j]) if idx is not None else f"e{tag}"
            if VEC > 1 and cin[j][-1] == 1:
                loads.append(f"float a{j}{tag}[{VEC}]; tj_load_vec(in{j} + ({off}), a{j}{tag});")
            else:
                loads.append(f"const float s{j}{tag} = tj_f32(in{j}[{off}]);")
        comp.append(f"float o{tag}[{len(outs)}][{VEC}];")
        comp.append("#pragma unroll")
        comp.append(f"for (int u = 0; u < {VEC}; ++u) {{")
        for j, n in enumerate(ins):
            src = f"a{j}{tag}[u]" if (VEC > 1 and cin[j][-1] == 1) else f"s{j}{tag}"
            comp.append(f"  const float x{j} = {src};")
        local = dict(names)
        for n in k.nodes:
            comp.append(f"  const float v{n.id} = {expr(n, local, fast)};")
            local[n.id] = f"v{n.id}"
        for j, o in enumerate(outs):
            comp.append(f"  o{tag}[{j}][u] = {local[o.id]};")
        comp.append("}")
        for j, o in enumerate(outs):
            if VEC > 1:
                comp.append(f"tj_store_vec(out{j} + e{tag}, o{tag}[{j}]);")
            else:
                comp.append(f"out{j}[e{tag}] = tj_from<{CTYPE[o.dtype]}>(o{tag}[{j}][0]);")
        return loads, comp

    L.append(f"  const long stride = (long)gridDim.x * {THREADS}L;")
    L.append(f"  long v = (long)blockIdx.x * {THREADS}L + threadIdx.x;")
    if nvec > 0:
        l0, c0 = body("v", "A")
        l1, c1 = body("v + stride", "B")
        L.append(f"  for (; v + stride < {nvec}L; v += {UNROLL} * stride) {{")
        L += ["    " + s for s in l0 + l1 + c0 + c1]
        L.append("  }")
        L.append(f"  if (v < {nvec}L) {{")
        L += ["    " + s for s in l0 + c0]
        L.append("  }")
    L.append("}")
    grid = max(1, min((nvec + THREADS * UNROLL - 1) // (THREADS * UNROLL), NUM_SMS * 8)) if nvec else 0
    ks = KernelSource(symbol, "copy" if k.kind == "copy" else "ewise", "\n".join(L), (grid, 1, 1), (THREADS, 1, 1),
                      [("node", n) for n in ins + outs] + ([("status", None)] if chk else []),
                      info={"vec": VEC, "numel": numel, "shape": list(cshape),
                            "bytes": sum(n.nbytes for n in ins) + sum(o.nbytes for o in outs)})
    ks.finalize_params()
    return ks
