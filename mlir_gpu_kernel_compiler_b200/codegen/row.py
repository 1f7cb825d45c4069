"""Row kernels: LayerNorm / RMSNorm / softmax (and stand-alone last-axis reductions).

Plan semantics (``tensorjit/backends/cuda_backend.py:168-289``, C twin
``c_backend.py:424-564``): a row kernel is a list of stages over ``rows x N``.
A vec stage is elementwise over the N elements of a row; a scalar stage works on
per-row values; a reduce stage runs a per-element prologue, reduces over N
(sum / max / mean = sum / N) and then a per-row scalar epilogue.  Values that a
later stage needs stay on chip.

B200 mapping: each row is owned by a group of ``TPR`` threads (a sub-warp, a
warp, or up to 1024 threads for 8192-wide rows), several rows per CTA so a CTA
always has 256 threads.  Every external row operand is read from HBM exactly
once, with 16-byte vector loads issued up front, and kept in registers for all
stages; every escaping value is written once with 16-byte stores.  Reductions
are warp shuffles, plus one shared-memory exchange per reduction when a row
spans several warps.  With ``N <= 8192`` (``ROW_FUSION_MAX_N``) a row always fits
one CTA's registers, so no cluster is needed.
"""
from __future__ import annotations

from ..plan import PKernel, PNode, broadcast_strides
from .common import (PDL, CTYPE, HEADER, KernelSource, checked, expr, fast_math_for, literal, offset_expr, params_struct,
                     pick_vec, prod, ptr_decl, split_out, split_store_lines, status_decl)

CTA_THREADS = 256


def _geometry(N: int, VEC: int, vpt_target: int = 4) -> tuple[int, int, int]:
    """(threads per row, vectors per thread, rows per CTA): threads per row sized for about
    ``vpt_target`` 16-byte vectors per thread."""
    nvec = (N + VEC - 1) // VEC
    target = max(1, (nvec + vpt_target - 1) // vpt_target)
    tpr = 1
    while tpr < target:
        tpr *= 2
    tpr = max(1, min(tpr, 1024))
    if tpr < 32:
        tpr = max(tpr, 1)
    vpt = (nvec + tpr - 1) // tpr
    rpc = max(1, CTA_THREADS // tpr)
    return tpr, vpt, rpc


def gen_row(k: PKernel, stages: list[PKernel], rows: tuple, N: int, symbol: str,
            kernel_id: int = 0) -> KernelSource:
    rows = tuple(rows)
    nrows = prod(rows)
    vec_shape = rows + (N,)
    ins, outs = list(k.inputs), list(k.outputs)
    inside = {n.id for n in k.nodes}
    escaping = {o.id: j for j, o in enumerate(outs)}
    stage_of = {n.id: si for si, st in enumerate(stages) for n in st.nodes}

    # -- classify where each external input is read ---------------------------
    def is_vec_stage(st: PKernel) -> bool:
        return st.kind == "elementwise" and tuple(st.iter_shape) == vec_shape

    vec_reads: dict[int, PNode] = {}       # external inputs read per element
    for st in stages:
        if is_vec_stage(st):
            readers = st.nodes
        elif st.kind == "reduce":
            pos = st.nodes.index(st.anchor)
            readers = st.nodes[: pos + 1]
        else:
            readers = []
        for n in ins:
            if any(any(i is n for i in r.inputs) for r in readers):
                vec_reads[n.id] = n

    vec_strides = {nid: broadcast_strides(n.shape, vec_shape) for nid, n in vec_reads.items()}
    vec_dtypes = [n.dtype for n in vec_reads.values()] + [o.dtype for o in outs]
    VEC = pick_vec(vec_dtypes) if vec_dtypes else 1
    ok = (VEC > 1 and N % VEC == 0 and "i32" not in vec_dtypes
          and all(st[-1] in (0, 1) and all(s % VEC == 0 for s in st[:-1]) for st in vec_strides.values()))
    if not ok:
        VEC = 1
    fast = fast_math_for([o.dtype for o in outs])
    # the row stays in registers across the stages: with more than two arrays read per element
    # (e.g. x, r and the gain of RMSNorm(x + r)) two vectors per thread keep enough warps resident
    TPR, VPT, RPC = _geometry(N, VEC, 4 if len(vec_reads) <= 2 else 2)
    NVEC = (N + VEC - 1) // VEC if N else 0
    if N == 0:
        VPT = 0
    all_valid = NVEC == TPR * VPT
    NW = (TPR + 31) // 32
    block = TPR * RPC
    grid = (nrows + RPC - 1) // RPC if nrows else 0

    chk = checked()
    nargs = len(ins) + len(outs) + (1 if chk else 0)     # + the status words in a checked build
    L = [HEADER, params_struct(nargs, 0)]
    entry_at = len(L)   # the entry line is added once the per-thread register arrays are known
    if chk:
        L.append("  " + status_decl(len(ins) + len(outs)))
    for j, n in enumerate(ins):
        L.append("  " + ptr_decl(f"in{j}", CTYPE[n.dtype], j, n.numel, True, kernel_id))
    fwd = split_out()       # outputs written as a 3xTF32 GEMM's hi / lo operand copies
    for j, o in enumerate(outs):
        L.append("  " + ptr_decl(f"out{j}", CTYPE[o.dtype], len(ins) + j, o.numel + fwd.get(o.id, 0), False,
                                 kernel_id))
    nred = sum(1 for st in stages if st.kind == "reduce")
    if TPR > 32 and nred:
        L.append(f"  __shared__ float red[{nred}][{RPC}][{NW}];")
    L.append(f"  const int grp = threadIdx.x / {TPR}, t = threadIdx.x % {TPR};")
    L.append(f"  const long r = (long)blockIdx.x * {RPC} + grp;")
    L.append(f"  const bool valid = r < {nrows}L;")
    # row multi-index
    rstr = []
    acc = 1
    for s in reversed(rows):
        rstr.append(acc)
        acc *= s
    rstr = list(reversed(rstr))
    row_idx = []
    rem = "r"
    for d, (s, st) in enumerate(zip(rows, rstr)):
        nm = f"ri{d}"
        row_idx.append(nm)
        if d == len(rows) - 1:
            L.append(f"  const long {nm} = {rem};")
        else:
            L.append(f"  const long {nm} = ({rem}) / {st}L;")
            L.append(f"  const long rr{d} = ({rem}) - {nm} * {st}L;")
            rem = f"rr{d}"
    in_idx = {n.id: j for j, n in enumerate(ins)}

    def vec_base(nid: int) -> str:
        st = vec_strides[nid]
        return offset_expr(row_idx, st[:-1])

    # -- per-element external operands in registers ----------------------------
    # Row data is loaded up front (every load in flight at once); an operand that is the same
    # for every row (a LayerNorm / RMSNorm gain, an L2-resident vector) is loaded vector by
    # vector inside each element loop that reads it, so it never holds a row of registers.
    per_elem = {}   # node id -> ("arr" | "bcast" | "rowconst", name)

    def bcast_load(nid: int) -> list[str]:
        """One 16-byte vector (or one element) of a row-broadcast operand at ``vv``."""
        j = in_idx[nid]
        st = vec_strides[nid]
        cond = "true" if all_valid else f"vv < {NVEC}L"
        if VEC > 1:
            return [f"float X{nid}v[{VEC}];",
                    f"if ({cond}) tj_load_vec(in{j} + {vec_base(nid)} + vv * {VEC}L, X{nid}v);",
                    f"else {{ for (int u = 0; u < {VEC}; ++u) X{nid}v[u] = 0.0f; }}"]
        nn = "vv" if st[-1] == 1 else ("0L" if st[-1] == 0 else f"vv * {st[-1]}L")
        return [f"float X{nid}v[1];", f"X{nid}v[0] = ({cond}) ? tj_f32(in{j}[{vec_base(nid)} + {nn}]) : 0.0f;"]

    def load_loop(nid: int) -> list[str]:
        j = in_idx[nid]
        st = vec_strides[nid]
        out = ["#pragma unroll", f"for (int jv = 0; jv < {VPT}; ++jv) {{", f"  const long vv = t + jv * {TPR}L;"]
        cond = "valid" if all_valid else f"valid && vv < {NVEC}L"
        stride_n = st[-1]
        if VEC > 1:
            out.append(f"  if ({cond}) tj_load_vec(in{j} + {vec_base(nid)} + vv * {VEC}L, X{nid}[jv]);")
            out.append(f"  else {{ for (int u = 0; u < {VEC}; ++u) X{nid}[jv][u] = 0.0f; }}")
        else:
            nn = "vv" if stride_n == 1 else ("0L" if stride_n == 0 else f"vv * {stride_n}L")
            out.append(f"  X{nid}[jv][0] = ({cond}) ? tj_f32(in{j}[{vec_base(nid)} + {nn}]) : 0.0f;")
        out.append("}")
        return out

    for nid, n in vec_reads.items():
        j = in_idx[nid]
        st = vec_strides[nid]
        if VPT == 0:
            continue
        if st[-1] == 0 and N > 1:
            L.append(f"  const float X{nid} = valid ? tj_f32(in{j}[{vec_base(nid)}]) : 0.0f;")
            per_elem[nid] = ("rowconst", f"X{nid}")
            continue
        if all(x == 0 for x in st[:-1]) and nrows > 1:
            per_elem[nid] = ("bcast", f"X{nid}")
            continue
        L.append(f"  float X{nid}[{VPT}][{VEC}];")
        per_elem[nid] = ("arr", f"X{nid}")
        L += ["  " + x for x in load_loop(nid)]

    # -- values computed per element that a later stage reads: register temps --
    computed_vec: set[int] = set()     # nodes computed per element
    computed_scalar: set[int] = set()  # per-row scalars
    temps: set[int] = set()
    for si, st in enumerate(stages):
        if is_vec_stage(st):
            vnodes = st.nodes
        elif st.kind == "reduce":
            vnodes = st.nodes[: st.nodes.index(st.anchor)]
        else:
            vnodes = []
        for n in vnodes:
            if any(u.id in inside and stage_of.get(u.id, si) != si for u in n.users):
                temps.add(n.id)
    # A cheap per-element value a later stage needs is recomputed there from what is live
    # anyway (row operands in registers, per-row scalars) instead of being kept in a per-row
    # register array: fewer registers per thread, more rows in flight per SM.
    node_by_id = {n.id: n for n in k.nodes}
    cheap = {"add", "sub", "mul", "neg", "abs", "maximum", "minimum", "relu", "where"} | ({"div"} if fast else set())
    scalar_ids = {n.id for st in stages for n in _scalar_nodes(st, is_vec_stage(st))}

    def rematerialisable(nid: int, depth: int = 0) -> bool:
        n = node_by_id.get(nid)
        if n is None or n.op not in cheap or depth > 3:
            return False
        for i in n.inputs:
            if i.op == "const" or i.id in per_elem or i.id in scalar_ids:
                continue
            if i.id in inside and not rematerialisable(i.id, depth + 1):
                return False
            if i.id not in inside and i.id not in per_elem:
                return False
        return True

    remat = {nid for nid in temps if rematerialisable(nid)}
    # a value inside a recomputed chain must be recomputable as well
    changed = True
    while changed:
        changed = False
        for nid in list(remat):
            for i in node_by_id[nid].inputs:
                if i.id in inside and i.op != "const" and i.id not in scalar_ids and i.id not in remat:
                    remat.add(i.id)
                    changed = True
    temps -= remat
    for nid in sorted(temps):
        if VPT:
            L.append(f"  float T{nid}[{VPT}][{VEC}];")
    # occupancy hint: the row arrays held across stages plus ~16 registers of addressing and
    # scalars; asking for that many CTAs per SM keeps ptxas from spending registers that would
    # cost a resident CTA (a memory-bound kernel needs rows in flight more than ILP)
    # (rows of one warp or less; a cross-warp reduction needs more scratch registers)
    live = VPT * VEC * (sum(1 for kind, _ in per_elem.values() if kind == "arr") + len(temps))
    min_ctas = min(6, 65536 // (block * (live + 16))) if block and TPR <= 32 else 1
    bounds = f"{block}, {min_ctas}" if min_ctas >= 2 else f"{block}"
    L.insert(entry_at, f'extern "C" __global__ void __launch_bounds__({bounds}) {symbol}(const __grid_constant__ Params prm) {{')
    L.insert(entry_at + 1, PDL)

    def elem_name(nid: int) -> str:
        kind, nm = per_elem[nid]
        return {"arr": f"{nm}[jv][u]", "bcast": f"{nm}v[u]", "rowconst": nm}[kind]

    def remat_expr(n: PNode) -> str:
        mm = {}
        for i in n.inputs:
            if i.op == "const":
                continue
            if i.id in remat:
                mm[i.id] = f"({remat_expr(node_by_id[i.id])})"
            elif i.id in scalar_ids:
                mm[i.id] = f"s{i.id}"
            else:
                mm[i.id] = elem_name(i.id)
        return expr(n, mm, fast)

    def ext_uses(nodes: list[PNode]) -> set[int]:
        """External per-element operands read by ``nodes``, through recomputed values too."""
        used: set[int] = set()

        def walk(n: PNode):
            for i in n.inputs:
                if i.id in per_elem:
                    used.add(i.id)
                elif i.id in remat:
                    walk(node_by_id[i.id])
        for n in nodes:
            walk(n)
        return used
    scal = [n for st in stages for n in _scalar_nodes(st, is_vec_stage(st))]
    if scal:
        L.append("  float " + ", ".join(f"s{n.id} = 0.0f" for n in scal) + ";")

    def operand_map(consumers: list[PNode], per_element: bool) -> dict[int, str]:
        m = {}
        for c in consumers:
            for i in c.inputs:
                if i.id in m or i.op == "const":
                    continue
                if i.id in computed_vec:
                    if i.id in temps:
                        m[i.id] = f"T{i.id}[jv][u]"
                    elif i.id in remat:
                        m[i.id] = f"({remat_expr(node_by_id[i.id])})"
                    else:
                        m[i.id] = f"v{i.id}"
                elif i.id in computed_scalar:
                    m[i.id] = f"s{i.id}"
                elif i.id in per_elem and per_element:
                    m[i.id] = elem_name(i.id)
        return m

    def scalar_load(n: PNode, iter_shape: tuple) -> str:
        st = broadcast_strides(n.shape, tuple(iter_shape))
        idx = list(row_idx) + (["0"] if len(iter_shape) == len(rows) + 1 else [])
        return f"(valid ? tj_f32(in{in_idx[n.id]}[{offset_expr(idx[:len(st)], st)}]) : 0.0f)"

    def emit_elem_loop(nodes: list[PNode], reduce_node: PNode | None = None, red_op: str = "") -> list[str]:
        """Per-element code over the thread's VPT x VEC elements."""
        out = []
        if VPT == 0:
            return out
        esc_nodes = [n for n in nodes if n.id in escaping]
        out.append("#pragma unroll")
        out.append(f"for (int jv = 0; jv < {VPT}; ++jv) {{")
        out.append(f"  const long vv = t + jv * {TPR}L;")
        for nid in sorted(nid for nid in ext_uses(nodes + ([reduce_node] if reduce_node else []))
                          if per_elem[nid][0] == "bcast"):
            out += ["  " + x for x in bcast_load(nid)]
        for n in esc_nodes:
            out.append(f"  float ob{n.id}[{VEC}];")
        out.append("  #pragma unroll")
        out.append(f"  for (int u = 0; u < {VEC}; ++u) {{")
        m = operand_map(nodes + ([reduce_node] if reduce_node else []), True)
        for n in nodes:
            out.append(f"    const float v{n.id} = {expr(n, m, fast)};")
            m[n.id] = f"v{n.id}"
            if n.id in temps:
                out.append(f"    T{n.id}[jv][u] = v{n.id};")
            if n.id in escaping:
                out.append(f"    ob{n.id}[u] = v{n.id};")
        if reduce_node is not None:
            x = reduce_node.inputs[0]
            xv = m.get(x.id) if x.op != "const" else literal(x.attrs["value"])
            upd = f"acc = fmaxf(acc, {xv});" if red_op == "max" else f"acc += {xv};"
            if all_valid:
                out.append(f"    {upd}")
            else:
                out.append(f"    if (vv < {NVEC}L) {{ {upd} }}")
        out.append("  }")
        for n in esc_nodes:
            j = escaping[n.id]
            o = outs[j]
            cond = "valid" if all_valid else f"valid && vv < {NVEC}L"
            if n.id in fwd:
                out.append(f"  if ({cond})")
                out += ["  " + x for x in split_store_lines(f"out{j}", f"r * {N}L + vv * {VEC}L", f"ob{n.id}", VEC,
                                                             fwd[n.id])]
            elif VEC > 1:
                out.append(f"  if ({cond}) tj_store_vec(out{j} + r * {N}L + vv * {VEC}L, ob{n.id});")
            else:
                out.append(f"  if ({cond}) out{j}[r * {N}L + vv] = tj_from<{CTYPE[o.dtype]}>(ob{n.id}[0]);")
        out.append("}")
        return out

    def emit_scalar(nodes: list[PNode], iter_shape: tuple, local: dict[int, str]) -> list[str]:
        out = []
        for n in nodes:
            m = dict(local)
            for i in n.inputs:
                if i.id in m or i.op == "const":
                    continue
                if i.id in computed_scalar:
                    m[i.id] = f"s{i.id}"
                elif i.id in computed_vec:
                    m[i.id] = f"T{i.id}[0][0]" if i.id in temps else f"v{i.id}"
                elif i.id in in_idx:
                    m[i.id] = scalar_load(i, iter_shape)
            out.append(f"s{n.id} = {expr(n, m, fast)};")
            computed_scalar.add(n.id)
            local[n.id] = f"s{n.id}"
            if n.id in escaping:
                j = escaping[n.id]
                out.append(f"if (valid && t == 0) out{j}[r] = tj_from<{CTYPE[outs[j].dtype]}>(s{n.id});")
        return out

    red_slot = 0
    for si, st in enumerate(stages):
        L.append(f"  // stage {si}: {st.kind} {[n.op for n in st.nodes]}")
        L.append("  {")
        if is_vec_stage(st):
            body = emit_elem_loop(st.nodes)
            for n in st.nodes:
                computed_vec.add(n.id)
            L += ["    " + s for s in body]
        elif st.kind == "elementwise":
            L += ["    " + s for s in emit_scalar(st.nodes, tuple(st.iter_shape), {})]
        elif st.kind == "reduce":
            red = st.anchor
            pos = st.nodes.index(red)
            prologue, epilogue = st.nodes[:pos], st.nodes[pos + 1:]
            init = "__int_as_float(0xff800000)" if red.op == "max" else "0.0f"
            L.append(f"    float acc = {init};")
            body = emit_elem_loop(prologue, reduce_node=red, red_op=red.op)
            for n in prologue:
                computed_vec.add(n.id)
            L += ["    " + s for s in body]
            fn = "tj_group_max" if red.op == "max" else "tj_group_sum"
            if TPR <= 32:
                L.append(f"    acc = {fn}<{max(TPR, 1)}>(acc);")
            else:
                comb = "fmaxf(tot, red[%d][grp][w])" if red.op == "max" else "tot + red[%d][grp][w]"
                L.append(f"    acc = {fn}<32>(acc);")
                L.append(f"    if ((t & 31) == 0) red[{red_slot}][grp][t >> 5] = acc;")
                L.append("    __syncthreads();")
                L.append(f"    float tot = {init};")
                L.append("    #pragma unroll")
                L.append(f"    for (int w = 0; w < {NW}; ++w) tot = {comb % red_slot};")
                L.append("    acc = tot;")
                red_slot += 1
            if red.op == "mean":
                L.append(f"    acc = acc / {float(N)!r}f;")
            L.append(f"    s{red.id} = acc;")
            computed_scalar.add(red.id)
            if red.id in escaping:
                j = escaping[red.id]
                L.append(f"    if (valid && t == 0) out{j}[r] = tj_from<{CTYPE[outs[j].dtype]}>(s{red.id});")
            L += ["    " + s for s in emit_scalar(epilogue, tuple(red.shape), {red.id: f"s{red.id}"})]
        else:
            raise NotImplementedError(f"row stage kind {st.kind}")
        L.append("  }")
    L.append("}")
    nbytes = sum(n.nbytes for n in ins) + sum(o.nbytes for o in outs)
    ks = KernelSource(symbol, "row", "\n".join(L), (grid, 1, 1), (block, 1, 1),
                      [("node", n) for n in ins + outs] + ([("status", None)] if chk else []),
                      info={"vec": VEC, "tpr": TPR, "vpt": VPT, "rpc": RPC, "rows": nrows, "n": N, "bytes": nbytes})
    ks.finalize_params()
    return ks


def _scalar_nodes(st: PKernel, vec_stage: bool) -> list[PNode]:
    if vec_stage:
        return []
    if st.kind == "reduce":
        pos = st.nodes.index(st.anchor)
        return st.nodes[pos:]
    return list(st.nodes)
