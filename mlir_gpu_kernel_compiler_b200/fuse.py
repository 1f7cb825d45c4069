"""Plan rewrites the B200 backend applies before code generation.

tensorjit's fusion pass (``tensorjit/passes/fusion.py:104-330``) stops at matmul
boundaries, so scaled-dot-product attention reaches a backend as three kernels:

    k_i    matmul   S = Q @ K^T            (trans_b) [* c | / c]       -> [.., Sq, Sk]
    k_i+1  row      P = exp(S - max(S)) / sum(exp(S - max(S)))  over the last axis
    k_i+2  matmul   O = P @ V                                            -> [.., Sq, Dv]

and, when Q/K/V come from a head split, with ``copy`` kernels (transposes) before
them and after O.  ``fuse_attention`` replaces such a chain by one kernel of kind
``attention`` whose score and probability matrices never reach HBM, and folds a
transpose that only feeds Q, K or V (or only consumes O) into that kernel's
addressing, so the copy kernel disappears as well.

``fuse_shared_a_gemms`` merges consecutive bare GEMMs that read the same A operand (the
q / k / v projections of a transformer block) into one ``matmul_multi`` kernel, and
``absorb_elementwise_epilogues`` moves an elementwise kernel that only post-processes a GEMM's
output (a residual add) into that GEMM's epilogue.

The attention rewrite is semantic-preserving for the plan's outputs only: S and P must not
escape (not graph outputs, no user outside the chain), otherwise the chain is left
as it is (e.g. a graph that returns the attention probabilities).  The memory plan
of the rewritten program no longer holds S, P or the folded transposes.

A fused kernel's ``attrs`` carry what code generation needs:
    q, k, v: (source node, element strides over the logical [*batch, S, D] index)
    out:     (node written, element strides over [*batch, Sq, Dv])
    batch, sq, sk, d, dv, dtype, scale
"""
from __future__ import annotations

import os
from typing import Optional

from .plan import PKernel, PNode, PProgram, contiguous_strides

ATTENTION_HEAD_DIMS = (64,)


def _const_value(n: PNode) -> Optional[float]:
    if n.op == "const" and "value" in n.attrs:
        return float(n.attrs["value"])
    return None


def _is_last_axis(node: PNode, rank: int) -> bool:
    ax = node.attrs.get("axis")
    return ax in (-1, rank - 1) and bool(node.attrs.get("keepdim"))


def _only_users(n: PNode, allowed: set[int]) -> bool:
    return bool(n.users) and all(u.id in allowed for u in n.users)


def _copy_transpose_producer(plan: PProgram, x: PNode, consumer: PNode, escaping: set[int]):
    """The copy kernel that materialises ``x`` as a plain transpose read only by
    ``consumer`` (so the copy can be folded into the consumer's addressing)."""
    if x.op != "transpose" or x.id in escaping or not _only_users(x, {consumer.id}):
        return None
    for ki, k in enumerate(plan.kernels):
        if k.kind == "copy" and len(k.nodes) == 1 and k.nodes[0] is x and k.outputs == [x]:
            return ki
    return None


def _operand(plan: PProgram, x: PNode, consumer: PNode, escaping: set[int]):
    """(memory node, logical strides, folded copy kernel index or None) for a matmul operand."""
    ki = _copy_transpose_producer(plan, x, consumer, escaping)
    if ki is not None:
        src = x.inputs[0]
        cs = contiguous_strides(src.shape)
        return src, tuple(cs[p] for p in x.attrs["perm"]), ki
    return x, contiguous_strides(x.shape), None


def match_attention(plan: PProgram, i: int, escaping: set[int]) -> Optional[dict]:
    ks = plan.kernels
    if i + 2 >= len(ks):
        return None
    k1, k2, k3 = ks[i], ks[i + 1], ks[i + 2]
    if (k1.kind, k2.kind, k3.kind) != ("matmul", "row", "matmul"):
        return None
    mm1 = k1.anchor
    if mm1 is None or mm1.op != "matmul" or not mm1.attrs.get("trans_b"):
        return None
    scale = 1.0
    if len(k1.nodes) == 1:
        s_node = mm1
    elif len(k1.nodes) == 2:
        e = k1.nodes[1]
        others = [x for x in e.inputs if x is not mm1]
        if len(e.inputs) != 2 or len(others) != 1 or _const_value(others[0]) is None:
            return None
        c = _const_value(others[0])
        if e.op == "mul":
            scale = c
        elif e.op == "div" and e.inputs[0] is mm1 and c != 0.0:
            scale = 1.0 / c
        else:
            return None
        if not _only_users(mm1, {e.id}):
            return None
        s_node = e
    else:
        return None
    if not (scale > 0.0 and scale < float("inf")):
        return None
    if k1.outputs != [s_node] or s_node.id in escaping or mm1.id in escaping:
        return None
    rank = len(s_node.shape)
    if rank < 2:
        return None
    # the row kernel must be exactly a last-axis softmax of S
    by_op: dict[str, list[PNode]] = {}
    for n in k2.nodes:
        by_op.setdefault(n.op, []).append(n)
    if sorted(by_op) != ["div", "exp", "max", "sub", "sum"] or any(len(v) != 1 for v in by_op.values()):
        return None
    mx, sb, ex, sm, dv = by_op["max"][0], by_op["sub"][0], by_op["exp"][0], by_op["sum"][0], by_op["div"][0]
    if not (mx.inputs == [s_node] and _is_last_axis(mx, rank) and sb.inputs == [s_node, mx]
            and ex.inputs == [sb] and sm.inputs == [ex] and _is_last_axis(sm, rank) and dv.inputs == [ex, sm]):
        return None
    if k2.outputs != [dv] or dv.id in escaping or not _only_users(s_node, {mx.id, sb.id}):
        return None
    mm2 = k3.anchor
    if mm2 is None or mm2.op != "matmul" or mm2.attrs.get("trans_b") or k3.nodes != [mm2] or k3.outputs != [mm2]:
        return None
    if mm2.inputs[0] is not dv or not _only_users(dv, {mm2.id}):
        return None
    q, kk, v = mm1.inputs[0], mm1.inputs[1], mm2.inputs[1]
    dt = q.dtype
    if dt not in ("bf16", "f16") or any(x.dtype != dt for x in (kk, v, mm1, s_node, mx, sb, ex, sm, dv, mm2)):
        return None
    if len(q.shape) != rank or len(kk.shape) != rank or len(v.shape) != rank:
        return None
    batch = tuple(q.shape[:-2])
    sq, d = q.shape[-2:]
    sk = kk.shape[-2]
    dv_ = v.shape[-1]
    if tuple(kk.shape[:-2]) != batch or tuple(v.shape[:-2]) != batch or kk.shape[-1] != d or v.shape[-2] != sk:
        return None
    if d not in ATTENTION_HEAD_DIMS or dv_ != d or sq < 1 or sk < 1:
        return None
    if sum(1 for b in batch if b != 1) > 3:
        return None
    folded = []
    ops = {}
    for name, x, consumer in (("q", q, mm1), ("k", kk, mm1), ("v", v, mm2)):
        src, st, ki = _operand(plan, x, consumer, escaping)
        if st[-1] != 1 or any(s % 8 for s, e in zip(st[:-1], x.shape[:-1]) if e != 1):
            return None   # TMA: unit-stride rows, 16-byte aligned row/batch strides
        ops[name] = (src, st)
        if ki is not None:
            folded.append(ki)
    # O, possibly written through a transpose that is its only consumer
    out_node, out_st = mm2, contiguous_strides(mm2.shape)
    if mm2.id not in escaping and len(mm2.users) == 1 and mm2.users[0].op == "transpose":
        t = mm2.users[0]
        for ki, k in enumerate(ks):
            if k.kind == "copy" and len(k.nodes) == 1 and k.nodes[0] is t and k.outputs == [t] and ki == i + 3:
                perm = t.attrs["perm"]
                cs_t = contiguous_strides(t.shape)
                st = [0] * len(perm)
                for dpos, p in enumerate(perm):
                    st[p] = cs_t[dpos]
                if st[-1] == 1 and all(s % 8 == 0 for s in st[:-1]):
                    out_node, out_st = t, tuple(st)
                    folded.append(ki)
                break
    return {
        "kernels": (i, i + 1, i + 2), "folded": sorted(set(folded)),
        "nodes": [mm1] + ([s_node] if s_node is not mm1 else []) + [mx, sb, ex, sm, dv, mm2],
        "q": ops["q"], "k": ops["k"], "v": ops["v"], "out": (out_node, out_st),
        "batch": batch, "sq": sq, "sk": sk, "d": d, "dv": dv_, "dtype": dt, "scale": scale,
    }


def fuse_attention(plan: PProgram) -> PProgram:
    """Return ``plan`` with every eligible attention chain replaced by one kernel
    (a new ``PProgram`` sharing the nodes; ``plan`` itself is not modified)."""
    escaping = {plan.resolve(o).id for o in plan.outputs}
    matches = []
    i = 0
    while i < len(plan.kernels):
        m = match_attention(plan, i, escaping)
        if m is not None:
            matches.append(m)
            i += 3
        else:
            i += 1
    if not matches:
        return plan
    drop: set[int] = set()
    replace: dict[int, PKernel] = {}
    for m in matches:
        i0, i1, i2 = m["kernels"]
        drop.update((i1, i2))
        drop.update(m["folded"])
        srcs: list[PNode] = []
        for name in ("q", "k", "v"):
            if all(s is not m[name][0] for s in srcs):
                srcs.append(m[name][0])
        out_node = m["out"][0]
        nodes = list(m["nodes"]) + ([out_node] if out_node is not m["nodes"][-1] else [])
        fk = PKernel(kind="attention", nodes=nodes, anchor=m["nodes"][0], inputs=srcs, outputs=[out_node],
                     iter_shape=tuple(out_node.shape))
        fk.attrs = {k: m[k] for k in ("q", "k", "v", "out", "batch", "sq", "sk", "d", "dv", "dtype", "scale")}
        replace[i0] = fk
    kernels = []
    for ki, k in enumerate(plan.kernels):
        if ki in replace:
            kernels.append(replace[ki])
        elif ki not in drop:
            kernels.append(k)
    return PProgram(name=plan.name, nodes=plan.nodes, inputs=plan.inputs, outputs=plan.outputs, kernels=kernels,
                    aliases=plan.aliases, meta=dict(plan.meta, fused_attention=len(matches)))


def _subdims(sizes_strides: list[tuple[int, int]]) -> list[tuple[int, int]]:
    """(size, element stride) pairs, outermost first, with size-1 dims dropped and adjacent
    dims merged where the outer one steps over the inner one exactly."""
    out: list[tuple[int, int]] = []
    for size, st in sizes_strides:
        if size == 1:
            continue
        if out and out[-1][1] == st * size:
            out[-1] = (out[-1][0] * size, st)
        else:
            out.append((size, st))
    return out


def strided_operand_layout(plan: PProgram, k: PKernel, which: int, escaping: set[int],
                           taken: frozenset = frozenset(), gather: bool = False) -> Optional[dict]:
    """How operand ``which`` (0 = A, 1 = B) of a bf16/f16 matmul kernel could be read straight
    from the source of the ``copy`` kernel (a transpose) that materialises it, instead of from
    the copy's output.

    The operand O[batch.., rows, k] (rows = M for A, N for a ``trans_b`` B), or O[batch.., k, n]
    for an N-major B (``n_major``: then its N dims come first, as rows), is the transpose T of X,
    optionally reshaped: each logical dim of O is a run of T's dims, and T's dim i has X's stride
    for dim perm[i].  The GEMM reads O by TMA through one tensor map over X whose dims are K0 [K1]
    R0 [R1] [B0 [B1]] (innermost first within each part): K0 unit-stride (a multiple of the
    64-element k-block when K1 exists), a row tile never straddles R1 (R0 a multiple of 128 for
    A, of 256 for B), at most two batch dims, rank <= 5, 16-byte strides; X not read elsewhere in
    the kernel, T read only here and not a program output.  ``taken``: copy kernels already
    folded into the other operand.  Returns {"src", "copy", "dims": [(size, stride)], "k_dims",
    "r_dims", "batch_dims", "n_major"} or None.

    ``gather``: the operand goes through the GEMM's pack / split pre-pass, which computes each
    element's offset in X itself: any dtype, any number of sub-dims, none of the tensor-map
    conditions; returns {"src", "copy", "k", "r", "b": [(size, stride)] innermost first}."""
    mm = k.anchor
    if k.kind != "matmul" or mm is None or mm.op != "matmul":
        return None
    n_major = which == 1 and not mm.attrs.get("trans_b")
    a, b = mm.inputs
    o = mm.inputs[which]
    t = plan.resolve(o)
    if (t.op != "transpose" or (not gather and (a.dtype not in ("bf16", "f16") or b.dtype != a.dtype))
            or t.id in escaping or o.id in escaping):
        return None
    copy_i = next((i for i, c in enumerate(plan.kernels) if c.kind == "copy" and len(c.nodes) == 1
                   and c.nodes[0] is t and c.outputs == [t]), None)
    if copy_i is None or copy_i in taken:
        return None
    # T (and the alias O) is read by this matmul alone, once, as this operand
    ids = {t.id, o.id}
    reads = lambda n: n.id in ids or plan.resolve(n).id == t.id  # noqa: E731
    readers = [j for j, c in enumerate(plan.kernels) if j != copy_i and any(reads(n) for n in c.inputs)]
    if readers != [plan.kernels.index(k)] or sum(1 for n in k.nodes for i in n.inputs if reads(i)) != 1:
        return None
    x = t.inputs[0]
    if any(n is x or plan.resolve(n) is plan.resolve(x) for n in k.inputs):   # X also read directly
        return None
    perm = t.attrs["perm"]
    cs = contiguous_strides(x.shape)
    tdims = [(int(t.shape[i]), int(cs[perm[i]])) for i in range(len(t.shape))]
    # each logical dim of O = a run of consecutive T dims (a reshape that only merges)
    groups, j = [], 0
    for size in o.shape:
        run, prod_ = [], 1
        while prod_ < size:
            if j >= len(tdims):
                return None
            run.append(tdims[j])
            prod_ *= tdims[j][0]
            j += 1
        if prod_ != size:
            return None
        groups.append(run)
    if any(tdims[q][0] != 1 for q in range(j, len(tdims))):
        return None
    inner, outer = _subdims(groups[-1])[::-1], _subdims(groups[-2])[::-1]     # innermost first
    k_dims, r_dims = (outer, inner) if n_major else (inner, outer)
    batch_dims = _subdims([d for g in groups[:-2] for d in g])[::-1]
    if gather:
        return {"src": x, "copy": copy_i, "k": k_dims, "r": r_dims, "b": batch_dims}
    if not inner or inner[0][1] != 1 or len(k_dims) > 2 or len(r_dims) > 2 or len(batch_dims) > 2:
        return None
    if len(inner) == 1 and int(o.shape[-1]) % 8:
        return None
    # a k-block (64) never straddles two K sub-dims; a row tile (128 rows of A, a 256-wide B tile,
    # 64-column chunks of an N-major B) never straddles two row sub-dims
    if len(k_dims) == 2 and k_dims[0][0] % 64:
        return None
    if len(r_dims) == 2 and r_dims[0][0] % (128 if which == 0 else 256):
        return None
    dims = (r_dims + k_dims if n_major else k_dims + r_dims) + batch_dims
    if len(dims) < 3 or len(dims) > 5 or any((st * 2) % 16 for _, st in dims[1:]):
        return None
    return {"src": x, "copy": copy_i, "dims": dims, "k_dims": len(k_dims), "r_dims": len(r_dims),
            "batch_dims": len(batch_dims), "n_major": n_major}


def strided_a_layout(plan: PProgram, k: PKernel, escaping: set[int]) -> Optional[dict]:
    """``strided_operand_layout`` of the A operand."""
    return strided_operand_layout(plan, k, 0, escaping)


def fold_copies_into_gemm(plan: PProgram) -> PProgram:
    """A transpose ``copy`` kernel whose output only feeds a GEMM operand is removed, saving its
    HBM round trip: a bf16/f16 GEMM reads that operand from the transpose's source through a
    permuted-stride tensor map (``strided_operand_layout``); a GEMM whose operands go through a
    pack / split pre-pass (f32 3xTF32, odd pitches) has that launch gather them from the source
    instead.  Outputs are unchanged."""
    from .codegen.gemm import gemm_form

    escaping = {plan.resolve(o).id for o in plan.outputs}
    drop, replace = set(), {}
    for i, k in enumerate(plan.kernels):
        if k.kind != "matmul" or k.anchor is None or k.anchor.op != "matmul":
            continue
        lay_a = strided_operand_layout(plan, k, 0, escaping)
        lay_b = strided_operand_layout(plan, k, 1, escaping,
                                       frozenset({lay_a["copy"]}) if lay_a else frozenset())
        f = gemm_form(k)
        if f.mode != "f16" or f.pack_a or f.pack_b:
            lay_a = lay_b = None
        if lay_a is None and lay_b is None:
            # operands copied by the GEMM's pack / split pre-pass: that launch gathers them from
            # the transpose's source instead (3xTF32 splits both operands; a pack, those it packs)
            if f.mode not in ("x3", "f16"):
                continue
            ga = strided_operand_layout(plan, k, 0, escaping, gather=True) if f.mode == "x3" or f.pack_a else None
            gb = (strided_operand_layout(plan, k, 1, escaping, frozenset({ga["copy"]}) if ga else frozenset(),
                                         gather=True) if f.mode == "x3" or f.pack_b else None)
            if ga is None and gb is None:
                continue
            attrs, subst = dict(k.attrs), {}
            for name, lay, node in (("a_gather", ga, k.anchor.inputs[0]), ("b_gather", gb, k.anchor.inputs[1])):
                if lay is not None:
                    attrs[name] = {key: lay[key] for key in ("src", "k", "r", "b")}
                    subst[node.id] = lay["src"]
                    drop.add(lay["copy"])
            fk = PKernel(kind="matmul", nodes=list(k.nodes), anchor=k.anchor,
                         inputs=[subst.get(n.id, n) for n in k.inputs], outputs=list(k.outputs),
                         iter_shape=tuple(k.iter_shape))
            fk.attrs = attrs
            replace[i] = fk
            continue
        attrs, subst = dict(k.attrs), {}
        for name, lay, node in (("a_strided", lay_a, k.anchor.inputs[0]), ("b_strided", lay_b, k.anchor.inputs[1])):
            if lay is not None:
                attrs[name] = {key: lay[key] for key in ("src", "dims", "k_dims", "r_dims", "batch_dims",
                                                         "n_major")}
                subst[node.id] = lay["src"]
                drop.add(lay["copy"])
        fk = PKernel(kind="matmul", nodes=list(k.nodes), anchor=k.anchor,
                     inputs=[subst.get(n.id, n) for n in k.inputs], outputs=list(k.outputs),
                     iter_shape=tuple(k.iter_shape))
        fk.attrs = attrs
        replace[i] = fk
    if not replace:
        return plan
    kernels = [replace.get(i, k) for i, k in enumerate(plan.kernels) if i not in drop]
    return PProgram(name=plan.name, nodes=plan.nodes, inputs=plan.inputs, outputs=plan.outputs, kernels=kernels,
                    aliases=plan.aliases, meta=dict(plan.meta, folded_copies=len(drop)))


def _plain_shared_a_matmul(k: PKernel):
    """(A, B, N) of a kernel that is a bare bf16/f16 ``A @ Bᵀ`` (2-D, no epilogue), else None."""
    if (k.kind != "matmul" or len(k.nodes) != 1 or k.outputs != [k.anchor]
            or any(k.attrs.get(f) for f in ("a_strided", "b_strided", "a_gather", "b_gather"))):
        return None
    mm = k.anchor
    if mm.op != "matmul" or not mm.attrs.get("trans_b"):
        return None
    a, b = mm.inputs
    if len(a.shape) != 2 or len(b.shape) != 2 or a.dtype not in ("bf16", "f16") or b.dtype != a.dtype:
        return None
    if mm.dtype != a.dtype or a.shape[1] != b.shape[1] or a.shape[1] % 8:
        return None
    return a, b, b.shape[0]


def fuse_shared_a_gemms(plan: PProgram) -> PProgram:
    """Consecutive bare GEMMs ``A @ B_gᵀ`` with the same A (q/k/v or gate/up projections)
    become one kernel of kind ``matmul_multi`` over the concatenated N (every N_g a multiple
    of the 256-column tile, so no tile straddles two products).  Outputs are unchanged."""
    ks = plan.kernels
    out: list[PKernel] = []
    i = 0
    changed = False
    while i < len(ks):
        first = _plain_shared_a_matmul(ks[i])
        run = [i]
        if first is not None and first[2] % 256 == 0:
            j = i + 1
            while j < len(ks):
                nxt = _plain_shared_a_matmul(ks[j])
                if nxt is None or nxt[0] is not first[0] or nxt[2] % 256 or nxt[0].dtype != first[0].dtype:
                    break
                run.append(j)
                j += 1
        if len(run) < 2:
            out.append(ks[i])
            i += 1
            continue
        parts = []
        for kj in run:
            a, b, n = _plain_shared_a_matmul(ks[kj])
            parts.append((b, ks[kj].anchor, n))
        a = first[0]
        fk = PKernel(kind="matmul_multi", nodes=[ks[kj].anchor for kj in run], anchor=ks[run[0]].anchor,
                     inputs=[a] + [p_[0] for p_ in parts], outputs=[p_[1] for p_ in parts],
                     iter_shape=(a.shape[0], sum(p_[2] for p_ in parts)))
        fk.attrs = {"a": a, "parts": parts}
        out.append(fk)
        i = run[-1] + 1
        changed = True
    if not changed:
        return plan
    return PProgram(name=plan.name, nodes=plan.nodes, inputs=plan.inputs, outputs=plan.outputs, kernels=out,
                    aliases=plan.aliases, meta=dict(plan.meta, fused_shared_a=True))


def absorb_elementwise_epilogues(plan: PProgram) -> PProgram:
    """An elementwise kernel right after a matmul kernel joins that GEMM's epilogue when it
    consumes the GEMM's only output, elementwise over exactly that output's shape, and nothing
    else reads that output (it is no graph output either): e.g. the residual add after a
    transformer MLP's down projection.  The GEMM then evaluates the added nodes on its f32
    accumulator tile and stores only their outputs, so the intermediate never reaches HBM (and
    is not rounded to the storage dtype in between).  The elementwise kernel's other inputs are
    produced before the GEMM runs, since the plan is in execution order."""
    from .codegen.common import EXPR
    from .plan import access_strides, first_consumer

    escaping = {plan.resolve(o).id for o in plan.outputs}
    ks = plan.kernels
    out: list[PKernel] = []
    changed = 0
    i = 0
    while i < len(ks):
        g = ks[i]
        e = ks[i + 1] if i + 1 < len(ks) else None
        if (e is not None and g.kind == "matmul" and e.kind == "elementwise" and len(g.outputs) == 1
                and g.outputs[0] in e.inputs):
            o = g.outputs[0]
            shape = tuple(o.shape)
            ok = (o.id not in escaping and tuple(e.iter_shape) == shape and _only_users(o, {n.id for n in e.nodes})
                  and all(n.op in EXPR for n in e.nodes))
            if ok:
                c = first_consumer(o, e.nodes, e.nodes[0])
                ok = tuple(access_strides(o, c, shape)) == contiguous_strides(shape)
            if ok:
                inputs = list(g.inputs) + [n for n in e.inputs if n is not o and n not in g.inputs]
                fk = PKernel(kind="matmul", nodes=list(g.nodes) + list(e.nodes), anchor=g.anchor, inputs=inputs,
                             outputs=list(e.outputs), iter_shape=tuple(g.iter_shape))
                fk.attrs = dict(g.attrs)
                out.append(fk)
                changed += 1
                i += 2
                continue
        out.append(g)
        i += 1
    if not changed:
        return plan
    return PProgram(name=plan.name, nodes=plan.nodes, inputs=plan.inputs, outputs=plan.outputs, kernels=out,
                    aliases=plan.aliases, meta=dict(plan.meta, absorbed_epilogues=changed))


def fuse(plan: PProgram) -> PProgram:
    """All backend rewrites (``TENSORJIT_B200_FUSE=0`` disables them): attention chains,
    transposes folded into the GEMM operands that read them, GEMMs that share their A operand,
    then elementwise kernels absorbed into the GEMM before them."""
    if os.environ.get("TENSORJIT_B200_FUSE", "1") == "0":
        return plan
    return absorb_elementwise_epilogues(fuse_shared_a_gemms(fold_copies_into_gemm(fuse_attention(plan))))
