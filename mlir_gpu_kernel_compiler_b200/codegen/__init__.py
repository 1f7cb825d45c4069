"""Plan -> sm_100a kernel sources.

``generate`` walks the fused plan in order and dispatches on ``Kernel.kind``
exactly like the reference backend (``tensorjit/backends/cuda_backend.py:437-456``):
elementwise/copy -> vectorised grid-stride kernel, row -> staged row kernel,
reduce -> row kernel with one stage, matmul -> the tcgen05 GEMM (bf16/f16 operands
read in place or after a pack pre-pass; everything else as 3xTF32 after an operand split
pre-pass; see ``gemm.gemm_form``); ``attention`` (the matmul -> softmax -> matmul chain
``fuse.py`` folds into one kernel) -> the fused tcgen05 attention kernel; ``matmul_multi``
(GEMMs sharing A, also from ``fuse.py``) -> one tcgen05 GEMM over the concatenated N.  A plan kernel can therefore become several launches;
``KernelSource.info["index"]`` names the plan kernel each launch belongs to.
"""
from __future__ import annotations

import os

from ..plan import PProgram
from .attention import gen_attention
from .common import KernelSource, checked_build, split_forwarding, store_mode
from .ewise import gen_elementwise
from .gemm import gen_gemm_multi, gen_matmul
from .row import gen_row


def generate(plan: PProgram, tiles: dict | None = None, prefix: str = "tj", checked: bool = False,
             tma_store: bool = True) -> list[KernelSource]:
    """``checked``: emit the checked build (every global access bounds-checked against its
    operand, TMA coordinates and TMEM columns checked in the templates; compile with
    -DTJ_CHECKED, ``toolchain.CHECKED_FLAGS``).  ``tma_store=False``: GEMM epilogues store
    with plain 16-byte stores (for outputs that may be a peer GPU's memory)."""
    with checked_build(checked), store_mode(tma_store):
        return _generate(plan, tiles, prefix)


def _generate(plan: PProgram, tiles: dict | None, prefix: str) -> list[KernelSource]:
    """With ``TENSORJIT_B200_FORWARD=1``, two passes when 3xTF32 operands can be forwarded
    (``_split_forwarding``): the first lays out every matmul's workspace, the second has the
    producers of forwarded operands write the hi / lo copies there and drops those operands from
    the split launches.  Off by default: on cfg1 the GEMM epilogue that then writes both copies
    costs more (its f32 stores are row-strided) than the split launch's activation pass saves."""
    first = _generate_pass(plan, tiles, prefix, {})
    if os.environ.get("TENSORJIT_B200_FORWARD", "0") != "1":   # off by default: measured slower
        return first
    fwd, skip = _split_forwarding(plan, first)
    if not fwd:
        return first
    with split_forwarding({nid: delta for nid, (_, delta) in fwd.items()}, skip):
        return _generate_pass(plan, tiles, prefix, fwd)


def _split_forwarding(plan: PProgram, ks: list[KernelSource]) -> tuple[dict, dict]:
    """f32 operands of 3xTF32 GEMMs (vectorised split form) that their producer can write as
    the hi / lo copies directly: the node is an intermediate (not a program input or output,
    no alias) read by that matmul alone, once, as its A or B operand, and produced by a row
    kernel (as a full row) or by a matmul's epilogue.  Returns ({node id: (workspace offset of
    the hi copy, elements from hi to lo)}, {matmul kernel index: {"a" / "b"}})."""
    escaping = {plan.resolve(o).id for o in plan.outputs}
    producer = {o.id: i for i, k in enumerate(plan.kernels) for o in k.outputs}
    readers: dict[int, list[int]] = {}
    for i, k in enumerate(plan.kernels):
        for n in k.inputs:
            readers.setdefault(n.id, []).append(i)
    fwd, skip = {}, {}
    for g in ks:
        x3v = g.info.get("x3_vec")
        if not x3v:
            continue
        ci, base = g.info["index"], g.info.get("scratch_base", 0)
        kc = plan.kernels[ci]
        for role, (nid, hi, lo) in x3v.items():
            node = next((n for n in kc.inputs if n.id == nid), None)
            if (node is None or node.op == "input" or node.dtype != "f32" or nid in escaping
                    or readers.get(nid) != [ci] or plan.resolve(node) is not node
                    or sum(1 for n in kc.nodes for i in n.inputs if i is node) != 1):
                continue
            pi = producer.get(nid)
            if pi is None or pi >= ci:
                continue
            pk = plan.kernels[pi]
            full_row = pk.kind == "row" and tuple(node.shape) == tuple(pk.rows) + (int(pk.n),)
            if not (full_row or pk.kind == "matmul"):
                continue
            fwd[nid] = (base + hi, (lo - hi) // 4)
            skip.setdefault(ci, set()).add(role)
    return fwd, skip


def _generate_pass(plan: PProgram, tiles: dict | None, prefix: str, fwd: dict) -> list[KernelSource]:
    """Each matmul with a pre-pass gets a workspace region of its own (``info["scratch_base"]``,
    offsets relative to the program's workspace): its pre-pass may split or pack the program
    inputs among its operands before waiting for the kernels ahead of it (programmatic
    dependent launch), which is only safe when no earlier matmul still reads that region.
    ``fwd``: outputs written as another matmul's hi / lo operand copies (their argument is
    that workspace offset instead of the node's own storage)."""
    out: list[KernelSource] = []
    ws_base = 0
    for idx, k in enumerate(plan.kernels):
        sym = f"{prefix}_{k.kind}_{idx}"
        if k.kind in ("elementwise", "copy"):
            ks = gen_elementwise(k, sym, idx)
        elif k.kind == "row":
            ks = gen_row(k, k.stages, tuple(k.rows), int(k.n), sym, idx)
        elif k.kind == "reduce":
            x = k.anchor.inputs[0]
            ks = gen_row(k, [k], tuple(x.shape[:-1]), int(x.shape[-1]) if x.shape else 1, sym, idx)
        elif k.kind == "attention":
            ks = gen_attention(k, sym, idx)
        elif k.kind == "matmul_multi":
            ks = gen_gemm_multi(k, sym, idx, (tiles or {}).get(idx))
        elif k.kind == "matmul":
            parts = gen_matmul(k, sym, idx, (tiles or {}).get(idx))
            ws = max(ks.info.get("scratch_bytes", 0) for ks in parts)
            for ks in parts:
                ks.info["kind"] = k.kind
                ks.info["index"] = idx
                if ws:      # this matmul's own workspace region
                    ks.args = [("scratch", a[1] + ws_base) if a[0] == "scratch" else a for a in ks.args]
                    ks.info["scratch_base"] = ws_base
                    ks.info["scratch_bytes"] = ws_base + ws
                _forward_outputs(ks, k, fwd)
            ws_base += (ws + 255) // 256 * 256
            out += parts
            continue
        else:
            raise NotImplementedError(f"kernel kind {k.kind!r} is not supported by the b200 backend")
        ks.info["kind"] = k.kind
        ks.info["index"] = idx
        _forward_outputs(ks, k, fwd)
        out.append(ks)
    return out


def _forward_outputs(ks: KernelSource, k, fwd: dict) -> None:
    """Point the arguments of ``k``'s forwarded outputs at their hi copies in the workspace."""
    mine = {o.id for o in k.outputs if o.id in fwd}
    hit = sorted({a[1].id for a in ks.args if a[0] == "node" and a[1].id in mine})
    if hit:
        ks.args = [("scratch", fwd[a[1].id][0]) if a[0] == "node" and a[1].id in mine else a for a in ks.args]
        ks.info["forwarded_outputs"] = hit


__all__ = ["generate", "KernelSource"]
