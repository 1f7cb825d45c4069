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

from ..plan import PProgram
from .attention import gen_attention
from .common import KernelSource, checked_build, store_mode
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
    """Each matmul with a pre-pass gets a workspace region of its own (``info["scratch_base"]``,
    offsets relative to the program's workspace): its pre-pass may split or pack the program
    inputs among its operands before waiting for the kernels ahead of it (programmatic
    dependent launch), which is only safe when no earlier matmul still reads that region."""
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
            ws_base += (ws + 255) // 256 * 256
            out += parts
            continue
        else:
            raise NotImplementedError(f"kernel kind {k.kind!r} is not supported by the b200 backend")
        ks.info["kind"] = k.kind
        ks.info["index"] = idx
        out.append(ks)
    return out


__all__ = ["generate", "KernelSource"]
