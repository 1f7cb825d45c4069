"""Matmul kernels with the fused pointwise epilogue.

Plan semantics (``tensorjit/backends/cuda_backend.py:299-429``, C twin
``c_backend.py:186-304``): ``C[b,i,j] = sum_k A[b,i,k] * B[b,k,j]`` (``B[b,j,k]``
when ``trans_b``), batch dims broadcast with stride 0 (``cuda_backend.py:330-340``),
accumulate in f32, then evaluate every epilogue node per output element in f32
and store each escaping node in its dtype.

Every matmul with work runs on the persistent tcgen05 kernel of
``csrc/kernels/gemm_sm100.cuh`` (TMA -> 128B-swizzled smem -> tcgen05.mma -> TMEM ->
epilogue), in one of two operand forms (``gemm_form``):

* ``f16``  A and B both bf16 or both f16: kind::f16 MMAs.  The tensor maps read the
  operands in place when their rows have a 16-byte pitch (K % 8 == 0, and N % 8 == 0 for an
  N-major B); otherwise one pack launch first copies them into K-major buffers with a padded
  pitch in the program's workspace.
* ``x3``   anything else (f32, mixed or integer operands): 3xTF32, A_hi·B_hi + A_hi·B_lo +
  A_lo·B_hi with kind::tf32.  One launch splits both operands into TF32 hi / lo copies in the
  workspace (transposing an N-major B and padding K to a 16-byte pitch on the way); a GEMM
  with too few output tiles is split over K (partial sums + a finalize launch).

A matmul with K == 0 or no output element is its epilogue over a zero accumulator (one
grid-stride launch, or none).
"""
from __future__ import annotations

import os

from ..plan import PKernel, PNode, access_strides, contiguous_strides, first_consumer
from .common import (PDL, BOUNDS_SITE, CTYPE, HEADER, ITEM, NUM_SMS, KernelSource, TMapSpec, checked,
                     decompose_stmts, expr, fast_math_for, offset_expr, params_struct, prod, ptr_decl, split_out,
                     split_skip, split_store_lines, status_decl, tma_store_allowed)


def _mm_dims(k: PKernel):
    mm = k.anchor
    a, b = mm.inputs
    tb = bool(mm.attrs.get("trans_b"))
    M, K = a.shape[-2], a.shape[-1]
    N = b.shape[-2] if tb else b.shape[-1]
    out_shape = tuple(mm.shape)
    return mm, a, b, tb, M, N, K, out_shape


def _batch_strides(t: PNode, batch_shape: tuple) -> tuple:
    """Per-batch-dim stride of operand ``t`` in units of whole matrices (0 = broadcast)."""
    mshape = t.shape[:-2]
    cs = contiguous_strides(mshape) if mshape else ()
    pad = len(batch_shape) - len(mshape)
    st = [0] * pad
    for d in range(len(mshape)):
        st.append(0 if mshape[d] == 1 and batch_shape[pad + d] != 1 else cs[d])
    return tuple(st)


class GemmForm:
    """How a plan matmul maps onto the tcgen05 kernel.

    ``mode``   "f16" (kind::f16 on bf16/f16 operands), "x3" (3xTF32) or "empty" (K == 0 or
               no output element: epilogue only).
    ``pack_a`` / ``pack_b``  the operand is first copied into the workspace (K-major, row pitch
               ``pitch`` elements); for "x3" both are always split into hi / lo copies.
    ``b_mn``   the kernel reads B N-major (an unpacked B of a plan matmul without ``trans_b``).
    """

    def __init__(self, mode: str, pack_a: bool, pack_b: bool, pitch: int, b_mn: bool):
        self.mode, self.pack_a, self.pack_b, self.pitch, self.b_mn = mode, pack_a, pack_b, pitch, b_mn

    def __repr__(self):
        return f"GemmForm({self.mode}, pack_a={self.pack_a}, pack_b={self.pack_b}, pitch={self.pitch}, b_mn={self.b_mn})"


def gemm_form(k: PKernel) -> GemmForm:
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    if K == 0 or M == 0 or N == 0 or prod(out_shape[:-2]) == 0:
        return GemmForm("empty", False, False, 0, False)
    if a.dtype in ("bf16", "f16") and b.dtype == a.dtype:
        pitch = (K + 7) // 8 * 8
        pack_a = K % 8 != 0
        pack_b = K % 8 != 0 or (not tb and N % 8 != 0)
        return GemmForm("f16", pack_a, pack_b, pitch, not tb and not pack_b)
    return GemmForm("x3", True, True, (K + 3) // 4 * 4, False)


def tc_eligible(k: PKernel) -> bool:
    """The matmul runs the tcgen05 GEMM (every matmul with work does)."""
    return gemm_form(k).mode != "empty"


def x3_eligible(k: PKernel) -> bool:
    """The matmul runs as 3xTF32 (f32, mixed or integer operands)."""
    return gemm_form(k).mode == "x3"


def gen_pack_operands(symbol: str, segments: list[dict], kernel_id: int = 0) -> KernelSource:
    """Copy GEMM operands into K-major buffers with a 16-byte row pitch in the workspace, for
    the cases the tensor maps cannot read in place: a K that breaks the 16-byte row pitch, an
    N-major B whose N does, and every operand of a 3xTF32 GEMM that is not an f32 K-major
    matrix with K % 4 == 0.  One launch packs all operands of a GEMM.  A CTA moves a 32 x 32
    tile (32 rows x 32 of K) through shared memory, so an N-major source is read along its rows
    and the K-major destination is written along K, both in 128-byte lines.  Columns K up to
    the pitch are written as zeros, so the kernel's k-blocks past K add nothing.

    ``segments``: dicts with ``src`` (argument ref), ``src_dtype``, ``mats`` (matrices),
    ``rows`` (M for A, N for B), ``K``, ``pitch``, ``k_major`` (source rows run along K),
    ``split`` (write TF32 hi / lo pairs: hi = the value with its 13 low mantissa bits cleared,
    lo = value - hi, both exact in f32), ``dst_dtype`` and the workspace offsets ``hi`` / ``lo``
    (``lo`` unused without ``split``)."""
    tiles = []
    for sg in segments:
        kt = (sg["pitch"] + 31) // 32
        rt = (sg["rows"] + 31) // 32
        tiles.append(sg["mats"] * rt * kt)
    total = sum(tiles)
    chk = checked()
    nptr = 3 * len(segments) + (1 if chk else 0)
    # program inputs (weights) are packed before the launch waits for the previous kernel
    early, late = _early_late([sg["src"] for sg in segments])
    prologue, loops, epilogue = _wait_split(early, late)
    L = [HEADER, params_struct(nptr, 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{',
         prologue]
    if chk:
        L.append("  " + status_decl(3 * len(segments)))
    for j, sg in enumerate(segments):
        n_src = sg["mats"] * sg["rows"] * sg["K"]
        n_dst = sg["mats"] * sg["rows"] * sg["pitch"]
        dt = "float" if sg["split"] else CTYPE[sg["dst_dtype"]]
        L.append("  " + ptr_decl(f"src{j}", CTYPE[sg["src_dtype"]], 3 * j, n_src, True, kernel_id))
        L.append("  " + ptr_decl(f"hi{j}", dt, 3 * j + 1, n_dst, False, kernel_id))
        if sg["split"]:
            L.append("  " + ptr_decl(f"lo{j}", dt, 3 * j + 2, n_dst, False, kernel_id))
    L += ["  __shared__ float tile[32][33];",
          "  const int tx = threadIdx.x & 31, ty = threadIdx.x >> 5;"]
    for idx, pre in loops:
        if pre:
            L.append(pre)
        L += _pack_loop(segments, tiles, idx)
    if epilogue:
        L.append(epilogue)
    L.append("}")
    args = []
    nbytes = 0
    for sg in segments:
        args += [sg["src"], ("scratch", sg["hi"]), ("scratch", sg.get("lo", sg["hi"]))]
    if chk:
        args.append(("status", None))
    for sg in segments:
        n_src = sg["mats"] * sg["rows"] * sg["K"]
        n_dst = sg["mats"] * sg["rows"] * sg["pitch"]
        nbytes += n_src * ITEM[sg["src_dtype"]] + n_dst * ITEM[sg["dst_dtype"]] * (2 if sg["split"] else 1)
    grid = max(1, min(total, NUM_SMS * 8))
    ks = KernelSource(symbol, "split", "\n".join(L), (grid, 1, 1), (256, 1, 1), args,
                      info={"bytes": nbytes, "numel": sum(sg["mats"] * sg["rows"] * sg["K"] for sg in segments),
                            "early_segments": len(early)})
    ks.finalize_params()
    return ks


def _pack_loop(segments: list[dict], tiles: list[int], idx: list[int]) -> list[str]:
    """Tile loop (one 32 x 32 tile per CTA iteration) over the segments ``idx``."""
    total = sum(tiles[j] for j in idx)
    L = [f"  for (long t = blockIdx.x; t < {total}L; t += gridDim.x) {{",
         "    long u = t;"]
    acc = 0
    for q, j in enumerate(idx):
        sg, nt = segments[j], tiles[j]
        R, K, P = sg["rows"], sg["K"], sg["pitch"]
        kt = (P + 31) // 32
        rt = (R + 31) // 32
        dt = CTYPE[sg["dst_dtype"]]
        cond = f"u < {acc + nt}L" if q < len(idx) - 1 else "true"
        L.append(f"    {'if' if q == 0 else 'else if'} ({cond}) {{")
        L.append(f"      u -= {acc}L;")
        L.append(f"      const long kt = u % {kt}L, rt = (u / {kt}L) % {rt}L, mat = u / {kt * rt}L;")
        L.append("      for (int y = ty; y < 32; y += 8) {")
        g = sg.get("gather")
        if sg["k_major"]:
            off = _gather_offset(g, "mat", "r", "kk") if g else f"mat * {R * K}L + r * {K}L + kk"
            L.append("        const long r = rt * 32 + y, kk = kt * 32 + tx;")
            L.append(f"        tile[y][tx] = (r < {R}L && kk < {K}L) ? tj_f32(src{j}[{off}]) : 0.0f;")
        else:   # source [K, rows]: consecutive threads read consecutive rows
            off = _gather_offset(g, "mat", "r", "kk") if g else f"mat * {R * K}L + kk * {R}L + r"
            L.append("        const long kk = kt * 32 + y, r = rt * 32 + tx;")
            L.append(f"        tile[tx][y] = (r < {R}L && kk < {K}L) ? tj_f32(src{j}[{off}]) : 0.0f;")
        L.append("      }")
        L.append("      __syncthreads();")
        L.append("      for (int y = ty; y < 32; y += 8) {")
        L.append("        const long r = rt * 32 + y, kk = kt * 32 + tx;")
        L.append(f"        if (r < {R}L && kk < {P}L) {{")
        L.append("          const float v = tile[y][tx];")
        L.append(f"          const long o = (mat * {R}L + r) * {P}L + kk;")
        if sg["split"]:
            L.append("          const float h = __uint_as_float(__float_as_uint(v) & 0xffffe000u);")
            L.append(f"          hi{j}[o] = h;")
            L.append(f"          lo{j}[o] = v - h;")
        else:
            L.append(f"          hi{j}[o] = tj_from<{dt}>(v);")
        L.append("        }")
        L.append("      }")
        L.append("      __syncthreads();")
        L.append("    }")
        acc += nt
    L.append("  }")
    return L


def gen_epilogue_only(k: PKernel, symbol: str, kernel_id: int = 0) -> KernelSource:
    """A matmul whose every dot product is empty (K == 0), or which has no output element: the
    epilogue over a zero accumulator as one grid-stride launch (none when nothing is stored)."""
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    chk = checked()
    epi = Epilogue(k, in_index, out_index, kernel_id, len(ins) + len(outs))
    total = prod(out_shape[:-2]) * M * N
    L = [HEADER, params_struct(len(ins) + len(outs) + (1 if chk else 0), 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{', PDL]
    L += ["  " + x for x in epi._ptr_lines()]
    L.append(f"  for (long e = (long)blockIdx.x * 256 + threadIdx.x; e < {total}L; e += (long)gridDim.x * 256) {{")
    L.append(f"    const long j = e % {max(N, 1)}L, row = e / {max(N, 1)}L, i = row % {max(M, 1)}L, "
             f"b = row / {max(M, 1)}L;")
    bl, bidx = epi.batch_index_lines("b")
    L += ["    " + x for x in bl]
    L += ["    " + x for x in epi.scalar_element_lines(bidx, "i", "j", "0.0f")]
    L += ["  }", "}"]
    grid = min((total + 255) // 256, NUM_SMS * 8) if total else 0
    ks = KernelSource(symbol, "ewise", "\n".join(L), (grid, 1, 1), (256, 1, 1),
                      [("node", n) for n in ins] + [("node", o) for o in outs] + ([("status", None)] if chk else []),
                      info={"bytes": sum(n.nbytes for n in k.inputs if n is not a and n is not b)
                            + sum(o.nbytes for o in outs), "numel": total, "flops": 0.0})
    ks.finalize_params()
    return ks


def _operand_segment(node: PNode, rows: int, K: int, pitch: int, k_major: bool, split: bool, dst_dtype: str,
                     hi: int, lo: int, gather: dict | None = None) -> dict:
    """``gather``: the operand is read from a folded transpose's source (``fuse.py``): its
    {"src", "k", "r", "b"} sub-dims give each element's offset there."""
    src = gather["src"] if gather else node
    return {"src": ("node", src), "src_dtype": node.dtype, "mats": prod(node.shape[:-2]), "rows": rows, "K": K,
            "pitch": pitch, "k_major": k_major, "split": split, "dst_dtype": dst_dtype, "hi": hi, "lo": lo,
            "gather": gather}


def _gather_offset(g: dict, mat: str, r: str, kk: str) -> str:
    """Offset in a folded transpose's source of operand element (mat, r, kk): each index split
    over its sub-dims (innermost first, mixed radix) times their strides."""
    terms = []
    for var, dims in ((kk, g["k"]), (r, g["r"]), (mat, g["b"])):
        div = 1
        for q, (size, stride) in enumerate(dims):
            v = var if div == 1 else f"({var} / {div}L)"
            if q < len(dims) - 1:
                v = f"({v} % {size}L)"
            terms.append(v if stride == 1 else f"{v} * {stride}L")
            div *= size
    return " + ".join(terms) if terms else "0L"


def gen_matmul(k: PKernel, symbol: str, kernel_id: int, tile: dict | None) -> list[KernelSource]:
    """The launches of one plan matmul: [pack or split pre-pass], tcgen05 GEMM, [split-K
    finalize]; or the epilogue alone when there is nothing to multiply."""
    form = gemm_form(k)
    if form.mode == "empty":
        return [gen_epilogue_only(k, symbol, kernel_id)]
    if form.mode == "x3":
        return gen_matmul_tc_x3(k, symbol, kernel_id, tile)
    if not (form.pack_a or form.pack_b):
        return [gen_gemm_tc(k, symbol, kernel_id, tile)]
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    P = form.pitch
    a_off = 0
    b_off = _align(prod(a.shape[:-2]) * M * P * ITEM[a.dtype]) if form.pack_a else 0
    ws = b_off + (_align(prod(b.shape[:-2]) * N * P * ITEM[b.dtype]) if form.pack_b else 0)
    segs = []
    if form.pack_a:
        segs.append(_operand_segment(a, M, K, P, True, False, a.dtype, a_off, a_off, k.attrs.get("a_gather")))
    if form.pack_b:
        segs.append(_operand_segment(b, N, K, P, tb, False, b.dtype, b_off, b_off, k.attrs.get("b_gather")))
    pk = gen_pack_operands(f"{symbol}_pack", segs, kernel_id)
    g = gen_gemm_tc(k, symbol, kernel_id, tile, packed={"a": a_off if form.pack_a else None,
                                                        "b": b_off if form.pack_b else None, "pitch": P})
    for ks in (pk, g):
        ks.info["scratch_bytes"] = ws
    return [pk, g]


def _is_program_input(ref) -> bool:
    """An argument that is a program input: no kernel of the program writes it, so a launch may
    read it before waiting for the previous kernel (programmatic dependent launch)."""
    return ref[0] == "node" and ref[1].op == "input"


def _early_late(srcs: list) -> tuple[list[int], list[int]]:
    """Segment indices split into (program inputs, the rest)."""
    early = [j for j, src in enumerate(srcs) if _is_program_input(src)]
    return early, [j for j in range(len(srcs)) if j not in early]


def _wait_split(early: list, late: list) -> tuple[str, list, str]:
    """(prologue, [(segments, preamble)], ...) of a pre-pass whose program-input segments run
    before ``tj_pdl_wait()``: those read only caller inputs and write this matmul's own
    workspace region, which nothing before it touches."""
    if early and late:
        return "  tj_pdl_launch_dependents();", [(early, ""), (late, "  tj_pdl_wait();")], ""
    if early:
        return "  tj_pdl_launch_dependents();", [(early, "")], "  tj_pdl_wait();"
    return PDL, [(late, "")], ""


def gen_split_tf32(symbol: str, segments: list[tuple], kernel_id: int = 0) -> KernelSource:
    """x -> (hi, lo) with hi = x with its 13 low mantissa bits cleared (exactly a TF32 value)
    and lo = x - hi (exact in f32): the operand split of 3xTF32 (hi*hi + hi*lo + lo*hi keeps
    ~21 mantissa bits of every product).  ``segments`` = [(numel, src, hi_off, lo_off), ...]:
    the operands of one GEMM are split by one grid-stride launch.  Segments that are program
    inputs (weights) are split first, before the launch waits for the previous kernel, so with
    programmatic dependent launch that part overlaps the kernels before it."""
    nseg = len(segments)
    chk = checked()
    early, late = _early_late([sg[1] for sg in segments])
    prologue, loops, epilogue = _wait_split(early, late)
    L = [HEADER, params_struct(3 * nseg + (1 if chk else 0), 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{',
         prologue]
    if chk:
        L.append("  " + status_decl(3 * nseg))
    for segs, pre in loops:
        if pre:
            L.append(pre)
        L += _split_loop(segments, segs, kernel_id, chk)
    if epilogue:
        L.append(epilogue)
    L.append("}")
    total4 = sum(sg[0] // 4 for sg in segments)
    grid = max(1, min((total4 + 255) // 256, NUM_SMS * 8))
    args = []
    for _numel, src, hi_off, lo_off in segments:
        args += [src, ("scratch", hi_off), ("scratch", lo_off)]
    if chk:
        args.append(("status", None))
    total = sum(sg[0] for sg in segments)
    ks = KernelSource(symbol, "split", "\n".join(L), (grid, 1, 1), (256, 1, 1), args,
                      info={"bytes": total * 12, "numel": total, "early_segments": len(early)})
    ks.finalize_params()
    return ks


def _split_loop(segments: list[tuple], idx: list[int], kernel_id: int, chk: bool) -> list[str]:
    """Grid-stride loop splitting the float4s of segments ``idx`` (argument slots 3j..3j+2)."""
    n4 = [segments[j][0] // 4 for j in idx]
    acc = sum(n4)
    L = [f"  for (long g = (long)blockIdx.x * 256 + threadIdx.x; g < {acc}L; g += (long)gridDim.x * 256) {{",
         "    int s = 0;",
         "    long i = g;"]
    for q in range(len(idx) - 1):
        L.append(f"    if (s == {q} && i >= {n4[q]}L) {{ i -= {n4[q]}L; s = {q + 1}; }}")

    def pick(slot: int) -> str:   # select the segment's pointer without indexing the params at run time
        e = f"prm.p[{3 * idx[-1] + slot}]"
        for q in range(len(idx) - 2, -1, -1):
            e = f"(s == {q} ? prm.p[{3 * idx[q] + slot}] : {e})"
        return e

    if chk:   # the segment's index stays inside its operand (in float4 units)
        lim = f"{n4[-1]}L"
        for q in range(len(idx) - 2, -1, -1):
            lim = f"(s == {q} ? {n4[q]}L : {lim})"
        arg = f"3 * {idx[0]}" if len(idx) == 1 else "3 * (" + "".join(
            f"s == {q} ? {idx[q]} : " for q in range(len(idx) - 1)) + f"{idx[-1]})"
        L.append(f"    if (!tj_check(i >= 0 && i < {lim}, tj_status, {kernel_id * 16 + BOUNDS_SITE}, {arg}, i)) "
                 "continue;")
    L += [f"    const float4* __restrict__ x = (const float4*){pick(0)};",
          f"    float4* __restrict__ hi = (float4*){pick(1)};",
          f"    float4* __restrict__ lo = (float4*){pick(2)};",
          "    const float4 v = __ldg(x + i);",
          "    float4 h;",
          "    h.x = __uint_as_float(__float_as_uint(v.x) & 0xffffe000u);",
          "    h.y = __uint_as_float(__float_as_uint(v.y) & 0xffffe000u);",
          "    h.z = __uint_as_float(__float_as_uint(v.z) & 0xffffe000u);",
          "    h.w = __uint_as_float(__float_as_uint(v.w) & 0xffffe000u);",
          "    hi[i] = h;",
          "    lo[i] = make_float4(v.x - h.x, v.y - h.y, v.z - h.z, v.w - h.w);",
          "  }"]
    return L


def _align(x: int, a: int = 256) -> int:
    return (x + a - 1) // a * a


def x3_ksplit(M: int, N: int, K: int, batch: int, BN: int) -> int:
    """K slices for a 3xTF32 GEMM with too few output tiles to fill the GPU: as many as keep
    every CTA on its own SM, each slice at least 8 k-blocks (256 of K), at most 8."""
    tiles = batch * ((M + 127) // 128) * ((N + BN - 1) // BN)
    k_blocks = (K + 31) // 32
    ks = min(8, NUM_SMS // max(tiles, 1), k_blocks // 8)
    if ks < 2:
        return 1
    kpb = (k_blocks + ks - 1) // ks
    return (k_blocks + kpb - 1) // kpb   # no empty slice


def x3_tile(M: int, N: int, K: int, batch: int, tile: dict | None) -> tuple[int, int]:
    """(BN, K slices) of a 3xTF32 GEMM.  Its k-blocks are bound by shared-memory traffic (hi and
    lo copies of a 128-row A tile and a BN-row B tile), so the cost of a choice is waves x
    k-blocks per CTA x bytes per k-block, plus a fixed cost for the finalize launch of a split
    (about 8 us, the time of 500 KB of k-block traffic)."""
    if tile and tile.get("BN"):
        return tile["BN"], x3_ksplit(M, N, K, batch, tile["BN"])
    k_blocks = (K + 31) // 32
    best = None
    for bn in (64, 128):
        ks = x3_ksplit(M, N, K, batch, bn)
        ctas = batch * ((M + 127) // 128) * ((N + bn - 1) // bn) * ks
        waves = (ctas + NUM_SMS - 1) // NUM_SMS
        cost = waves * ((k_blocks + ks - 1) // ks) * (2 * (128 + bn) * 128 // 1024) + (500 if ks > 1 else 0)
        if best is None or cost < best[0]:
            best = (cost, bn, ks)
    return best[1], best[2]


def gen_matmul_tc_x3(k: PKernel, symbol: str, kernel_id: int, tile: dict | None) -> list[KernelSource]:
    """f32 matmul as [split(A and B), 3xTF32 tcgen05 GEMM]; the hi/lo copies live in the
    program's workspace (arena space after the planned intermediates).  With few output tiles
    the GEMM is split over K into partial sums in the workspace and a finalize launch adds
    them and applies the epilogue."""
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    P = (K + 3) // 4 * 4
    a_bytes = prod(a.shape[:-2]) * M * P * 4
    b_bytes = prod(b.shape[:-2]) * N * P * 4
    a_hi, a_lo = 0, _align(a_bytes)
    b_hi = a_lo + _align(a_bytes)
    b_lo = b_hi + _align(b_bytes)
    part = b_lo + _align(b_bytes)
    batch = prod(out_shape[:-2])
    BN, ksplit = x3_tile(M, N, K, batch, tile)
    tile = dict(tile or {"STAGES": 4, "GROUP_M": 16}, BN=BN)
    ws = part + (_align(ksplit * batch * M * N * 4) if ksplit > 1 else 0)
    ga, gb = k.attrs.get("a_gather"), k.attrs.get("b_gather")      # folded transposes (fuse.py)
    vec_split = a.dtype == b.dtype == "f32" and tb and K % 4 == 0 and not ga and not gb
    skip = split_skip(kernel_id) if vec_split else set()
    if vec_split:
        # both operands already K-major f32 with a 16-byte pitch: the vectorised split, minus the
        # operands whose producer writes the hi / lo copies itself (3xTF32 operand forwarding)
        segs = [seg for role, seg in (("a", (a.numel, ("node", a), a_hi, a_lo)),
                                      ("b", (b.numel, ("node", b), b_hi, b_lo))) if role not in skip]
        sp = gen_split_tf32(f"{symbol}_split", segs, kernel_id) if segs else None
    else:
        sp = gen_pack_operands(f"{symbol}_split", [_operand_segment(a, M, K, P, True, True, "f32", a_hi, a_lo, ga),
                                                   _operand_segment(b, N, K, P, tb, True, "f32", b_hi, b_lo, gb)],
                               kernel_id)
    g = gen_gemm_tc(k, symbol, kernel_id, tile, x3_scratch=(a_hi, b_hi, a_lo, b_lo),
                    ksplit=ksplit, partial_scratch=part)
    if vec_split:
        # where each operand's hi / lo copies are (workspace offsets), for operand forwarding
        g.info["x3_vec"] = {"a": (a.id, a_hi, a_lo), "b": (b.id, b_hi, b_lo)}
        g.info["x3_forwarded"] = sorted(skip)
    parts = [sp, g] if sp is not None else [g]
    if ksplit > 1:
        parts.append(gen_ksplit_finalize(k, f"{symbol}_finalize", g.args, ksplit, kernel_id))
    for ks in parts:
        ks.info["scratch_bytes"] = ws
    return parts


def gen_ksplit_finalize(k: PKernel, symbol: str, args: list, ksplit: int, kernel_id: int = 0) -> KernelSource:
    """out = epilogue(sum over the K slices of the partial sums): the second half of a split-K
    GEMM.  Takes the GEMM launch's argument list, so operand indices are the same."""
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    epi = Epilogue(k, in_index, out_index, kernel_id, len(ins) + len(outs))   # the GEMM's status argument
    batch = prod(out_shape[:-2])
    total = batch * M * N
    part_idx = len(args) - 1
    L = [HEADER, params_struct(len(args), 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{', PDL]
    L += ["  " + x for x in epi._ptr_lines()]
    L.append("  " + ptr_decl("part", "float", part_idx, ksplit * total, True, kernel_id))
    if epi.vec_ok():
        # 8 consecutive columns per thread: two 16-byte loads per K slice, the GEMM's 8-wide epilogue
        groups = total // 8
        L.append(f"  for (long g = (long)blockIdx.x * 256 + threadIdx.x; g < {groups}L; g += (long)gridDim.x * 256) {{")
        L.append(f"    const long row = g / {N // 8}L, j = (g - row * {N // 8}L) * 8, i = row % {M}L, b = row / {M}L;")
        L.append("    float s8[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};")
        L.append("    #pragma unroll")
        L.append(f"    for (int s = 0; s < {ksplit}; ++s) {{")
        L.append("      float p8[8];")
        L.append(f"      tj_load_vec(part + (s * {total}L + row * {N}L + j), p8);")
        L.append(f"      tj_load_vec(part + (s * {total}L + row * {N}L + j) + 4, p8 + 4);")
        L.append("      #pragma unroll")
        L.append("      for (int u = 0; u < 8; ++u) s8[u] += p8[u];")
        L.append("    }")
        bl, bidx = epi.batch_index_lines("b")
        L += ["    " + x for x in bl]
        L += ["    " + x for x in epi.vec8_lines(bidx, "s8[u]")]
        L.append("  }")
        L.append("}")
        grid = max(1, min((groups + 255) // 256, NUM_SMS * 8))
        ks = KernelSource(symbol, "ewise", "\n".join(L), (grid, 1, 1), (256, 1, 1), list(args),
                          info={"bytes": total * 4 * (ksplit + 1), "numel": total, "ksplit": ksplit, "vec": 8})
        ks.finalize_params()
        return ks
    L.append(f"  for (long e = (long)blockIdx.x * 256 + threadIdx.x; e < {total}L; e += (long)gridDim.x * 256) {{")
    L.append(f"    const long j = e % {N}L, row = e / {N}L, i = row % {M}L, b = row / {M}L;")
    L.append("    float acc = 0.0f;")
    L.append("    #pragma unroll")
    L.append(f"    for (int s = 0; s < {ksplit}; ++s) acc += part[s * {total}L + e];")
    bl, bidx = epi.batch_index_lines("b")
    L += ["    " + x for x in bl]
    L += ["    " + x for x in epi.scalar_element_lines(bidx, "i", "j", "acc")]
    L.append("  }")
    L.append("}")
    grid = max(1, min((total + 255) // 256, NUM_SMS * 8))
    ks = KernelSource(symbol, "ewise", "\n".join(L), (grid, 1, 1), (256, 1, 1), list(args),
                      info={"bytes": total * 4 * (ksplit + 1), "numel": total, "ksplit": ksplit})
    ks.finalize_params()
    return ks


# ---------------------------------------------------------------------------
# epilogue generator (shared by both GEMM implementations)
# ---------------------------------------------------------------------------
class Epilogue:
    """Emits the per-element epilogue of a matmul kernel: load epilogue inputs at
    (batch, i, j), evaluate the DAG, store every escaping node."""

    def __init__(self, k: PKernel, in_index: dict[int, int], out_index: dict[int, int], kernel_id: int = 0,
                 status_idx: int | None = None):
        self.k = k
        self.kernel_id, self.status_idx = kernel_id, status_idx
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        self.mm, self.M, self.N, self.out_shape = mm, M, N, out_shape
        self.batch_shape = out_shape[:-2]
        self.epi_nodes = [n for n in k.nodes if n is not mm]
        # operands read from a folded transpose's source
        srcs = [(k.attrs.get(f) or {}).get("src") for f in ("a_strided", "b_strided", "a_gather", "b_gather")]
        self.epi_inputs = [n for n in k.inputs if n is not a and n is not b and all(n is not x for x in srcs)]
        self.in_index, self.out_index = in_index, out_index
        self.strides = {}
        for n in self.epi_inputs:
            c = first_consumer(n, self.epi_nodes, self.epi_nodes[0] if self.epi_nodes else mm)
            self.strides[n.id] = access_strides(n, c, out_shape)
        self.dtype_out = {o.id: o.dtype for o in k.outputs}
        self.fast = fast_math_for(self.dtype_out.values())
        self.fwd = {o.id: split_out()[o.id] for o in k.outputs if o.id in split_out()}   # hi -> lo distance

    def vec_ok(self) -> bool:
        """8-column vector path: every epilogue operand unit-stride or broadcast along j,
        every other stride and N a multiple of 8, no i32."""
        if self.N % 8 != 0:
            return False
        for n in self.epi_inputs:
            st = self.strides[n.id]
            if st[-1] not in (0, 1) or any(s % 8 != 0 for s in st[:-1]) or n.dtype == "i32":
                return False
        return all(d in ("bf16", "f16", "f32") for d in self.dtype_out.values())

    def batch_index_lines(self, bvar: str) -> tuple[list[str], list[str]]:
        if not self.batch_shape:
            return [], []
        return decompose_stmts(bvar, self.batch_shape, "eb")

    def offset(self, n: PNode, bidx: list[str], ivar: str, jvar: str) -> str:
        return offset_expr(bidx + [ivar, jvar], self.strides[n.id])

    def out_offset(self, bidx: list[str], ivar: str, jvar: str) -> str:
        return offset_expr(bidx + [ivar, jvar], contiguous_strides(self.out_shape))

    def compute_lines(self, acc: str, val: dict[int, str]) -> tuple[list[str], dict[int, str]]:
        """f32 evaluation of the DAG given the accumulator and loaded operands."""
        m = dict(val)
        m[self.mm.id] = acc
        lines = []
        for n in self.epi_nodes:
            lines.append(f"const float e{n.id} = {expr(n, m, self.fast)};")
            m[n.id] = f"e{n.id}"
        return lines, m

    def chunk32_function(self) -> str:
        """``epilogue(prm, b, i, j0, acc[32])`` for the tcgen05 kernel (one row, 32 columns)."""
        L = ["  template <class P>",
             "  static __device__ __forceinline__ void epilogue(const P& prm, long b, long i, long j0, const float (&acc)[32]) {",
             f"    if (i >= {self.M}L) return;"]
        L += ["    " + s for s in self._ptr_lines()]
        bl, bidx = self.batch_index_lines("b")
        L += ["    " + s for s in bl]
        if self.vec_ok():
            L.append("    #pragma unroll")
            L.append("    for (int c = 0; c < 32; c += 8) {")
            L.append("      const long j = j0 + c;")
            L.append(f"      if (j >= {self.N}L) break;")
            L += ["      " + x for x in self.vec8_lines(bidx, "acc[c + u]")]
            L.append("    }")
        else:
            L.append("    #pragma unroll 4")
            L.append("    for (int c = 0; c < 32; ++c) {")
            L.append("      const long j = j0 + c;")
            L.append(f"      if (j >= {self.N}L) break;")
            L += ["      " + s for s in self.scalar_element_lines(bidx, "i", "j", "acc[c]")]
            L.append("    }")
        L.append("  }")
        return "\n".join(L)

    def vec8_lines(self, bidx: list[str], acc: str) -> list[str]:
        """Epilogue of the 8 columns j..j+7 of row i (vector path): load the operands, evaluate
        the DAG on the accumulator values ``acc`` (an expression of ``u``), store the outputs."""
        L, val = [], {}
        for n in self.epi_inputs:
            st = self.strides[n.id]
            idx = self.in_index[n.id]
            off = self.offset(n, bidx, "i", "j")
            if st[-1] == 1:
                if n.dtype == "f32":   # 8 f32 = two 16-byte loads
                    L.append(f"float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id}); "
                             f"tj_load_vec(in{idx} + ({off}) + 4, x{n.id} + 4);")
                else:
                    L.append(f"float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id});")
                val[n.id] = f"x{n.id}[u]"
            else:
                L.append(f"const float x{n.id} = tj_f32(in{idx}[{off}]);")
                val[n.id] = f"x{n.id}"
        outs = self.k.outputs
        for j, o in enumerate(outs):
            L.append(f"float o{j}[8];")
        L.append("#pragma unroll")
        L.append("for (int u = 0; u < 8; ++u) {")
        comp, m = self.compute_lines(acc, val)
        L += ["  " + s for s in comp]
        for j, o in enumerate(outs):
            L.append(f"  o{j}[u] = {m[o.id]};")
        L.append("}")
        off = self.out_offset(bidx, "i", "j")
        for j, o in enumerate(outs):
            oi = self.out_index[o.id]
            if o.id in self.fwd:
                L += split_store_lines(f"out{oi}", off, f"o{j}", 8, self.fwd[o.id])
            elif o.dtype == "f32":
                L.append(f"tj_store_vec(out{oi} + ({off}), o{j}); tj_store_vec(out{oi} + ({off}) + 4, o{j} + 4);")
            else:
                L.append(f"tj_store_vec(out{oi} + ({off}), o{j});")
        return L

    def tma_store_ok(self) -> bool:
        """One half-precision output written by 32 x 32 TMA stores: needs a 16-byte row
        pitch (N % 8 == 0) and the vectorised operand path."""
        outs = self.k.outputs
        return (len(outs) == 1 and outs[0].dtype in ("bf16", "f16") and self.N % 8 == 0 and self.vec_ok()
                and os.environ.get("TENSORJIT_B200_NO_TMA_STORE") != "1" and tma_store_allowed())

    def staged_store_ok(self) -> bool:
        """The staged plain-store path (outputs that may be a peer GPU's memory): the same
        output forms as the TMA-store path."""
        outs = self.k.outputs
        return len(outs) == 1 and outs[0].dtype in ("bf16", "f16") and self.N % 8 == 0 and self.vec_ok()

    def stage_last_ok(self) -> bool:
        """The last-tile staged path for one f32 output (16-byte pieces of 4 columns; the
        vector operand path of ``epilogue_vals``)."""
        outs = self.k.outputs
        return len(outs) == 1 and outs[0].dtype == "f32" and self.N % 8 == 0 and self.vec_ok() and not self.fwd

    def store4_function(self) -> str:
        """``store4(prm, b, i, j, v)``: 4 f32 output values at (batch b, row i, columns j..j+3),
        nothing outside the output (the last-tile staged path)."""
        o = self.k.outputs[0]
        oi = self.out_index[o.id]
        L = ["  template <class P>",
             "  static __device__ __forceinline__ void store4(const P& prm, long b, long i, long j, const float4& v) {",
             f"    if (i >= {self.M}L || j >= {self.N}L) return;"]
        L += ["    " + x for x in self._status_lines()]
        L.append("    " + ptr_decl(f"out{oi}", "float", oi, o.numel, False, self.kernel_id))
        bl, bidx = self.batch_index_lines("b")
        L += ["    " + x for x in bl]
        L.append(f"    tj_st16(out{oi} + ({self.out_offset(bidx, 'i', 'j')}), make_uint4(__float_as_uint(v.x), "
                 "__float_as_uint(v.y), __float_as_uint(v.z), __float_as_uint(v.w)));")
        L.append("  }")
        return "\n".join(L)

    def store16_function(self) -> str:
        """``store16(prm, b, i, j, v)``: 8 packed output elements at (batch b, row i, column j),
        nothing outside the output (the staged store path)."""
        o = self.k.outputs[0]
        oi = self.out_index[o.id]
        L = ["  template <class P>",
             "  static __device__ __forceinline__ void store16(const P& prm, long b, long i, long j, const uint4& v) {",
             f"    if (i >= {self.M}L || j >= {self.N}L) return;"]
        L += ["    " + x for x in self._status_lines()]
        L.append("    " + ptr_decl(f"out{oi}", CTYPE[o.dtype], oi, o.numel, False, self.kernel_id))
        bl, bidx = self.batch_index_lines("b")
        L += ["    " + x for x in bl]
        L.append(f"    tj_st16(out{oi} + ({self.out_offset(bidx, 'i', 'j')}), v);")
        L.append("  }")
        return "\n".join(L)

    def vals32_function(self) -> str:
        """``epilogue_vals(prm, b, i, j0, acc[32], out[32])``: the output values of one row's 32
        columns (rows >= M and columns >= N are left at 0; the TMA store clips them)."""
        o = self.k.outputs[0]
        L = ["  template <class P>",
             "  static __device__ __forceinline__ void epilogue_vals(const P& prm, long b, long i, long j0, "
             "const float (&acc)[32], float (&out)[32]) {",
             "    #pragma unroll",
             "    for (int c = 0; c < 32; ++c) out[c] = 0.0f;",
             f"    if (i >= {self.M}L) return;"]
        L += ["    " + x for x in self._status_lines() + self._in_lines()]
        bl, bidx = self.batch_index_lines("b")
        L += ["    " + s for s in bl]
        L.append("    #pragma unroll")
        L.append("    for (int c = 0; c < 32; c += 8) {")
        L.append("      const long j = j0 + c;")
        L.append(f"      if (j >= {self.N}L) break;")
        val = {}
        for n in self.epi_inputs:
            st = self.strides[n.id]
            idx = self.in_index[n.id]
            off = self.offset(n, bidx, "i", "j")
            if st[-1] == 1:
                if n.dtype == "f32":
                    L.append(f"      float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id}); "
                             f"tj_load_vec(in{idx} + ({off}) + 4, x{n.id} + 4);")
                else:
                    L.append(f"      float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id});")
                val[n.id] = f"x{n.id}[u]"
            else:
                L.append(f"      const float x{n.id} = tj_f32(in{idx}[{off}]);")
                val[n.id] = f"x{n.id}"
        L.append("      #pragma unroll")
        L.append("      for (int u = 0; u < 8; ++u) {")
        comp, m = self.compute_lines("acc[c + u]", val)
        L += ["        " + s for s in comp]
        L.append(f"        out[c + u] = {m[o.id]};")
        L.append("      }")
        L.append("    }")
        L.append("  }")
        return "\n".join(L)

    def _status_lines(self) -> list[str]:
        return [status_decl(self.status_idx)] if checked() else []

    def _in_lines(self) -> list[str]:
        return [ptr_decl(f"in{self.in_index[n.id]}", CTYPE[n.dtype], self.in_index[n.id], n.numel, True, self.kernel_id)
                for n in self.epi_inputs]

    def _ptr_lines(self) -> list[str]:
        L = self._status_lines() + self._in_lines()
        for o in self.k.outputs:
            oi = self.out_index[o.id]
            L.append(ptr_decl(f"out{oi}", CTYPE[o.dtype], oi, o.numel + self.fwd.get(o.id, 0), False,
                              self.kernel_id))
        return L

    def scalar_element_lines(self, bidx: list[str], ivar: str, jvar: str, acc: str) -> list[str]:
        L = []
        val = {}
        for n in self.epi_inputs:
            idx = self.in_index[n.id]
            L.append(f"const float x{n.id} = tj_f32(in{idx}[{self.offset(n, bidx, ivar, jvar)}]);")
            val[n.id] = f"x{n.id}"
        comp, m = self.compute_lines(acc, val)
        L += comp
        off = self.out_offset(bidx, ivar, jvar)
        for o in self.k.outputs:
            oi = self.out_index[o.id]
            if o.id in self.fwd:
                L.append(f"const float so{o.id}[1] = {{{m[o.id]}}};")
                L += split_store_lines(f"out{oi}", off, f"so{o.id}", 1, self.fwd[o.id])
            else:
                L.append(f"out{oi}[{off}] = tj_from<{CTYPE[o.dtype]}>({m[o.id]});")
        return L


# ---------------------------------------------------------------------------
# tcgen05 kernel
# ---------------------------------------------------------------------------
def partial_stage_functions(M: int, N: int, part_idx: int, numel: int = 0, kernel_id: int = 0,
                            status_idx: int = 0) -> str:
    """``epilogue_vals`` (the raw accumulator) and ``store4`` (into partial-sum slice b) of a
    split-K GEMM, for the last-tile staged path (N % 4 == 0)."""
    return "\n".join([
        "  template <class P>",
        "  static __device__ __forceinline__ void epilogue_vals(const P&, long, long, long, const float (&acc)[32], "
        "float (&out)[32]) {",
        "    #pragma unroll",
        "    for (int c = 0; c < 32; ++c) out[c] = acc[c];",
        "  }",
        "  template <class P>",
        "  static __device__ __forceinline__ void store4(const P& prm, long b, long i, long j, const float4& v) {",
        f"    if (i >= {M}L || j >= {N}L) return;",
        *(["    " + status_decl(status_idx)] if checked() else []),
        "    " + ptr_decl("part", "float", part_idx, numel, False, kernel_id),
        f"    tj_st16(part + ((b * {M}L + i) * {N}L + j), make_uint4(__float_as_uint(v.x), __float_as_uint(v.y), "
        "__float_as_uint(v.z), __float_as_uint(v.w)));",
        "  }"])


def partial_store_function(M: int, N: int, part_idx: int, numel: int = 0, kernel_id: int = 0,
                           status_idx: int = 0) -> str:
    """``epilogue(prm, b, i, j0, acc[32])`` of a split-K GEMM: the raw f32 accumulator row
    into partial-sum slice ``b`` (= slice * batch + batch index) of the workspace."""
    vec = N % 4 == 0
    L = ["  template <class P>",
         "  static __device__ __forceinline__ void epilogue(const P& prm, long b, long i, long j0, const float (&acc)[32]) {",
         f"    if (i >= {M}L) return;",
         *(["    " + status_decl(status_idx)] if checked() else []),
         "    " + ptr_decl("part", "float", part_idx, numel, False, kernel_id),
         f"    const auto row = part + (b * {M}L + i) * {N}L;",
         "    #pragma unroll",
         "    for (int c = 0; c < 32; c += 4) {",
         "      const long j = j0 + c;"]
    if vec:
        L += [f"      if (j >= {N}L) break;",
              "      tj_store_vec(row + j, &acc[c]);"]
    else:
        L += ["      #pragma unroll",
              f"      for (int u = 0; u < 4; ++u) if (j + u < {N}L) row[j + u] = acc[c + u];"]
    L += ["    }", "  }"]
    return "\n".join(L)


def choose_tile(M: int, N: int, batch: int, b_mn_major: bool, override: dict | None = None) -> tuple[int, int, int]:
    """(BN, STAGES, GROUP_M): largest N tile that still gives every SM work."""
    if override:
        return override["BN"], override["STAGES"], override.get("GROUP_M", 16)
    m_tiles = (M + 127) // 128
    cands = [256, 128, 64] if not b_mn_major else [256, 128, 64]
    BN = 64
    for bn in cands:
        if N < bn and bn > 64 and N <= bn // 2:
            continue
        tiles = batch * m_tiles * ((N + bn - 1) // bn)
        if tiles >= NUM_SMS or bn == 64:
            BN = bn
            break
    if N <= 32 and not b_mn_major:
        BN = 32
    stage_bytes = 128 * 64 * 2 + BN * 64 * 2
    STAGES = max(2, min(8, (200 * 1024) // stage_bytes))
    return BN, STAGES, 16


def _operand_map_order(sd: dict) -> tuple[list[str], list[int]]:
    """Roles of a folded-transpose operand's dims (K0 [K1] R0 [R1] [B0 [B1]], as
    ``fuse.strided_operand_layout`` lists them; R = rows, M for A, N for B) and the order of those
    dims in the tensor map: sorted by stride, as the attention kernel's maps are, so the map's
    strides never decrease.  Only K0 (unit stride, always first) and R0 have box extents above
    1, so a tile lands in shared memory as rows of one 64-element k-block (for an N-major B, R0
    is unit-stride and first: 64 x 64 chunks as the N-major path loads them)."""
    k_roles, r_roles = ["k0", "k1"][: sd["k_dims"]], ["r0", "r1"][: sd["r_dims"]]
    roles = (r_roles + k_roles if sd.get("n_major") else k_roles + r_roles) + ["b0", "b1"][: sd["batch_dims"]]
    order = sorted(range(len(roles)), key=lambda i: sd["dims"][i][1])
    return roles, order


def _operand_coords_function(sd: dict, name: str, rvar: str, bvar: str) -> list[str]:
    """``<name>(batch, r0, k0, c)``: tensor-map coordinates of the operand tile at row r0 (of M
    for A, N for B), column k0 of operand matrix ``batch`` when the operand is read from a folded
    transpose's source.  Two batch dims split the batch index (inner dim first)."""
    dims = sd["dims"]
    roles, order = _operand_map_order(sd)
    size = {r: dims[i][0] for i, r in enumerate(roles)}
    value = {"k0": f"k0 % {size['k0']}" if "k1" in roles else "k0", "k1": f"k0 / {size['k0']}",
             "r0": f"{rvar} % {size['r0']}" if "r1" in roles else rvar, "r1": f"{rvar} / {size['r0']}",
             "b0": f"static_cast<int>({bvar} % {size['b0']}L)" if "b1" in roles else f"static_cast<int>({bvar})",
             "b1": f"static_cast<int>({bvar} / {size.get('b0', 1)}L)"}
    L = [f"  static __device__ __forceinline__ void {name}(long {bvar}, int {rvar}, int k0, int (&c)[5]) {{"]
    if "b0" not in roles:
        L.append(f"    (void){bvar};")
    for pos, i in enumerate(order):
        L.append(f"    c[{pos}] = {value[roles[i]]};")
    L.append("  }")
    return L


def gen_gemm_tc(k: PKernel, symbol: str, kernel_id: int, tile: dict | None = None,
                x3_scratch: tuple | None = None, ksplit: int = 1, partial_scratch: int = 0,
                packed: dict | None = None) -> KernelSource:
    """The tcgen05 GEMM launch of one plan matmul.  ``x3_scratch`` = workspace offsets of the
    (A hi, B hi, A lo, B lo) copies of a 3xTF32 GEMM; ``packed`` = {"a": offset | None, "b":
    offset | None, "pitch": P} for bf16/f16 operands the pack pre-pass copied into the workspace
    (K-major, row pitch P elements), which the tensor maps then read instead of the plan's."""
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    batch_shape = out_shape[:-2]
    batch = prod(batch_shape)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    x3 = x3_scratch is not None
    pk_a = packed is not None and packed.get("a") is not None
    pk_b = packed is not None and packed.get("b") is not None
    # + status word (+ hi/lo operand copies) (+ packed operands) (+ the partial sums of a split-K GEMM)
    nptr = len(ins) + len(outs) + 1 + (4 if x3 else 0) + int(pk_a) + int(pk_b) + (1 if ksplit > 1 else 0)
    status_idx = len(ins) + len(outs)
    epi = Epilogue(k, in_index, out_index, kernel_id, status_idx)
    # B is read N-major only in place from a plan matmul without trans_b; the workspace copies
    # (3xTF32 hi / lo, packed operands) are always K-major
    b_mn = not (tb or pk_b or x3)
    if x3 and not tile:
        tile = {"BN": x3_tile(M, N, K, batch, None)[0], "STAGES": 4, "GROUP_M": 16}
    BN, STAGES, GROUP_M = choose_tile(M, N, batch, b_mn, tile)
    if x3:
        STAGES = min(STAGES, max(2, (200 * 1024) // (2 * (128 * 128 + BN * 128))))
    sa = k.attrs.get("a_strided")       # A read from a folded transpose's source (fuse.py)
    sb = k.attrs.get("b_strided")       # K-major B read from a folded transpose's source
    assert not sa or not (x3 or pk_a), "a folded transpose needs the plain 16-bit A path"
    assert not sb or not (x3 or pk_b or b_mn != bool(sb.get("n_major"))), "a folded B needs the plain 16-bit path"
    pair = (bool(tile and tile.get("PAIR")) and not b_mn and BN in (128, 256) and not x3 and not sa
            and not sb)
    if tile and tile.get("PAIR") and not pair:
        # a CTA-pair tile run on one CTA (e.g. A read from a folded transpose): each stage then
        # holds the whole B tile, so keep only as many stages as fit beside the epilogue staging
        per_stage = (2 if x3 else 1) * (128 * 128 + BN * 128)
        STAGES = min(STAGES, max(2, (232448 - 1024 - 8 * 2 * 32 * 32 * 2 - 512) // per_stage))
    a_bs = _batch_strides(a, batch_shape)
    b_bs = _batch_strides(b, batch_shape)
    a_mats = prod(a.shape[:-2])
    b_mats = prod(b.shape[:-2])
    bl, bidx = decompose_stmts("b", batch_shape, "bb") if batch_shape else ([], [])
    tma_store = epi.tma_store_ok() and not x3 and ksplit == 1
    # outputs that may be a peer GPU's memory: staged in shared memory like the TMA-store path,
    # then written with plain coalesced 16-byte stores (whole row segments per instruction)
    staged = not tma_store and not tma_store_allowed() and epi.staged_store_ok() and not x3 and ksplit == 1
    # split-K partial sums: the CTA's last tile staged in the idle pipeline memory and written as
    # whole row segments (single-CTA kernel).  TENSORJIT_B200_STAGE_LAST=all also stages f32
    # outputs with an epilogue; measured slower there (cfg1's GELU GEMM: 25.4 -> 29.1 us), the
    # partial sums faster (cfg1's second GEMM: 20.5 -> 18.5 us).
    mode = os.environ.get("TENSORJIT_B200_STAGE_LAST", "1")
    stage_last = (not tma_store and not staged and not pair and tma_store_allowed() and mode != "0"
                  and (N % 4 == 0 if ksplit > 1 else (mode == "all" and epi.stage_last_ok())))
    L = [HEADER, '#include "gemm_sm100_pair.cuh"' if pair else '#include "gemm_sm100.cuh"',
         params_struct(nptr, 4 if x3 else (3 if tma_store else 2))]
    L.append("struct Cfg {")
    epi_warps = 8 if (BN % 64 == 0 or pair) else 4
    threads = 64 + 32 * epi_warps
    out_stage = epi_warps * 2 * 32 * 32 * 2 if (tma_store or staged) else 0
    GROUP_N = int((tile or {}).get("GROUP_N", 0))
    L.append(f"  static constexpr int BN = {BN}, STAGES = {STAGES}, M = {M}, N = {N}, K = {K}, GROUP_M = {GROUP_M};")
    L.append(f"  static constexpr int GROUP_N = {GROUP_N};")
    L.append(f"  static constexpr int EPI_WARPS = {epi_warps}, KSPLIT = {ksplit}, NSEG = 1;")
    L.append("  static __device__ __forceinline__ int segment(int) { return 0; }")
    L.append("  static __device__ __forceinline__ int seg_tile0(int) { return 0; }")
    L.append(f"  static constexpr bool TF32X3 = {'true' if x3 else 'false'};")
    L.append(f"  static constexpr bool TMA_STORE = {'true' if tma_store else 'false'};")
    L.append(f"  static constexpr bool STAGED_STORE = {'true' if staged else 'false'};")
    L.append(f"  static constexpr bool STAGE_LAST = {'true' if stage_last else 'false'};")
    L.append(f"  static constexpr int A_RANK = {len(sa['dims']) if sa else 2};")
    L.append(f"  static constexpr int B_RANK = {len(sb['dims']) if sb else (3 if b_mn else 2)};")
    L.append(f"  static constexpr bool B_FOLDED = {'true' if sb else 'false'};")
    if sa:
        L += _operand_coords_function(sa, "a_coords", "m0", "ab")
    if sb:
        L += _operand_coords_function(sb, "b_coords", "n0", "bb")
    L.append(f"  using OutT = {CTYPE[outs[0].dtype] if (tma_store or staged) else 'float'};")
    L.append(f"  static constexpr long BATCH = {batch}L, A_MATS = {a_mats}L, B_MATS = {b_mats}L;")
    L.append(f"  static constexpr bool BF16 = {'true' if a.dtype == 'bf16' else 'false'}, B_MN_MAJOR = {'true' if b_mn else 'false'};")
    L.append("  static __device__ __forceinline__ void batch_map(long b, long& ab, long& bb_) {")
    L += ["    " + s for s in bl]
    L.append(f"    ab = {offset_expr(bidx, a_bs) if batch_shape else '0L'};")
    L.append(f"    bb_ = {offset_expr(bidx, b_bs) if batch_shape else '0L'};")
    L.append("  }")
    if ksplit > 1:
        L.append(partial_store_function(M, N, nptr - 1, ksplit * batch * M * N, kernel_id, status_idx))
        if stage_last:
            L.append(partial_stage_functions(M, N, nptr - 1, ksplit * batch * M * N, kernel_id, status_idx))
    elif stage_last:
        L.append(epi.chunk32_function())
        L.append(epi.vals32_function())
        L.append(epi.store4_function())
    elif staged:
        L.append(epi.vals32_function())
        L.append(epi.store16_function())
    else:
        L.append(epi.vals32_function() if tma_store else epi.chunk32_function())
    L.append("};")
    b_rows = BN // 2 if pair else BN
    smem = 1024 + STAGES * (2 if x3 else 1) * (128 * 128 + b_rows * 128) + out_stage + (2 * STAGES + 6) * 8 + 16
    if smem > 232448:
        raise ValueError(f"tile BN={BN} STAGES={STAGES} pair={pair} needs {smem} B of shared memory")
    L.append(f'extern "C" __global__ void __launch_bounds__({threads}, 1) {symbol}(const __grid_constant__ Params prm) {{')
    fn = "gemm_sm100_pair" if pair else "gemm_sm100"
    L.append(f"  tjg::{fn}<Cfg>(prm, (int*)prm.p[{status_idx}], {kernel_id});")
    L.append("}")
    m_tiles = (M + (255 if pair else 127)) // (256 if pair else 128)
    n_tiles = (N + BN - 1) // BN
    num_tiles = batch * m_tiles * n_tiles * ksplit
    grid = 2 * min(num_tiles, NUM_SMS // 2) if pair else min(num_tiles, NUM_SMS)
    op_dt = "f32" if x3 else a.dtype
    esz = ITEM[op_dt]
    bk = 128 // esz                      # K elements per 128-byte swizzle row
    # row pitch (elements) of each operand as the tensor maps read it
    pitch = (K + 3) // 4 * 4 if x3 else (packed["pitch"] if (pk_a or pk_b) else K)
    a_pitch = pitch if (x3 or pk_a) else K
    b_pitch = pitch if (x3 or pk_b) else K
    pk_arg = status_idx + 1
    a_arg = status_idx + 1 if x3 else (pk_arg if pk_a else in_index[(sa["src"] if sa else a).id])
    b_arg = status_idx + 2 if x3 else (pk_arg + int(pk_a) if pk_b else in_index[(sb["src"] if sb else b).id])
    if sa:
        roles, order = _operand_map_order(sa)
        box = [bk if roles[i] == "k0" else (128 if roles[i] == "r0" else 1) for i in order]
        tmA = TMapSpec(arg=a_arg, dtype=op_dt, dims=[sa["dims"][i][0] for i in order],
                       strides=[sa["dims"][i][1] * esz for i in order[1:]], box=box, swizzle=3)
    else:
        tmA = TMapSpec(arg=a_arg, dtype=op_dt, dims=[K, a_mats * M], strides=[a_pitch * esz], box=[bk, 128],
                       swizzle=3)
    if sb:
        roles, order = _operand_map_order(sb)
        if sb.get("n_major"):   # 64-column x 64-k chunks, as the N-major path loads them
            box = [64 if roles[i] in ("r0", "k0") else 1 for i in order]
        else:
            box = [bk if roles[i] == "k0" else (BN if roles[i] == "r0" else 1) for i in order]
        tmB = TMapSpec(arg=b_arg, dtype=op_dt, dims=[sb["dims"][i][0] for i in order],
                       strides=[sb["dims"][i][1] * esz for i in order[1:]], box=box, swizzle=3)
    elif not b_mn:
        tmB = TMapSpec(arg=b_arg, dtype=op_dt, dims=[K, b_mats * N], strides=[b_pitch * esz],
                       box=[bk, BN // 2 if pair else BN], swizzle=3)
    else:
        tmB = TMapSpec(arg=b_arg, dtype=op_dt, dims=[N, K, b_mats], strides=[N * esz, K * N * esz],
                       box=[64, 64, 1], swizzle=3)
    tmaps = [tmA, tmB]
    if x3:
        tmaps.append(TMapSpec(arg=status_idx + 3, dtype="f32", dims=[K, a_mats * M], strides=[pitch * 4],
                              box=[32, 128], swizzle=3))
        tmaps.append(TMapSpec(arg=status_idx + 4, dtype="f32", dims=[K, b_mats * N], strides=[pitch * 4],
                              box=[32, BN], swizzle=3))
    if tma_store:
        o = outs[0]
        oe = ITEM[o.dtype]
        tmaps.append(TMapSpec(arg=out_index[o.id], dtype=o.dtype, dims=[N, M, batch], strides=[N * oe, M * N * oe],
                              box=[32, 32, 1], swizzle=2))
    args = [("node", n) for n in ins] + [("node", o) for o in outs] + [("status", None)]
    if x3:
        a_hi, b_hi, a_lo, b_lo = x3_scratch
        args += [("scratch", a_hi), ("scratch", b_hi), ("scratch", a_lo), ("scratch", b_lo)]
    if pk_a:
        args.append(("scratch", packed["a"]))
    if pk_b:
        args.append(("scratch", packed["b"]))
    if ksplit > 1:
        args.append(("scratch", partial_scratch))
    ks = KernelSource(symbol, "gemm_tc", "\n".join(L), (grid, 1, 1), (threads, 1, 1), args, smem=smem,
                      tmaps=tmaps, cluster=(2, 1, 1) if pair else (1, 1, 1),
                      info={"M": M, "N": N, "K": K, "batch": batch, "BN": BN, "stages": STAGES,
                            "tma_store": tma_store, "staged_store": staged, "stage_last": stage_last,
                            "a_strided": bool(sa), "b_strided": bool(sb),
                            "epi_warps": epi_warps, "pair": pair,
                            "tf32x3": x3,
                            "ksplit": ksplit, "packed": [x for x, f in (("a", pk_a), ("b", pk_b)) if f],
                            "flops": 2.0 * batch * M * N * K, "tiles": num_tiles,
                            "bytes": sum(n.nbytes for n in ins) + sum(o.nbytes for o in outs)})
    ks.finalize_params()
    return ks


# ---------------------------------------------------------------------------
# several GEMMs sharing A (kind "matmul_multi", built by fuse.py)
# ---------------------------------------------------------------------------
def gen_gemm_multi(k: PKernel, symbol: str, kernel_id: int, tile: dict | None = None) -> KernelSource:
    """C_g = A · B_gᵀ for g = 0..G-1 as one tcgen05 GEMM over the concatenated N: the column
    tiles of segment g read B_g through its own tensor map and store to C_g, so the A tiles
    are read once for all G products and the GPU sees one launch with G times the tiles."""
    parts = k.attrs["parts"]             # [(B node, output node, N)]
    a = k.attrs["a"]
    dt = a.dtype
    M, K = a.shape
    BN = 256
    # CTA pair (256 x 256 tiles, each CTA loading half of every B tile) unless the tile says
    # otherwise or there is less than one 256-row tile
    pair = bool((tile or {}).get("PAIR", os.environ.get("TENSORJIT_B200_PAIR") != "0")) and M >= 256
    STAGES = (tile or {}).get("STAGES", 6 if pair else 4)
    GROUP_M = (tile or {}).get("GROUP_M", 16)
    ins = [a] + [p_[0] for p_ in parts]
    outs = [p_[1] for p_ in parts]
    N = sum(p_[2] for p_ in parts)
    status_idx = len(ins) + len(outs)
    seg_tiles = [p_[2] // BN for p_ in parts]
    starts = [sum(seg_tiles[:g]) for g in range(len(parts))]
    col0 = [sum(p_[2] for p_ in parts[:g]) for g in range(len(parts))]
    L = [HEADER, '#include "gemm_sm100_pair.cuh"' if pair else '#include "gemm_sm100.cuh"',
         params_struct(status_idx + 1, 1 + len(parts))]
    L.append("struct Cfg {")
    L.append(f"  static constexpr int BN = {BN}, STAGES = {STAGES}, M = {M}, N = {N}, K = {K}, GROUP_M = {GROUP_M};")
    L.append(f"  static constexpr int GROUP_N = {int((tile or {}).get('GROUP_N', 0))};")
    L.append(f"  static constexpr int EPI_WARPS = 8, KSPLIT = 1, NSEG = {len(parts)};")
    L.append("  static constexpr bool TF32X3 = false, TMA_STORE = false, STAGED_STORE = false, STAGE_LAST = false;")
    L.append("  static constexpr int A_RANK = 2, B_RANK = 2;")
    L.append("  static constexpr bool B_FOLDED = false;")
    L.append("  using OutT = float;")
    L.append("  static constexpr long BATCH = 1L, A_MATS = 1L, B_MATS = 1L;")
    L.append(f"  static constexpr bool BF16 = {'true' if dt == 'bf16' else 'false'}, B_MN_MAJOR = false;")
    L.append("  static __device__ __forceinline__ void batch_map(long, long& ab, long& bb_) { ab = 0; bb_ = 0; }")
    seg = " : ".join(f"nt < {starts[g] + seg_tiles[g]} ? {g}" for g in range(len(parts) - 1)) + f" : {len(parts) - 1}"
    L.append(f"  static __device__ __forceinline__ int segment(int nt) {{ return {seg}; }}")
    st0 = " : ".join(f"g == {g} ? {starts[g]}" for g in range(len(parts) - 1)) + f" : {starts[-1]}"
    L.append(f"  static __device__ __forceinline__ int seg_tile0(int g) {{ return {st0}; }}")
    L.append("  template <class P>")
    L.append("  static __device__ __forceinline__ void epilogue(const P& prm, long, long i, long j0, const float (&acc)[32]) {")
    L.append(f"    if (i >= {M}L) return;")
    for g, (bnode, onode, ng) in enumerate(parts):
        if g == len(parts) - 1:
            L.append("    else {")
        else:
            L.append(f"    {'if' if g == 0 else 'else if'} (j0 < {col0[g] + ng}L) {{")
        if checked():
            L.append("      " + status_decl(status_idx))
        L.append("      " + ptr_decl("outg", CTYPE[onode.dtype], len(ins) + g, onode.numel, False, kernel_id))
        L.append(f"      const auto dst = outg + (i * {ng}L + (j0 - {col0[g]}L));")
        L.append("      #pragma unroll")
        L.append("      for (int c = 0; c < 32; c += 8) tj_store_vec(dst + c, acc + c);")
        L.append("    }")
    L.append("  }")
    L.append("};")
    b_rows = BN // 2 if pair else BN
    smem = 1024 + STAGES * (128 * 128 + b_rows * 128) + (2 * STAGES + 6) * 8 + 16
    if smem > 232448:
        raise ValueError(f"shared-A GEMM STAGES={STAGES} pair={pair} needs {smem} B of shared memory")
    L.append(f'extern "C" __global__ void __launch_bounds__(320, 1) {symbol}(const __grid_constant__ Params prm) {{')
    L.append(f"  tjg::{'gemm_sm100_pair' if pair else 'gemm_sm100'}<Cfg>(prm, (int*)prm.p[{status_idx}], {kernel_id});")
    L.append("}")
    esz = ITEM[dt]
    tmaps = [TMapSpec(arg=0, dtype=dt, dims=[K, M], strides=[K * esz], box=[128 // esz, 128], swizzle=3)]
    for g, (bnode, _o, ng) in enumerate(parts):
        tmaps.append(TMapSpec(arg=1 + g, dtype=dt, dims=[K, ng], strides=[K * esz], box=[128 // esz, b_rows],
                              swizzle=3))
    num_tiles = ((M + (255 if pair else 127)) // (256 if pair else 128)) * (N // BN)
    grid = 2 * min(num_tiles, NUM_SMS // 2) if pair else min(num_tiles, NUM_SMS)
    args = [("node", n) for n in ins] + [("node", o) for o in outs] + [("status", None)]
    ks = KernelSource(symbol, "gemm_tc", "\n".join(L), (grid, 1, 1), (320, 1, 1), args, smem=smem,
                      tmaps=tmaps, cluster=(2, 1, 1) if pair else (1, 1, 1),
                      info={"M": M, "N": N, "K": K, "batch": 1, "BN": BN, "stages": STAGES, "tma_store": False,
                            "epi_warps": 8, "pair": pair, "tf32x3": False, "ksplit": 1, "segments": len(parts),
                            "flops": 2.0 * M * N * K, "tiles": num_tiles,
                            "bytes": sum(n.nbytes for n in ins) + sum(o.nbytes for o in outs)})
    ks.finalize_params()
    return ks
