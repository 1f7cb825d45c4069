"""Matmul kernels with the fused pointwise epilogue.

Plan semantics (``tensorjit/backends/cuda_backend.py:299-429``, C twin
``c_backend.py:186-304``): ``C[b,i,j] = sum_k A[b,i,k] * B[b,k,j]`` (``B[b,j,k]``
when ``trans_b``), batch dims broadcast with stride 0 (``cuda_backend.py:330-340``),
accumulate in f32, then evaluate every epilogue node per output element in f32
and store each escaping node in its dtype.

Implementations:

* ``tc``   bf16/f16 operands: the persistent tcgen05 kernel of
  ``csrc/kernels/gemm_sm100.cuh`` (TMA -> 128B-swizzled smem -> tcgen05.mma ->
  TMEM -> epilogue).  Needs K % 8 == 0 (16-byte TMA row pitch) and, for an
  N-major B, N % 8 == 0.
* ``tc`` in 3xTF32 mode for f32 operands with a K-major B and K % 4 == 0: one launch
  splits A and B into TF32 hi / lo copies, the same kernel issues hi*hi + hi*lo + lo*hi;
  a GEMM with too few output tiles is split over K (partial sums + a finalize launch).
* ``simt`` every other case (odd pitches, N-major f32 B, K == 0): a 64x64 tile,
  4x4 register micro-tile FFMA kernel with bounds checks, f32 accumulate.
"""
from __future__ import annotations

import os

from ..plan import PKernel, PNode, access_strides, contiguous_strides, first_consumer
from .common import (CTYPE, HEADER, ITEM, NUM_SMS, TMAP_DTYPE, KernelSource, TMapSpec, decompose_stmts, expr,
                     fast_math_for, offset_expr, params_struct, prod)


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


def tc_eligible(k: PKernel) -> bool:
    mm, a, b, tb, M, N, K, _ = _mm_dims(k)
    if os.environ.get("TENSORJIT_B200_NO_TCGEN05") == "1":
        return False
    if M == 0 or N == 0:
        return False
    if a.dtype == "f32" and b.dtype == "f32":
        return x3_eligible(k)
    if a.dtype not in ("bf16", "f16") or b.dtype != a.dtype:
        return False
    if K < 8 or K % 8 != 0:
        return False
    if not tb and N % 8 != 0:
        return False
    return True


def x3_eligible(k: PKernel) -> bool:
    """f32 operands on the tensor cores as 3xTF32: needs a K-major B (nn.Linear weights)
    and a 16-byte row pitch (K % 4 == 0)."""
    mm, a, b, tb, M, N, K, _ = _mm_dims(k)
    if os.environ.get("TENSORJIT_B200_NO_TF32X3") == "1":
        return False
    return a.dtype == b.dtype == "f32" and tb and K >= 4 and K % 4 == 0 and M > 0 and N > 0


def gen_split_tf32(symbol: str, segments: list[tuple]) -> KernelSource:
    """x -> (hi, lo) with hi = x with its 13 low mantissa bits cleared (exactly a TF32 value)
    and lo = x - hi (exact in f32): the operand split of 3xTF32 (hi*hi + hi*lo + lo*hi keeps
    ~21 mantissa bits of every product).  ``segments`` = [(numel, src, hi_off, lo_off), ...]:
    the operands of one GEMM are split by one grid-stride launch."""
    bounds, acc = [], 0
    for numel, _src, _hi, _lo in segments:
        acc += numel // 4
        bounds.append(acc)
    nseg = len(segments)
    L = [HEADER, params_struct(3 * nseg, 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{',
         f"  for (long g = (long)blockIdx.x * 256 + threadIdx.x; g < {acc}L; g += (long)gridDim.x * 256) {{",
         "    int s = 0;",
         "    long i = g;"]
    for j in range(nseg - 1):
        n = bounds[j] - (bounds[j - 1] if j else 0)
        L.append(f"    if (s == {j} && i >= {n}L) {{ i -= {n}L; s = {j + 1}; }}")

    def pick(slot: int) -> str:   # select the segment's pointer without indexing the params at run time
        e = f"prm.p[{3 * (nseg - 1) + slot}]"
        for j in range(nseg - 2, -1, -1):
            e = f"(s == {j} ? prm.p[{3 * j + slot}] : {e})"
        return e

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
          "  }",
          "}"]
    grid = max(1, min((acc + 255) // 256, NUM_SMS * 8))
    args = []
    for _numel, src, hi_off, lo_off in segments:
        args += [src, ("scratch", hi_off), ("scratch", lo_off)]
    total = sum(sg[0] for sg in segments)
    ks = KernelSource(symbol, "split", "\n".join(L), (grid, 1, 1), (256, 1, 1), args,
                      info={"bytes": total * 12, "numel": total})
    ks.finalize_params()
    return ks


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
    a_hi, a_lo = 0, _align(a.nbytes)
    b_hi = a_lo + _align(a.nbytes)
    b_lo = b_hi + _align(b.nbytes)
    part = b_lo + _align(b.nbytes)
    batch = prod(out_shape[:-2])
    BN, ksplit = x3_tile(M, N, K, batch, tile)
    tile = dict(tile or {"STAGES": 4, "GROUP_M": 16}, BN=BN)
    ws = part + (_align(ksplit * batch * M * N * 4) if ksplit > 1 else 0)
    sp = gen_split_tf32(f"{symbol}_split", [(a.numel, ("node", a), a_hi, a_lo), (b.numel, ("node", b), b_hi, b_lo)])
    g = gen_gemm_tc(k, symbol, kernel_id, tile, x3_scratch=(a_hi, b_hi, a_lo, b_lo),
                    ksplit=ksplit, partial_scratch=part)
    parts = [sp, g]
    if ksplit > 1:
        parts.append(gen_ksplit_finalize(k, f"{symbol}_finalize", g.args, ksplit))
    for ks in parts:
        ks.info["scratch_bytes"] = ws
    return parts


def gen_ksplit_finalize(k: PKernel, symbol: str, args: list, ksplit: int) -> KernelSource:
    """out = epilogue(sum over the K slices of the partial sums): the second half of a split-K
    GEMM.  Takes the GEMM launch's argument list, so operand indices are the same."""
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    epi = Epilogue(k, in_index, out_index)
    batch = prod(out_shape[:-2])
    total = batch * M * N
    part_idx = len(args) - 1
    L = [HEADER, params_struct(len(args), 0),
         f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{',
         f"  const float* __restrict__ part = (const float*)prm.p[{part_idx}];"]
    L += ["  " + x for x in epi._ptr_lines()]
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

    def __init__(self, k: PKernel, in_index: dict[int, int], out_index: dict[int, int]):
        self.k = k
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        self.mm, self.M, self.N, self.out_shape = mm, M, N, out_shape
        self.batch_shape = out_shape[:-2]
        self.epi_nodes = [n for n in k.nodes if n is not mm]
        self.epi_inputs = [n for n in k.inputs if n is not a and n is not b]
        self.in_index, self.out_index = in_index, out_index
        self.strides = {}
        for n in self.epi_inputs:
            c = first_consumer(n, self.epi_nodes, self.epi_nodes[0] if self.epi_nodes else mm)
            self.strides[n.id] = access_strides(n, c, out_shape)
        self.dtype_out = {o.id: o.dtype for o in k.outputs}
        self.fast = fast_math_for(self.dtype_out.values())

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
            val = {}
            for n in self.epi_inputs:
                st = self.strides[n.id]
                idx = self.in_index[n.id]
                off = self.offset(n, bidx, "i", "j")
                if st[-1] == 1:
                    if n.dtype == "f32":   # 8 f32 = two 16-byte loads
                        L.append(f"      float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id}); "
                                 f"tj_load_vec(in{idx} + ({off}) + 4, x{n.id} + 4);")
                    else:
                        L.append(f"      float x{n.id}[8]; tj_load_vec(in{idx} + ({off}), x{n.id});")
                    val[n.id] = f"x{n.id}[u]"
                else:
                    L.append(f"      const float x{n.id} = tj_f32(in{idx}[{off}]);")
                    val[n.id] = f"x{n.id}"
            outs = self.k.outputs
            for j, o in enumerate(outs):
                L.append(f"      float o{j}[8];")
            L.append("      #pragma unroll")
            L.append("      for (int u = 0; u < 8; ++u) {")
            comp, m = self.compute_lines("acc[c + u]", val)
            L += ["        " + s for s in comp]
            for j, o in enumerate(outs):
                L.append(f"        o{j}[u] = {m[o.id]};")
            L.append("      }")
            off = self.out_offset(bidx, "i", "j")
            for j, o in enumerate(outs):
                oi = self.out_index[o.id]
                if o.dtype == "f32":
                    L.append(f"      tj_store_vec(out{oi} + ({off}), o{j}); tj_store_vec(out{oi} + ({off}) + 4, o{j} + 4);")
                else:
                    L.append(f"      tj_store_vec(out{oi} + ({off}), o{j});")
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

    def tma_store_ok(self) -> bool:
        """One half-precision output written by 32 x 32 TMA stores: needs a 16-byte row
        pitch (N % 8 == 0) and the vectorised operand path."""
        outs = self.k.outputs
        return (len(outs) == 1 and outs[0].dtype in ("bf16", "f16") and self.N % 8 == 0 and self.vec_ok()
                and os.environ.get("TENSORJIT_B200_NO_TMA_STORE") != "1")

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
        for n in self.epi_inputs:
            idx = self.in_index[n.id]
            L.append(f"    const {CTYPE[n.dtype]}* __restrict__ in{idx} = (const {CTYPE[n.dtype]}*)prm.p[{idx}];")
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

    def _ptr_lines(self) -> list[str]:
        L = []
        for n in self.epi_inputs:
            idx = self.in_index[n.id]
            L.append(f"const {CTYPE[n.dtype]}* __restrict__ in{idx} = (const {CTYPE[n.dtype]}*)prm.p[{idx}];")
        for o in self.k.outputs:
            oi = self.out_index[o.id]
            L.append(f"{CTYPE[o.dtype]}* __restrict__ out{oi} = ({CTYPE[o.dtype]}*)prm.p[{oi}];")
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
            L.append(f"out{oi}[{off}] = tj_from<{CTYPE[o.dtype]}>({m[o.id]});")
        return L


# ---------------------------------------------------------------------------
# tcgen05 kernel
# ---------------------------------------------------------------------------
def partial_store_function(M: int, N: int, part_idx: int) -> str:
    """``epilogue(prm, b, i, j0, acc[32])`` of a split-K GEMM: the raw f32 accumulator row
    into partial-sum slice ``b`` (= slice * batch + batch index) of the workspace."""
    vec = N % 4 == 0
    L = ["  template <class P>",
         "  static __device__ __forceinline__ void epilogue(const P& prm, long b, long i, long j0, const float (&acc)[32]) {",
         f"    if (i >= {M}L) return;",
         f"    float* __restrict__ row = (float*)prm.p[{part_idx}] + (b * {M}L + i) * {N}L;",
         "    #pragma unroll",
         "    for (int c = 0; c < 32; c += 4) {",
         "      const long j = j0 + c;"]
    if vec:
        L += [f"      if (j >= {N}L) break;",
              "      *reinterpret_cast<float4*>(row + j) = make_float4(acc[c], acc[c + 1], acc[c + 2], acc[c + 3]);"]
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


def gen_gemm_tc(k: PKernel, symbol: str, kernel_id: int, tile: dict | None = None,
                x3_scratch: tuple | None = None, ksplit: int = 1, partial_scratch: int = 0) -> KernelSource:
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    batch_shape = out_shape[:-2]
    batch = prod(batch_shape)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    x3 = x3_scratch is not None
    # + status word (+ hi/lo operand copies) (+ the partial sums of a split-K GEMM)
    nptr = len(ins) + len(outs) + 1 + (4 if x3 else 0) + (1 if ksplit > 1 else 0)
    status_idx = len(ins) + len(outs)
    epi = Epilogue(k, in_index, out_index)
    b_mn = not tb
    if x3 and not tile:
        tile = {"BN": x3_tile(M, N, K, batch, None)[0], "STAGES": 4, "GROUP_M": 16}
    BN, STAGES, GROUP_M = choose_tile(M, N, batch, b_mn, tile)
    if x3:
        STAGES = min(STAGES, max(2, (200 * 1024) // (2 * (128 * 128 + BN * 128))))
    pair = bool(tile and tile.get("PAIR")) and tb and BN in (128, 256) and not x3
    a_bs = _batch_strides(a, batch_shape)
    b_bs = _batch_strides(b, batch_shape)
    a_mats = prod(a.shape[:-2])
    b_mats = prod(b.shape[:-2])
    bl, bidx = decompose_stmts("b", batch_shape, "bb") if batch_shape else ([], [])
    tma_store = epi.tma_store_ok() and not x3 and ksplit == 1
    L = [HEADER, '#include "gemm_sm100_pair.cuh"' if pair else '#include "gemm_sm100.cuh"',
         params_struct(nptr, 4 if x3 else (3 if tma_store else 2))]
    L.append("struct Cfg {")
    epi_warps = 8 if (BN % 64 == 0 or pair) else 4
    threads = 64 + 32 * epi_warps
    out_stage = epi_warps * 2 * 32 * 32 * 2 if tma_store else 0
    L.append(f"  static constexpr int BN = {BN}, STAGES = {STAGES}, M = {M}, N = {N}, K = {K}, GROUP_M = {GROUP_M};")
    L.append(f"  static constexpr int EPI_WARPS = {epi_warps}, KSPLIT = {ksplit}, NSEG = 1;")
    L.append("  static __device__ __forceinline__ int segment(int) { return 0; }")
    L.append("  static __device__ __forceinline__ int seg_tile0(int) { return 0; }")
    L.append(f"  static constexpr bool TF32X3 = {'true' if x3 else 'false'};")
    L.append(f"  static constexpr bool TMA_STORE = {'true' if tma_store else 'false'};")
    L.append(f"  using OutT = {CTYPE[outs[0].dtype] if tma_store else 'float'};")
    L.append(f"  static constexpr long BATCH = {batch}L;")
    L.append(f"  static constexpr bool BF16 = {'true' if a.dtype == 'bf16' else 'false'}, B_MN_MAJOR = {'true' if b_mn else 'false'};")
    L.append("  static __device__ __forceinline__ void batch_map(long b, long& ab, long& bb_) {")
    L += ["    " + s for s in bl]
    L.append(f"    ab = {offset_expr(bidx, a_bs) if batch_shape else '0L'};")
    L.append(f"    bb_ = {offset_expr(bidx, b_bs) if batch_shape else '0L'};")
    L.append("  }")
    if ksplit > 1:
        L.append(partial_store_function(M, N, nptr - 1))
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
    esz = ITEM[a.dtype]
    bk = 128 // esz                      # K elements per 128-byte swizzle row
    a_arg = in_index[a.id] if not x3 else status_idx + 1
    b_arg = in_index[b.id] if not x3 else status_idx + 2
    tmA = TMapSpec(arg=a_arg, dtype=a.dtype, dims=[K, a_mats * M], strides=[K * esz], box=[bk, 128], swizzle=3)
    if tb:
        tmB = TMapSpec(arg=b_arg, dtype=b.dtype, dims=[K, b_mats * N], strides=[K * esz],
                       box=[bk, BN // 2 if pair else BN], swizzle=3)
    else:
        tmB = TMapSpec(arg=in_index[b.id], dtype=b.dtype, dims=[N, K, b_mats], strides=[N * esz, K * N * esz],
                       box=[64, 64, 1], swizzle=3)
    tmaps = [tmA, tmB]
    if x3:
        tmaps.append(TMapSpec(arg=status_idx + 3, dtype="f32", dims=[K, a_mats * M], strides=[K * 4], box=[32, 128],
                              swizzle=3))
        tmaps.append(TMapSpec(arg=status_idx + 4, dtype="f32", dims=[K, b_mats * N], strides=[K * 4], box=[32, BN],
                              swizzle=3))
    if tma_store:
        o = outs[0]
        oe = ITEM[o.dtype]
        tmaps.append(TMapSpec(arg=out_index[o.id], dtype=o.dtype, dims=[N, M, batch], strides=[N * oe, M * N * oe],
                              box=[32, 32, 1], swizzle=2))
    args = [("node", n) for n in ins] + [("node", o) for o in outs] + [("status", None)]
    if x3:
        a_hi, b_hi, a_lo, b_lo = x3_scratch
        args += [("scratch", a_hi), ("scratch", b_hi), ("scratch", a_lo), ("scratch", b_lo)]
    if ksplit > 1:
        args.append(("scratch", partial_scratch))
    ks = KernelSource(symbol, "gemm_tc", "\n".join(L), (grid, 1, 1), (threads, 1, 1), args, smem=smem,
                      tmaps=tmaps, cluster=(2, 1, 1) if pair else (1, 1, 1),
                      info={"M": M, "N": N, "K": K, "batch": batch, "BN": BN, "stages": STAGES,
                            "tma_store": tma_store, "epi_warps": epi_warps, "pair": pair, "tf32x3": x3,
                            "ksplit": ksplit,
                            "flops": 2.0 * batch * M * N * K, "tiles": num_tiles,
                            "bytes": sum(n.nbytes for n in ins) + sum(o.nbytes for o in outs)})
    ks.finalize_params()
    return ks


# ---------------------------------------------------------------------------
# SIMT fallback
# ---------------------------------------------------------------------------
def gen_gemm_simt(k: PKernel, symbol: str) -> KernelSource:
    mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
    batch_shape = out_shape[:-2]
    batch = prod(batch_shape)
    ins, outs = list(k.inputs), list(k.outputs)
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_index = {o.id: len(ins) + j for j, o in enumerate(outs)}
    epi = Epilogue(k, in_index, out_index)
    a_bs = _batch_strides(a, batch_shape)
    b_bs = _batch_strides(b, batch_shape)
    ia, ib = in_index[a.id], in_index[b.id]
    BM_, BN_, BK_ = 64, 64, 16
    L = [HEADER, params_struct(len(ins) + len(outs), 0)]
    L.append(f'extern "C" __global__ void __launch_bounds__(256) {symbol}(const __grid_constant__ Params prm) {{')
    L.append(f"  const {CTYPE[a.dtype]}* __restrict__ A = (const {CTYPE[a.dtype]}*)prm.p[{ia}];")
    L.append(f"  const {CTYPE[b.dtype]}* __restrict__ B = (const {CTYPE[b.dtype]}*)prm.p[{ib}];")
    L += ["  " + s for s in epi._ptr_lines()]
    L.append("  const long bz = blockIdx.z;")
    bl, bidx = decompose_stmts("bz", batch_shape, "bb") if batch_shape else ([], [])
    L += ["  " + s for s in bl]
    L.append(f"  const long aoff = ({offset_expr(bidx, a_bs) if batch_shape else '0L'}) * {M * K}L;")
    L.append(f"  const long boff = ({offset_expr(bidx, b_bs) if batch_shape else '0L'}) * {N * K}L;")
    L.append(f"  __shared__ float As[{BK_}][{BM_} + 4];")
    L.append(f"  __shared__ float Bs[{BK_}][{BN_} + 4];")
    L.append(f"  const int tid = threadIdx.x, tr = tid / 16, tc = tid % 16;")
    L.append(f"  const long i0 = (long)blockIdx.y * {BM_}, j0 = (long)blockIdx.x * {BN_};")
    L.append("  float acc[4][4];")
    L.append("  #pragma unroll")
    L.append("  for (int x = 0; x < 4; ++x) for (int y = 0; y < 4; ++y) acc[x][y] = 0.0f;")
    L.append(f"  for (long k0 = 0; k0 < {K}L; k0 += {BK_}) {{")
    L.append(f"    for (int t = tid; t < {BM_ * BK_}; t += 256) {{")
    L.append(f"      const int r = t / {BK_}, c = t % {BK_};")
    L.append("      const long gi = i0 + r, gk = k0 + c;")
    L.append(f"      As[c][r] = (gi < {M}L && gk < {K}L) ? tj_f32(A[aoff + gi * {K}L + gk]) : 0.0f;")
    L.append("    }")
    L.append(f"    for (int t = tid; t < {BK_ * BN_}; t += 256) {{")
    if tb:
        L.append(f"      const int c = t / {BN_}, r = t % {BN_};")
        L.append("      const long gk = k0 + c, gj = j0 + r;")
        L.append(f"      Bs[c][r] = (gk < {K}L && gj < {N}L) ? tj_f32(B[boff + gj * {K}L + gk]) : 0.0f;")
    else:
        L.append(f"      const int r = t / {BN_}, c = t % {BN_};")
        L.append("      const long gk = k0 + r, gj = j0 + c;")
        L.append(f"      Bs[r][c] = (gk < {K}L && gj < {N}L) ? tj_f32(B[boff + gk * {N}L + gj]) : 0.0f;")
    L.append("    }")
    L.append("    __syncthreads();")
    L.append("    #pragma unroll")
    L.append(f"    for (int kk = 0; kk < {BK_}; ++kk) {{")
    L.append("      float av[4], bv[4];")
    L.append("      #pragma unroll")
    L.append("      for (int x = 0; x < 4; ++x) av[x] = As[kk][tr * 4 + x];")
    L.append("      #pragma unroll")
    L.append("      for (int y = 0; y < 4; ++y) bv[y] = Bs[kk][tc * 4 + y];")
    L.append("      #pragma unroll")
    L.append("      for (int x = 0; x < 4; ++x) for (int y = 0; y < 4; ++y) acc[x][y] = fmaf(av[x], bv[y], acc[x][y]);")
    L.append("    }")
    L.append("    __syncthreads();")
    L.append("  }")
    L.append("  #pragma unroll")
    L.append("  for (int x = 0; x < 4; ++x) {")
    L.append("    #pragma unroll")
    L.append("    for (int y = 0; y < 4; ++y) {")
    L.append("      const long i = i0 + tr * 4 + x, j = j0 + tc * 4 + y;")
    L.append(f"      if (i < {M}L && j < {N}L) {{")
    L += ["        " + s for s in epi.scalar_element_lines(bidx, "i", "j", "acc[x][y]")]
    L.append("      }")
    L.append("    }")
    L.append("  }")
    L.append("}")
    grid = ((N + BN_ - 1) // BN_, (M + BM_ - 1) // BM_, batch) if M and N and batch else (0, 1, 1)
    ks = KernelSource(symbol, "gemm_simt", "\n".join(L), grid, (256, 1, 1), [("node", n) for n in ins + outs],
                      info={"M": M, "N": N, "K": K, "batch": batch, "flops": 2.0 * batch * M * N * K,
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
    L.append(f"  static constexpr int EPI_WARPS = 8, KSPLIT = 1, NSEG = {len(parts)};")
    L.append("  static constexpr bool TF32X3 = false, TMA_STORE = false;")
    L.append("  using OutT = float;")
    L.append("  static constexpr long BATCH = 1L;")
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
        L.append(f"      {CTYPE[onode.dtype]}* __restrict__ dst = ({CTYPE[onode.dtype]}*)prm.p[{len(ins) + g}] + "
                 f"i * {ng}L + (j0 - {col0[g]}L);")
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
