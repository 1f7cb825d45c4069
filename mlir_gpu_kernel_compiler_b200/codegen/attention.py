"""Code generation for ``attention`` kernels (the fused chain built by ``fuse.py``).

The generated translation unit binds the shapes, the softmax scale and the
operand addressing (including folded transposes) as compile-time constants of a
``Cfg`` struct and instantiates ``tja::attention_sm100`` from
``csrc/kernels/attention_sm100.cuh``.

Addressing: every operand is read through a TMA tensor map whose dimensions are
the operand's non-trivial logical dims ordered by memory stride (the head
dimension first, stride 1).  The box is 64 elements of the head dimension by 128
rows of the sequence dimension and 1 of every batch dimension, so whatever the
memory layout ([B, H, S, D] contiguous, or the [B, S, H, D] a head split leaves
before its transpose) the tile lands in shared memory as [128 rows][64] with the
128-byte swizzle the tensor core reads.
"""
from __future__ import annotations

import os

from ..plan import PKernel
from .common import CTYPE, ITEM, HEADER, KernelSource, TMapSpec, decompose_stmts, params_struct, prod

LOG2E = 1.4426950408889634
# Softmax tuning: EMU of every 16 exponential pairs on the FMA pipe (polynomial) instead of
# MUFU; DESYNC staggers the two query tiles by one key block; STAGES is the depth of the
# K/V ring; SPEC starts a block's exponentials with the current row max (speculation, redone
# when the max moved past the rescale threshold); ALT makes the two query tiles take turns on the
# MUFU (exponential phases alternate).
# SPLIT selects the split-row kernel (``attention_split_sm100.cuh``: the two threads of a query
# row keep separate softmax statistics and O accumulators, combined once at the end, instead of
# exchanging row maxima every key block).
# ``TENSORJIT_B200_ATTN="EMU=4,DESYNC=1"`` overrides.
# NAP: nanoseconds the producer and MMA warps sleep between barrier polls.  ROW selects the
# one-thread-per-row kernel (``attention_row_sm100.cuh``: 64-key blocks, S and P double-buffered
# in TMEM, 384 threads; STAGES then counts 64-key K/V stages).
# QUAD selects the four-threads-per-row kernel (``attention_quad_sm100.cuh``: one query tile per CTA,
# 256 TMEM columns, two CTAs per SM; STAGES is then at most 2).
# F2: the softmax's scale-and-shift FMAs and running sums as packed f32x2 instructions (sm_100),
# bit-identical to the scalar form with half the instructions.
ATTN_DEFAULTS = {"EMU": 0, "DESYNC": 1, "STAGES": 3, "SPEC": 0, "ALT": 1, "SPLIT": 0, "NAP": 0, "ROW": 0, "QUAD": 0,
                 "F2": 0}


def attention_knobs() -> dict:
    k = dict(ATTN_DEFAULTS)
    env = os.environ.get("TENSORJIT_B200_ATTN", "")
    for part in filter(None, (x.strip() for x in env.split(","))):
        name, _, val = part.partition("=")
        if name not in k:
            raise ValueError(f"TENSORJIT_B200_ATTN: unknown knob {name!r}")
        k[name] = int(val)
    if not 0 <= k["EMU"] <= 16:
        raise ValueError("TENSORJIT_B200_ATTN: EMU must be in 0..16")
    if not 2 <= k["STAGES"] <= (10 if k["ROW"] else 6):
        raise ValueError("TENSORJIT_B200_ATTN: STAGES must be in 2..6 (2..10 with ROW)")
    return k
BM = 128
BN = 128
THREADS = 640


def _map_for(shape: tuple, strides: tuple, n_batch: int):
    """Tensor-map dims of a logical [*batch, S, D] operand: ``ordered`` lists
    (element stride, role, extent) innermost first, role 'd', 's' or a batch dim
    index (size-1 batch dims are dropped); ``dims`` the extents in that order."""
    roles = []
    for i, (e, st) in enumerate(zip(shape, strides)):
        if i < n_batch and e == 1:
            continue
        role = "d" if i == len(shape) - 1 else ("s" if i == len(shape) - 2 else i)
        roles.append((st, role, e))
    d = [x for x in roles if x[1] == "d"]
    rest = sorted([x for x in roles if x[1] != "d"], key=lambda x: x[0])
    ordered = d + rest
    dims = [e for _, _, e in ordered]
    return ordered, dims


def gen_attention(k: PKernel, symbol: str, kernel_id: int) -> KernelSource:
    a = k.attrs
    batch = tuple(a["batch"])
    nb = len(batch)
    sq, sk, d, dv, dt = a["sq"], a["sk"], a["d"], a["dv"], a["dtype"]
    esz = ITEM[dt]
    ins = list(k.inputs)
    out_node, out_st = a["out"]
    in_index = {n.id: j for j, n in enumerate(ins)}
    out_idx = len(ins)
    status_idx = out_idx + 1
    bh_total = prod(batch)
    qpairs = (sq + 2 * BM - 1) // (2 * BM)

    kn = attention_knobs()
    STAGES = kn["STAGES"]
    bl, bidx = decompose_stmts("bh", batch, "b") if batch else ([], [])
    split = bool(kn["SPLIT"])
    row = bool(kn["ROW"])
    quad = bool(kn["QUAD"])
    if sum((split, row, quad)) > 1 or ((row or quad) and kn["SPEC"]):
        raise ValueError("TENSORJIT_B200_ATTN: SPLIT, ROW and QUAD exclude each other (and SPEC)")
    if quad:
        STAGES = min(STAGES, 2)       # two CTAs per SM must fit in shared memory
    kv_rows = 64 if row else BN
    threads = 384 if row else (576 if quad else THREADS)
    if split and kn["SPEC"]:
        raise ValueError("TENSORJIT_B200_ATTN: SPEC applies to the row-exchange kernel, not SPLIT")
    header = ("attention_row_sm100.cuh" if row else "attention_quad_sm100.cuh" if quad
              else "attention_split_sm100.cuh" if split else "attention_sm100.cuh")
    L = [HEADER, f'#include "{header}"',
         params_struct(status_idx + 1, 3)]
    L.append("struct Cfg {")
    L.append(f"  using T = {CTYPE[dt]};")
    L.append(f"  static constexpr int SQ = {sq}, SK = {sk}, D = {d}, DV = {dv}, STAGES = {STAGES};")
    L.append(f"  static constexpr long BATCH = {bh_total}L, O_NUMEL = {out_node.numel}L;")
    L.append(f"  static constexpr bool BF16 = {'true' if dt == 'bf16' else 'false'};")
    L.append(f"  static constexpr int EMU = {kn['EMU']};")
    L.append(f"  static constexpr bool DESYNC = {'true' if kn['DESYNC'] else 'false'};")
    L.append(f"  static constexpr bool SPEC = {'true' if kn['SPEC'] else 'false'};")
    L.append(f"  static constexpr bool ALT = {'true' if kn['ALT'] else 'false'};")
    L.append(f"  static constexpr int NAP = {int(kn['NAP'])};")
    L.append(f"  static constexpr bool F2 = {'true' if kn['F2'] else 'false'};")
    c = float(a["scale"]) * LOG2E
    L.append(f"  static constexpr float C = {c!r}f;")
    tmaps = []
    for name, seq in (("q", sq), ("k", sk), ("v", sk)):
        src, st = a[name]
        shape = batch + (seq, d if name != "v" else dv)
        ordered, dims = _map_for(shape, tuple(st), nb)
        rank = len(ordered)
        if not 2 <= rank <= 5:
            raise ValueError(f"attention operand {name}: tensor map rank {rank}")
        L.append(f"  static constexpr int {name.upper()}R = {rank};")
        L.append(f"  static __device__ __forceinline__ void {name}_coords(long bh, int s0, int (&c)[5]) {{")
        L += ["    " + s for s in bl]
        for mi, (_, role, _) in enumerate(ordered):
            if role == "d":
                e = "0"
            elif role == "s":
                e = "s0"
            else:
                e = f"static_cast<int>({bidx[role]})"
            L.append(f"    c[{mi}] = {e};")
        L.append("  }")
        box = [64] + [(BM if name == "q" else kv_rows) if role == "s" else 1 for _, role, _ in ordered[1:]]
        tmaps.append(TMapSpec(arg=in_index[src.id], dtype=dt, dims=dims,
                              strides=[s * esz for s, _, _ in ordered[1:]], box=box, swizzle=3))
    L.append("  static __device__ __forceinline__ long out_offset(long bh, long s) {")
    L += ["    " + s for s in bl]
    terms = [f"{bidx[i]} * {out_st[i]}L" for i in range(nb) if batch[i] != 1 and out_st[i] != 0]
    terms.append(f"s * {out_st[nb]}L")
    L.append(f"    return {' + '.join(terms)};")
    L.append("  }")
    L.append("};")
    L.append(f'extern "C" __global__ void __launch_bounds__({threads}, {2 if quad else 1}) '
             f'{symbol}(const __grid_constant__ Params prm) {{')
    fn = ("attention_row_sm100" if row else "attention_quad_sm100" if quad
          else "attention_split_sm100" if split else "attention_sm100")
    L.append(f"  tja::{fn}<Cfg>(prm, ({CTYPE[dt]}*)prm.p[{out_idx}], (int*)prm.p[{status_idx}], {kernel_id});")
    L.append("}")
    q_bytes, kv_bytes = BM * d * esz, BN * d * esz
    # + half-row maxima (2 parities x 2 tiles x 2 halves x 128 f32) and sums (2 x 2 x 128 f32)
    # + mbarriers (q_full, k/v_full and kv_empty per stage, s_full/s_free/p_ready/o_done/drain
    # per tile, 8 half-row exchange barriers, 2 turn tokens) + TMEM slot and abort flag
    smem = 1024 + 2 * q_bytes + STAGES * 2 * kv_bytes + 4096 + 2048 + (21 + 3 * STAGES) * 8 + 8
    if row:   # 64-key K / V stages; barriers (q_full, 3 per stage, 4 x 4 per tile buffer, 2 drain) + slot
        smem = 1024 + 2 * q_bytes + STAGES * 2 * (kv_rows * d * esz) + (1 + 3 * STAGES + 18) * 8 + 16
    if quad:  # one Q tile, the quarter-row exchange (2 x 4 x 128 f32), barriers + slot
        smem = 1024 + q_bytes + STAGES * 2 * kv_bytes + 4096 + (1 + 3 * STAGES + 9) * 8 + 16
    args = [("node", n) for n in ins] + [("node", out_node), ("status", None)]
    flops = 2.0 * bh_total * sq * sk * (d + dv)
    nbytes = sum(n.nbytes for n in ins) + out_node.nbytes
    grid = bh_total * ((sq + BM - 1) // BM if quad else qpairs)
    ks = KernelSource(symbol, "attention", "\n".join(L), (grid, 1, 1), (threads, 1, 1), args,
                      smem=smem, tmaps=tmaps,
                      info={"batch": bh_total, "sq": sq, "sk": sk, "d": d, "dv": dv, "flops": flops,
                            "bytes": nbytes, "exps": float(bh_total * sq * sk), "scale": a["scale"],
                            "ctas": bh_total * qpairs})
    ks.finalize_params()
    return ks
