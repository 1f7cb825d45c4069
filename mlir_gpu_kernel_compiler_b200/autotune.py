"""Tile search for the tcgen05 GEMM, rebuilt for Blackwell.

The reference autotuner (``tensorjit/runtime/autotune.py:48-118``) ranks candidate
tiles with a roofline-style cost model, times the top-k and persists the winner;
its CUDA backend ignores it (fixed 64x64x16 tiles, ``cuda_backend.py:556-557``).
Here the same three steps run over the sm_100a space:

* candidates: accumulator tile 128 x BN with BN in {64, 128, 256}, the number of
  shared-memory stages that fit in ~200 KB, and the L2 raster group GROUP_M;
* cost model: tensor time at the tile's MMA shape efficiency + wave
  quantisation over 148 SMs + the epilogue's HBM traffic;
* timing: ``autotune_plan`` compiles the top-k candidates and times them with
  CUDA events on the device (GPU only); winners are stored in
  ``<cache>/autotune_b200.json`` keyed by (M, N, K, batch, dtype, B layout).
  Winners measured on B200 for the benchmark programs ship in ``tuned_tiles.json``
  (consulted after the local store, before the cost model).

    python -m mlir_gpu_kernel_compiler_b200.autotune plan.json [...] [--out tuned_tiles.json]
"""
from __future__ import annotations

import json
import math
import os
import threading
from dataclasses import asdict, dataclass
from pathlib import Path

from .codegen.common import NUM_SMS

_lock = threading.Lock()


@dataclass(frozen=True)
class TileConfig:
    BN: int
    STAGES: int
    GROUP_M: int = 16
    PAIR: bool = False      # 2-SM cluster (cta_group::2), 256-row tiles

    def as_dict(self) -> dict:
        return asdict(self)


STAGING = 32 * 1024          # TMA-store staging of the epilogue (8 warps x 2 x 2 KB)
SMEM_BUDGET = 232448 - 1024 - STAGING - 256


def candidates(N: int, b_mn_major: bool) -> list[TileConfig]:
    out = []
    # CTA-pair (cta_group::2) tiles are correct but measured ~1.8x slower than single-CTA
    # 128 x 256 tiles on B200 (cfg3: 1.52 ms vs 0.83 ms); they are searched only on request.
    pairs = (False, True) if os.environ.get("TENSORJIT_B200_PAIR") == "1" else (False,)
    for pair in pairs:
        if pair and b_mn_major:
            continue
        for bn in ((256, 128) if pair else (256, 128, 64, 32)):
            if b_mn_major and bn % 64:
                continue
            if bn > 64 and N <= bn // 2:
                continue
            stage = 128 * 64 * 2 + (bn // 2 if pair else bn) * 64 * 2
            smax = max(2, min(8, SMEM_BUDGET // stage))
            for st in sorted({smax, max(2, smax - 1), 3, 4} - {0}):
                if st > smax:
                    continue
                for gm in (8, 16, 32):
                    out.append(TileConfig(bn, st, gm, pair))
    return out


def cost_model(cfg: TileConfig, M: int, N: int, K: int, batch: int) -> float:
    """Lower is better (arbitrary units proportional to time)."""
    rows = 256 if cfg.PAIR else 128
    m_tiles = math.ceil(M / rows)
    n_tiles = math.ceil(N / cfg.BN)
    tiles = batch * m_tiles * n_tiles
    waves = math.ceil(tiles / (NUM_SMS // 2 if cfg.PAIR else NUM_SMS))
    # MMA issue efficiency per tile: wider N amortises the A operand and the per-k overheads
    eff = {256: 1.0, 128: 0.93, 64: 0.8, 32: 0.6}[cfg.BN]
    # work per wave in units of a full 128 x 256 x K tile per SM
    tile_work = (128 * cfg.BN * K) / (128 * 256 * max(K, 1))
    t = waves * tile_work / eff
    if cfg.PAIR:
        t *= 0.93     # half the B operand traffic per SM
    # fill: padded tile area / useful area
    t *= (m_tiles * rows * n_tiles * cfg.BN) / max(M * N, 1)
    # shallow pipelines stall on HBM latency; every extra stage hides a little more
    if cfg.STAGES < 3:
        t *= 1.25
    t *= 1.0 + 0.01 * (8 - min(cfg.STAGES, 8))
    # L2 raster: prefer groups covering ~16 m-tiles for wide problems
    t *= 1.0 + 0.02 * abs(math.log2(cfg.GROUP_M / 16))
    return t


def pick(M: int, N: int, K: int, batch: int, b_mn_major: bool) -> TileConfig:
    cands = candidates(N, b_mn_major)
    return min(cands, key=lambda c: cost_model(c, M, N, K, batch))


def store_path() -> Path:
    from .toolchain import cache_dir

    return cache_dir() / "autotune_b200.json"


def _load() -> dict:
    try:
        return json.loads(store_path().read_text())
    except (OSError, ValueError):
        return {}


def key(M, N, K, batch, dtype, b_mn_major) -> str:
    return f"b200|gemm|{M}x{N}x{K}|b{batch}|{dtype}|{'nn' if b_mn_major else 'nt'}"


def lookup(M, N, K, batch, dtype, b_mn_major) -> TileConfig | None:
    with _lock:
        d = _load().get(key(M, N, K, batch, dtype, b_mn_major))
    return TileConfig(**d["config"]) if d else None


def record(M, N, K, batch, dtype, b_mn_major, cfg: TileConfig, ms: float) -> None:
    with _lock:
        d = _load()
        d[key(M, N, K, batch, dtype, b_mn_major)] = {"config": cfg.as_dict(), "ms": ms}
        p = store_path()
        tmp = p.with_suffix(f".{os.getpid()}.tmp")
        tmp.write_text(json.dumps(d, indent=1, sort_keys=True))
        os.replace(tmp, p)


def _shipped() -> dict:
    """Timed winners shipped with the package (measured on B200 by ``autotune_plan``)."""
    p = Path(__file__).resolve().parent / "tuned_tiles.json"
    try:
        return json.loads(p.read_text())
    except (OSError, ValueError):
        return {}


def lookup_any(M, N, K, batch, dtype, b_mn_major) -> TileConfig | None:
    cfg = lookup(M, N, K, batch, dtype, b_mn_major)
    if cfg is None:
        d = _shipped().get(key(M, N, K, batch, dtype, b_mn_major))
        cfg = TileConfig(**d["config"]) if d else None
    return cfg


def _single_kernel_plan(plan, k):
    """A program holding just kernel ``k`` (its inputs become program inputs)."""
    from .plan import PProgram

    nodes = list(k.inputs) + [n for n in k.nodes if n not in k.inputs]
    consts = [i for n in k.nodes for i in n.inputs if i.op == "const" and i not in nodes]
    return PProgram(name=f"{plan.name}_k", nodes=consts + nodes, inputs=list(k.inputs), outputs=list(k.outputs),
                    kernels=[k], aliases={})


def _ranked_candidates(M, N, K, batch, b_mn_major, top_k):
    ranked = sorted(candidates(N, b_mn_major), key=lambda c: cost_model(c, M, N, K, batch))
    per_bn: dict[tuple, list] = {}
    for c in ranked:                      # the best two of every tile shape, best shapes first
        per_bn.setdefault((c.BN, c.PAIR), [])
        if len(per_bn[(c.BN, c.PAIR)]) < 2:
            per_bn[(c.BN, c.PAIR)].append(c)
    return [c for lst in per_bn.values() for c in lst][:top_k]


def candidate_sources(plan, top_k: int = 6) -> list[tuple[str, str]]:
    """(name, CUDA source) of every candidate ``autotune_plan`` would time, so they can be
    compiled ahead of time (nvcc runs on the CPU)."""
    from .codegen import generate
    from .codegen.gemm import _mm_dims, tc_eligible

    out = []
    for k in plan.kernels:
        if k.kind != "matmul" or not tc_eligible(k):
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        sub = _single_kernel_plan(plan, k)
        for cfg in _ranked_candidates(M, N, K, batch, not tb, top_k):
            ks = generate(sub, tiles={0: cfg.as_dict()})[0]
            out.append((ks.symbol, ks.source))
    return out


def autotune_plan(plan, device="cuda", top_k: int = 6, iters: int = 10, verbose: bool = False) -> dict:
    """Time the top-k cost-model candidates of every tcgen05 GEMM of ``plan`` on the
    device and record the fastest (CUDA events around the kernel, inputs random)."""
    import torch

    from .codegen.gemm import _mm_dims, tc_eligible
    from .program import TORCH_DTYPE, B200Program

    results = {}
    for idx, k in enumerate(plan.kernels):
        if k.kind != "matmul" or not tc_eligible(k):
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        sub = _single_kernel_plan(plan, k)
        ins = [torch.randn(n.shape, device=device).mul_(0.05).to(TORCH_DTYPE[n.dtype]) for n in sub.inputs]
        cands = _ranked_candidates(M, N, K, batch, not tb, top_k)
        best, best_ms = None, float("inf")
        for cfg in cands:
            try:
                prog = B200Program(sub, device=device, use_graph=False, tiles={0: cfg.as_dict()})
                outs = [torch.empty(s, dtype=d, device=device) for s, d in prog.output_specs()]
                prog.time_kernels(ins, outs, iters=2)
                ms = sum(prog.time_kernels(ins, outs, iters=iters))
                prog.check()
                prog.close()
            except Exception as e:  # a candidate that does not build or run is skipped
                if verbose:
                    print(f"  {cfg}: failed {str(e)[:120]}")
                continue
            if verbose:
                print(f"  kernel {idx} {M}x{N}x{K} b{batch}: {cfg} {ms * 1e3:.1f} us")
            if ms < best_ms:
                best, best_ms = cfg, ms
        if best is not None:
            record(M, N, K, batch, a.dtype, not tb, best, best_ms)
            results[key(M, N, K, batch, a.dtype, not tb)] = {"config": best.as_dict(), "ms": best_ms}
    return results


def tiles_for_plan(plan) -> dict:
    """Tile choice per matmul kernel index: a stored (timed) winner if there is one,
    else the cost-model pick.  ``TENSORJIT_B200_TILE=BN:STAGES[:GROUP_M[:PAIR]]`` overrides."""
    from .codegen.gemm import _mm_dims, tc_eligible

    env = os.environ.get("TENSORJIT_B200_TILE")
    out = {}
    for idx, k in enumerate(plan.kernels):
        if k.kind != "matmul" or not tc_eligible(k):
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        if a.dtype == "f32":      # 3xTF32 kernels: a timed entry, else the generator's own choice
            cfg = lookup_any(M, N, K, batch, a.dtype, not tb)
            if cfg is not None:
                out[idx] = cfg.as_dict()
            continue
        if env:
            parts = [int(x) for x in env.split(":")]
            cfg = TileConfig(parts[0], parts[1], parts[2] if len(parts) > 2 else 16,
                             bool(parts[3]) if len(parts) > 3 else False)
            if cfg.PAIR and not tb:
                cfg = TileConfig(cfg.BN, cfg.STAGES, cfg.GROUP_M, False)
        else:
            cfg = lookup_any(M, N, K, batch, a.dtype, not tb) or pick(M, N, K, batch, not tb)
        out[idx] = cfg.as_dict()
    return out


def main(argv=None):
    import argparse

    from .plan import PProgram

    ap = argparse.ArgumentParser(description="time tcgen05 GEMM tile candidates for plans on the GPU")
    ap.add_argument("plans", nargs="+")
    ap.add_argument("--top-k", type=int, default=6)
    ap.add_argument("--out", default=None, help="also merge the winners into this JSON file")
    a = ap.parse_args(argv)
    allres = {}
    for p in a.plans:
        print(p)
        allres.update(autotune_plan(PProgram.load(p), top_k=a.top_k, verbose=True))
    if a.out:
        try:
            cur = json.loads(Path(a.out).read_text())
        except (OSError, ValueError):
            cur = {}
        cur.update(allres)
        Path(a.out).write_text(json.dumps(cur, indent=1, sort_keys=True))
    print(json.dumps(allres, indent=1))


if __name__ == "__main__":
    main()
