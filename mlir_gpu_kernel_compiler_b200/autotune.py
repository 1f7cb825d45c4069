"""Tile search for the tcgen05 GEMM, rebuilt for Blackwell.

The reference autotuner (``tensorjit/runtime/autotune.py:48-118``) ranks candidate
tiles with a roofline-style cost model, times the top-k and persists the winner;
its CUDA backend ignores it (fixed 64x64x16 tiles, ``cuda_backend.py:556-557``).
Here the same three steps run over the sm_100a space:

* candidates: accumulator tile 128 x BN with BN in {64, 128, 256}, the number of
  shared-memory stages that fit in ~200 KB, and the L2 raster group GROUP_M;
* cost model: tensor time at the tile's MMA shape efficiency + wave
  quantisation over 148 SMs + the epilogue's HBM traffic;
* timing: ``autotune_gemm`` compiles the top-k candidates and times them with
  CUDA events on the device (GPU only); winners are stored in
  ``<cache>/autotune_b200.json`` keyed by (M, N, K, batch, dtype, B layout).
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

    def as_dict(self) -> dict:
        return asdict(self)


def candidates(N: int, b_mn_major: bool) -> list[TileConfig]:
    out = []
    for bn in (256, 128, 64, 32):
        if b_mn_major and bn % 64:
            continue
        if bn > 64 and N <= bn // 2:
            continue
        stage = 128 * 64 * 2 + bn * 64 * 2
        smax = max(2, min(8, (200 * 1024) // stage))
        for st in sorted({smax, max(2, smax - 1), 3, 4} - {0}):
            if st > smax:
                continue
            for gm in (8, 16, 32):
                out.append(TileConfig(bn, st, gm))
    return out


def cost_model(cfg: TileConfig, M: int, N: int, K: int, batch: int) -> float:
    """Lower is better (arbitrary units proportional to time)."""
    m_tiles = math.ceil(M / 128)
    n_tiles = math.ceil(N / cfg.BN)
    tiles = batch * m_tiles * n_tiles
    waves = math.ceil(tiles / NUM_SMS)
    # MMA issue efficiency per tile: wider N amortises the A operand and the per-k overheads
    eff = {256: 1.0, 128: 0.93, 64: 0.8, 32: 0.6}[cfg.BN]
    # work per wave in units of a full 128 x 256 x K tile
    tile_work = (128 * cfg.BN * K) / (128 * 256 * max(K, 1))
    t = waves * tile_work / eff
    # fill: padded tile area / useful area
    t *= (m_tiles * 128 * n_tiles * cfg.BN) / max(M * N, 1)
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


def tiles_for_plan(plan) -> dict:
    """Tile choice per matmul kernel index: a stored (timed) winner if there is one,
    else the cost-model pick.  ``TENSORJIT_B200_TILE=BN:STAGES[:GROUP_M]`` overrides."""
    from .codegen.gemm import _mm_dims, tc_eligible

    env = os.environ.get("TENSORJIT_B200_TILE")
    out = {}
    for idx, k in enumerate(plan.kernels):
        if k.kind != "matmul" or not tc_eligible(k):
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        if env:
            parts = [int(x) for x in env.split(":")]
            cfg = TileConfig(parts[0], parts[1], parts[2] if len(parts) > 2 else 16)
        else:
            cfg = lookup(M, N, K, batch, a.dtype, not tb) or pick(M, N, K, batch, not tb)
        out[idx] = cfg.as_dict()
    return out
