"""Tile search for the tcgen05 GEMM, rebuilt for Blackwell.

The reference autotuner (``tensorjit/runtime/autotune.py:48-118``) ranks candidate
tiles with a roofline-style cost model, times the top-k and persists the winner;
its CUDA backend ignores it (fixed 64x64x16 tiles, ``cuda_backend.py:556-557``).
Here the same three steps run over the sm_100a space:

* candidates: accumulator tile 128 x BN with BN in {32, 64, 128, 256}, or 256 x BN
  (BN in {128, 256}) on a CTA pair (``cta_group::2``: two SMs share one MMA stream and
  each loads half of B), the number of shared-memory stages that fit in ~200 KB, and
  the L2 raster group GROUP_M;
* cost model: tensor time at the tile's MMA shape efficiency + wave
  quantisation over 148 SMs + the epilogue's HBM traffic;
* timing: ``autotune_plan`` compiles the top-k candidates and times them with
  CUDA events on the device (GPU only); winners are stored in
  ``<cache>/autotune_b200.json`` keyed by (M, N, K, batch, dtype, B layout).
  Winners measured on B200 for the benchmark programs ship in ``tuned_tiles.json``
  (consulted after the local store, before the cost model).

    python -m mlir_gpu_kernel_compiler_b200.autotune plan.json [...] [--out tuned_tiles.json]
    python -m mlir_gpu_kernel_compiler_b200.autotune --compare M N K --tile 256:4:16:0 --tile 256:5:16:1
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
    GROUP_N: int = 0        # column tiles per raster band (0 = all of N in one band)

    def as_dict(self) -> dict:
        return asdict(self)


STAGING = 32 * 1024          # TMA-store staging of the epilogue (8 warps x 2 x 2 KB)
SMEM_BUDGET = 232448 - 1024 - STAGING - 256


def candidates(N: int, b_mn_major: bool) -> list[TileConfig]:
    out = []
    # CTA-pair (cta_group::2) 256-row tiles need a K-major B; TENSORJIT_B200_PAIR=0 leaves
    # them out of the search
    pairs = (False,) if os.environ.get("TENSORJIT_B200_PAIR") == "0" else (False, True)
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
    eff = {256: 1.0, 128: 0.85, 64: 0.75, 32: 0.55}[cfg.BN]
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
    from .codegen.gemm import _mm_dims, gemm_form

    out = []
    for k in plan.kernels:
        form = gemm_form(k) if k.kind == "matmul" else None
        if form is None or form.mode != "f16":
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        sub = _single_kernel_plan(plan, k)
        for cfg in _ranked_candidates(M, N, K, batch, form.b_mn, top_k):
            for ks in generate(sub, tiles={0: cfg.as_dict()}):
                out.append((ks.symbol, ks.source))
    return out


def autotune_plan(plan, device="cuda", top_k: int = 6, iters: int = 10, verbose: bool = False) -> dict:
    """Time the top-k cost-model candidates of every tcgen05 GEMM of ``plan`` on the
    device and record the fastest (CUDA events around the kernel, inputs random)."""
    import torch

    from .codegen.gemm import _mm_dims, gemm_form
    from .program import TORCH_DTYPE, B200Program

    results = {}
    for idx, k in enumerate(plan.kernels):
        form = gemm_form(k) if k.kind == "matmul" else None
        if form is None or form.mode != "f16":
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        sub = _single_kernel_plan(plan, k)
        ins = [torch.randn(n.shape, device=device).mul_(0.05).to(TORCH_DTYPE[n.dtype]) for n in sub.inputs]
        cands = _ranked_candidates(M, N, K, batch, form.b_mn, top_k)
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
            record(M, N, K, batch, a.dtype, form.b_mn, best, best_ms)
            results[key(M, N, K, batch, a.dtype, form.b_mn)] = {"config": best.as_dict(), "ms": best_ms}
    return results


def tiles_for_plan(plan) -> dict:
    """Tile choice per matmul kernel index: a stored (timed) winner if there is one,
    else the cost-model pick.  ``TENSORJIT_B200_TILE=BN:STAGES[:GROUP_M[:PAIR]]`` overrides."""
    from .codegen.gemm import _mm_dims, gemm_form

    env = os.environ.get("TENSORJIT_B200_TILE")
    out = {}
    for idx, k in enumerate(plan.kernels):
        form = gemm_form(k) if k.kind == "matmul" else None
        if form is None or form.mode == "empty":
            continue
        mm, a, b, tb, M, N, K, out_shape = _mm_dims(k)
        batch = math.prod(out_shape[:-2]) if len(out_shape) > 2 else 1
        if form.mode == "x3":     # 3xTF32 kernels: a timed entry, else the generator's own choice
            cfg = lookup_any(M, N, K, batch, a.dtype, not tb)
            if cfg is not None:
                out[idx] = cfg.as_dict()
            continue
        if env:
            cfg = parse_tile(env)
            if cfg.PAIR and form.b_mn:
                cfg = TileConfig(cfg.BN, cfg.STAGES, cfg.GROUP_M, False, cfg.GROUP_N)
        else:
            cfg = lookup_any(M, N, K, batch, a.dtype, form.b_mn) or pick(M, N, K, batch, form.b_mn)
        out[idx] = cfg.as_dict()
    return out


def parse_tile(s: str) -> TileConfig:
    """``BN:STAGES[:GROUP_M[:PAIR[:GROUP_N]]]`` (the ``TENSORJIT_B200_TILE`` syntax)."""
    parts = [int(x) for x in s.split(":")]
    return TileConfig(parts[0], parts[1], parts[2] if len(parts) > 2 else 16, bool(parts[3]) if len(parts) > 3 else False,
                      parts[4] if len(parts) > 4 else 0)


def plain_gemm_plan(M: int, N: int, K: int, dtype: str = "bf16"):
    """A one-kernel plan ``y[M, N] = a[M, K] @ b[N, K]^T`` with no epilogue: the bare
    tcgen05 GEMM, for comparing tiles with a library GEMM on identical operands."""
    from .plan import PProgram

    nodes = [{"id": 0, "op": "input", "name": "a", "inputs": [], "shape": [M, K], "dtype": dtype, "attrs": {}},
             {"id": 1, "op": "input", "name": "b", "inputs": [], "shape": [N, K], "dtype": dtype, "attrs": {}},
             {"id": 2, "op": "matmul", "name": "y", "inputs": [0, 1], "shape": [M, N], "dtype": dtype,
              "attrs": {"trans_b": True}}]
    return PProgram.from_dict({
        "format": "tensorjit-plan/1", "name": f"gemm_{M}x{N}x{K}_{dtype}", "nodes": nodes, "inputs": [0, 1],
        "outputs": [2], "aliases": {}, "meta": {"dtype": dtype},
        "kernels": [{"kind": "matmul", "nodes": [2], "anchor": 2, "inputs": [0, 1], "outputs": [2],
                     "iter_shape": [M, N]}]})


def compare_with_library(M: int, N: int, K: int, tiles: list[TileConfig], rounds: int = 4, seconds: float = 1.0,
                         dtype: str = "bf16", device: str = "cuda") -> dict:
    """Time the bare GEMM with each tile and torch's library GEMM (``F.linear``, cuBLAS) on
    the same operands.  The arms take turns (order reversed every round) for ``rounds``
    rounds of about ``seconds`` each, so drift of temperature and power-capped clocks
    reaches every arm alike; the median SM clock and board power over each arm's rounds
    are sampled through NVML.  ``rounds=0`` runs every arm twice, untimed (a short
    command to profile).  Returns {arm: {"ms", "tflops", "sm_mhz", "watts"}}."""
    import statistics
    import time

    import torch

    from .program import TORCH_DTYPE, B200Program

    dt = TORCH_DTYPE[dtype]
    g = torch.Generator(device=device).manual_seed(1)
    a = torch.randn((M, K), generator=g, device=device).to(dt)
    b = (torch.randn((N, K), generator=g, device=device) * 0.02).to(dt)
    out = torch.empty((M, N), dtype=dt, device=device)
    arms = {}
    for cfg in tiles:
        prog = B200Program(plain_gemm_plan(M, N, K, dtype), device=device, use_graph=False,
                           tiles={0: cfg.as_dict()})
        arms[f"{cfg.BN}:{cfg.STAGES}:{cfg.GROUP_M}:{int(cfg.PAIR)}" + (f":{cfg.GROUP_N}" if cfg.GROUP_N else "")] = prog

    def run(name, iters):
        if name == "library":
            for _ in range(iters):
                torch.nn.functional.linear(a, b)
        else:
            for _ in range(iters):
                arms[name].run_into([a, b], [out])

    names = list(arms) + ["library"]
    if rounds <= 0:
        for n in names:
            run(n, 2)
        torch.cuda.synchronize()
        for prog in arms.values():
            prog.check()
        return {}
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    run(names[0], 2)
    ev0.record()
    run(names[0], 3)
    ev1.record()
    torch.cuda.synchronize()
    iters = max(3, int(seconds * 1000 / max(ev0.elapsed_time(ev1) / 3, 1e-3)))
    samples = []
    sampler = _PowerSampler(torch.cuda.current_device(), samples)
    res = {n: [] for n in names}
    with sampler:
        for r in range(rounds):
            for n in (names if r % 2 == 0 else names[::-1]):
                run(n, 1)
                torch.cuda.synchronize()
                t0 = time.time()
                ev0.record()
                run(n, iters)
                ev1.record()
                torch.cuda.synchronize()
                t1 = time.time()
                sel = [s for s in samples if t0 <= s[0] <= t1]
                res[n].append((ev0.elapsed_time(ev1) / iters, statistics.median(s[1] for s in sel) if sel else None,
                               statistics.median(s[2] for s in sel) if sel else None))
    for prog in arms.values():
        prog.check()
    summary = {}
    for n, v in res.items():
        ms = statistics.median(x[0] for x in v)
        clk = [x[1] for x in v if x[1] is not None]
        pw = [x[2] for x in v if x[2] is not None]
        summary[n] = {"ms": ms, "tflops": 2.0 * M * N * K / ms / 1e9,
                      "sm_mhz": statistics.median(clk) if clk else None, "watts": statistics.median(pw) if pw else None}
    return summary


class _PowerSampler:
    """(time, SM MHz, board W) every ~5 ms from NVML while the ``with`` block runs."""

    def __init__(self, index: int, out: list):
        self.index, self.out, self._stop, self._t = index, out, threading.Event(), None

    def _run(self):
        import time

        try:
            import pynvml

            pynvml.nvmlInit()
        except Exception:
            return
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            while not self._stop.is_set():
                self.out.append((time.time(), pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM),
                                 pynvml.nvmlDeviceGetPowerUsage(h) / 1000.0))
                self._stop.wait(0.005)
        finally:
            pynvml.nvmlShutdown()

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        return self

    def __exit__(self, *exc):
        self._stop.set()
        self._t.join(timeout=10)


def main(argv=None):
    import argparse

    from .plan import PProgram

    ap = argparse.ArgumentParser(description="time tcgen05 GEMM tile candidates for plans on the GPU")
    ap.add_argument("plans", nargs="*")
    ap.add_argument("--top-k", type=int, default=6)
    ap.add_argument("--out", default=None, help="also merge the winners into this JSON file")
    ap.add_argument("--compare", type=int, nargs=3, metavar=("M", "N", "K"), default=None,
                    help="time the bare GEMM of this shape with each --tile against the library GEMM")
    ap.add_argument("--tile", action="append", default=[], help="BN:STAGES[:GROUP_M[:PAIR]] (repeatable)")
    ap.add_argument("--rounds", type=int, default=4)
    ap.add_argument("--dtype", default="bf16", choices=["bf16", "f16"])
    a = ap.parse_args(argv)
    if a.compare:
        M, N, K = a.compare
        tiles = [parse_tile(t) for t in a.tile] or [pick(M, N, K, 1, False)]
        res = compare_with_library(M, N, K, tiles, rounds=a.rounds, dtype=a.dtype)
        for n, r in res.items():
            print(f"{M}x{N}x{K} {n:12s} {r['ms']:.4f} ms  {r['tflops']:7.1f} TFLOP/s  "
                  f"SM {r['sm_mhz']} MHz  {r['watts']} W")
        if a.rounds <= 0:
            print("ran every arm twice")
        return
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
