"""bench.py's host-side parts, without a GPU: the DRAM-traffic figures it attaches to the
roofline, and the reference arm (the reference's own generated C/OpenMP kernels on the host
cores) printing the contract's JSON line."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]


def _bench():
    sys.path.insert(0, str(ROOT))
    import bench

    return bench


def _sources(plan_name):
    from mlir_gpu_kernel_compiler_b200.autotune import tiles_for_plan
    from mlir_gpu_kernel_compiler_b200.codegen import generate
    from mlir_gpu_kernel_compiler_b200.fuse import fuse
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    x = fuse(PProgram.load(str(ROOT / "tests" / "golden" / "plans" / f"{plan_name}.json")))
    return {k.symbol: k for k in generate(x, tiles=tiles_for_plan(x))}


def test_cfg5_traffic_scales_with_rows_and_follows_the_tile_kind():
    b = _bench()
    full = _sources("cfg5_m131072")
    shard = _sources("cfg5_m16384")
    for sym in ("tj_matmul_1", "tj_matmul_2"):
        for k, scale in ((full[sym], 8), (shard[sym], 1)):
            per, rows = b.TRAFFIC[("cfg5", sym, b.tile_signature(k))]
            traffic, src = b.traffic_per_launch("cfg5", k)
            assert rows == 16384 and traffic == pytest.approx(per * scale) and "scaled" in src
    assert b.traffic_per_launch("cfg5", full["tj_row_0"])[0] is None


def test_traffic_is_withheld_for_a_tile_that_was_not_captured():
    b = _bench()
    k = _sources("cfg5_m131072")["tj_matmul_1"]
    k.info = dict(k.info, BN=64)          # a different tile than the captured one
    traffic, src = b.traffic_per_launch("cfg5", k)
    assert traffic is None and "no ncu capture" in src


def test_traffic_of_the_other_configs_names_their_dominant_kernels():
    b = _bench()
    for cfg, sym in (("cfg3", "tj_matmul_0"), ("cfg4", "tj_attention_2"), ("cfg2", "tj_row_0")):
        k = _sources(cfg)[sym]
        traffic, _ = b.traffic_per_launch(cfg, k)
        assert traffic == b.TRAFFIC[(cfg, sym, b.tile_signature(k))][0] > 0


def test_reference_arm_prints_the_contract_line():
    r = subprocess.run([sys.executable, "bench.py", "--config", "cfg1", "--impl", "reference", "--steps", "1",
                        "--warmup", "1"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better",
                "scaling", "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"):
        assert key in line
    assert line["impl"] == "reference" and line["value"] > 0 and line["unit"] == "TFLOP/s"
    assert line["cpu_baseline"]["kind"] == "reference" and line["cpu_baseline"]["value"] == line["value"]
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["d2h_bytes_per_step"] == 0


def test_reference_arm_uses_every_host_core_under_a_launcher():
    """torchrun sets OMP_NUM_THREADS=1 in every rank; the reference arm still runs rank 0 on
    every host core (and the other ranks exit without work)."""
    import os

    env = dict(os.environ, OMP_NUM_THREADS="1", RANK="0", WORLD_SIZE="2", LOCAL_RANK="0")
    r = subprocess.run([sys.executable, "bench.py", "--config", "cfg1", "--impl", "reference", "--steps", "1",
                        "--warmup", "1", "--gpus", "2"], cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stderr[-2000:]
    line = json.loads([x for x in r.stdout.splitlines() if x.startswith("{")][-1])
    if "unavailable" in line:
        pytest.skip(line["unavailable"])
    assert line["cpu_baseline"]["cores"] == len(os.sched_getaffinity(0)) and line["n_gpus"] == 2
    env["RANK"] = "1"
    r = subprocess.run([sys.executable, "bench.py", "--config", "cfg1", "--impl", "reference", "--steps", "1",
                        "--warmup", "1", "--gpus", "2"], cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0 and not r.stdout.strip()
