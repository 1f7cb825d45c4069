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
        k_full, k_shard = full[sym], shard[sym]
        per = b.CFG5_TRAFFIC_16K[(sym, bool(k_full.info["pair"]))]
        assert b.traffic_per_launch("cfg5", k_full) == pytest.approx(per * 8)
        per_s = b.CFG5_TRAFFIC_16K[(sym, bool(k_shard.info["pair"]))]
        assert b.traffic_per_launch("cfg5", k_shard) == pytest.approx(per_s)
    assert b.traffic_per_launch("cfg5", full["tj_row_0"]) is None


def test_traffic_of_the_other_configs_names_their_dominant_kernels():
    b = _bench()
    for cfg, sym in (("cfg3", "tj_matmul_0"), ("cfg4", "tj_attention_2"), ("cfg2", "tj_row_0")):
        k = _sources(cfg)[sym]
        assert b.traffic_per_launch(cfg, k) == b.TRAFFIC[(cfg, sym)] > 0


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
