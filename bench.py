#!/usr/bin/env python
"""Benchmark of the tensorjit B200 backend on the BASELINE programs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg5] [--impl b200|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Default workload: cfg5, the large-batch MLP x + linear(gelu(linear(rms_norm(x,g),w1,b1)),w2,b2)
in bf16 with x[131072,4096], w1[16384,4096], w2[4096,16384] — the program the
reference's north star runs at 1/2/4/8 GPUs.  Its rows are split across ranks
(rank p owns rows [p*R/N, (p+1)*R/N), weights replicated, no collective in the
step), so the global batch is fixed: strong scaling.  A step is one execution
of the whole compiled program (RMSNorm row kernel + two tcgen05 GEMMs with
fused epilogues) over the rank's rows, as one CUDA graph.

``value``  whole-job algorithmic TFLOP/s with inputs resident in HBM
           (inputs are larger than L2, so no flush is needed between steps).
``e2e``    the same through the public call ``program(*inputs)`` with the rank's
           rows copied from pinned host memory every step and the result copied
           back (the weights stay resident, as a served model's would).
``roofline`` the dominant kernel's achieved rate from CUDA events around each
           kernel, against MEASURED_PEAKS.json.
``cpu_baseline`` the reference's own ``c`` backend (its generated C/OpenMP kernels,
           built for this host by oracle/ref_runner.py) on a bounded row sample.

``--impl reference`` times that reference implementation alone, on the same
metric, and prints its own line (rank 0 only under torchrun).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import threading
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "program latency; GEMM TFLOP/s and row-kernel HBM GB/s vs B200 peak, 1/2/4/8 GPU"
REF_SAMPLE = {"cfg1": ("cfg1", None), "cfg2": ("cfg2", None), "cfg3": ("cfg3_m512", 512), "cfg4": ("cfg4", None),
              "cfg5": ("cfg5_m1024", 1024)}


L2_BYTES = 126 * 1024 * 1024  # B200 L2


def _tensor_family(family: str) -> bool:
    """Kernels whose roofline is the tensor core (GEMMs and the fused attention)."""
    return family.startswith("gemm") or family == "attention"


def peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": d["hbm_gbs"], "bf16_tflops": d["bf16_tflops"],
                "bf16_tflops_sustained": d.get("bf16_tflops_sustained", d["bf16_tflops"]), "source": "measured"}
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0, "source": "fallback"}


class Clocks:
    """SM clock and throttle reasons sampled every ~3 ms during the timed region (NVML;
    nvidia-smi every 200 ms if NVML is unavailable).  ``__enter__`` returns only once the
    sampler is running, so even a timed region of a few milliseconds gets samples."""

    REASONS = {"hw_slowdown": 0x8, "sw_thermal_slowdown": 0x20, "hw_thermal_slowdown": 0x40, "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index, self.rows, self._stop = index, [], threading.Event()
        self._ready = threading.Event()
        self._t = None

    def _run_nvml(self):
        import pynvml

        pynvml.nvmlInit()
        try:
            h = pynvml.nvmlDeviceGetHandleByIndex(self.index)
            mx = pynvml.nvmlDeviceGetMaxClockInfo(h, pynvml.NVML_CLOCK_SM)
            self._ready.set()
            while not self._stop.is_set():
                sm = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM)
                r = pynvml.nvmlDeviceGetCurrentClocksThrottleReasons(h)
                self.rows.append((float(sm), float(mx), [k for k, v in self.REASONS.items() if r & v]))
                self._stop.wait(0.003)
        finally:
            pynvml.nvmlShutdown()

    def _run_smi(self):
        q = ("clocks.sm,clocks.max.sm,clocks_event_reasons.hw_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_power_cap")
        names = ["hw_slowdown", "sw_thermal_slowdown", "hw_thermal_slowdown", "sw_power_cap"]
        while not self._stop.is_set():
            r = subprocess.run(["nvidia-smi", f"--id={self.index}", f"--query-gpu={q}", "--format=csv,noheader,nounits"],
                               capture_output=True, text=True, timeout=5)
            if r.returncode == 0 and r.stdout.strip():
                f = [x.strip() for x in r.stdout.strip().split(",")]
                self.rows.append((float(f[0]), float(f[1]), [n for n, v in zip(names, f[2:]) if v == "Active"]))
            self._stop.wait(0.2)

    def _run(self):
        try:
            self._run_nvml()
        except Exception:
            self._ready.set()
            try:
                self._run_smi()
            except Exception:
                pass

    def __enter__(self):
        self._t = threading.Thread(target=self._run, daemon=True)
        self._t.start()
        self._ready.wait(timeout=10)
        return self

    def __exit__(self, *a):
        self._stop.set()
        if self._t:
            self._t.join(timeout=10)

    def summary(self) -> dict:
        if not self.rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        import statistics

        return {"sm_mhz": statistics.median(r[0] for r in self.rows), "sm_max_mhz": max(r[1] for r in self.rows),
                "reasons": sorted({x for r in self.rows for x in r[2]}), "samples": len(self.rows)}


def _trace(*a):
    if os.environ.get("TJ_BENCH_TRACE") == "1":
        print("[bench]", *a, file=sys.stderr, flush=True)


def _dist():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def reference_baseline(cfg: str, steps: int, warmup: int, threads: int | None = None) -> dict | None:
    """Time the reference c backend's kernels on a bounded sample; None if unavailable."""
    import numpy as np

    from mlir_gpu_kernel_compiler_b200 import workloads as W
    from oracle import ref_runner

    name, rows = REF_SAMPLE[cfg]
    if not ref_runner.available(name):
        return None
    w = W.WORKLOADS[cfg]
    ins = [t.float().numpy() for t in W.make_inputs(w, rows=(0, rows) if rows else None)]
    prog = ref_runner.RefProgram(name)
    for _ in range(max(warmup, 1)):
        prog.run(ins)
    ts = []
    for _ in range(steps):
        t0 = time.perf_counter()
        prog.run(ins)
        ts.append(time.perf_counter() - t0)
    sec = float(np.median(ts))
    frac = (rows / w.rows) if rows else 1.0
    work = (w.flops or w.hbm_bytes) * frac
    unit_scale = 1e12 if w.flops else 1e9
    return {"value": work / sec / unit_scale, "unit": "TFLOP/s" if w.flops else "GB/s",
            "cores": int(os.environ.get("OMP_NUM_THREADS", os.cpu_count() or 1)), "kind": "reference",
            "sample": f"{name}: reference c backend (generated C/OpenMP, -O3 -march=native -fopenmp) on "
                      f"{rows or 'all'} rows, median of {steps} runs, {sec * 1e3:.1f} ms per sample",
            "ms_per_sample": sec * 1e3}


def run_reference(a) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
    os.environ.setdefault("OMP_NUM_THREADS", str(os.cpu_count() or 1))
    res = reference_baseline(a.config, a.steps, a.warmup)
    if res is None:
        print(json.dumps({"impl": "reference", "unavailable": "oracle/_ref has no generated reference kernels "
                                                              "(run oracle/build_ref.py where the reference is present)"}))
        return
    from mlir_gpu_kernel_compiler_b200 import workloads as W

    w = W.WORKLOADS[a.config]
    sharded = a.config == "cfg5"
    total_rows = a.rows or w.rows
    line = {"metric": METRIC, "impl": "reference", "value": res["value"], "unit": res["unit"], "n_gpus": world,
            "steps": a.steps, "warmup": a.warmup, "ms_per_step": res["ms_per_sample"], "higher_is_better": True,
            "scaling": "strong" if sharded else "weak", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic: seeded CPU-generator inputs with the BASELINE shapes and distributions",
            "config": {"workload": f"{a.config}: {w.description}",
                       "plan": W.sharded_plan_name(w, world, total_rows) if sharded else w.plan,
                       "global_rows": total_rows if sharded else None,
                       "parallelism": f"rows{world}" if sharded else f"replicas{world}",
                       "sample": res["sample"]},
            "cpu_baseline": {k: res[k] for k in ("value", "unit", "cores", "kind", "sample")},
            "e2e": {"value": res["value"], "unit": res["unit"], "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line))


def run_b200(a) -> None:
    import torch
    import torch.distributed as dist

    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    world, rank, local = _dist()
    _trace("start", world, rank)
    if world > 1:
        from datetime import timedelta

        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=timedelta(seconds=180))
    dev = torch.device("cuda", local)
    torch.cuda.set_device(dev)
    w = W.WORKLOADS[a.config]
    sharded = a.config == "cfg5"
    total_rows = a.rows or w.rows
    if a.rows and (not sharded or w.rows % a.rows or a.rows % world):
        raise SystemExit("--rows: cfg5 only, a divisor of its 131072 rows and a multiple of the GPU count")
    plan_name = W.sharded_plan_name(w, world, total_rows) if sharded else w.plan
    plan = PProgram.load(ROOT / "tests" / "golden" / "plans" / f"{plan_name}.json")
    rows = W.shard_rows(total_rows, world, rank) if sharded else None
    _trace("inputs")
    ins = W.make_inputs(w, device=dev, rows=rows)
    _trace("compile")
    prog = B200Program(plan, device=dev, use_graph=True)
    outs = [torch.empty(s, dtype=d, device=dev) for s, d in prog.output_specs()]
    _trace("run")
    stream = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    for _ in range(a.warmup):
        prog.run_into(ins, outs)
    torch.cuda.synchronize(dev)
    prog.check()
    barrier()
    torch.cuda.synchronize(dev)
    # A step whose inputs, outputs and intermediates together exceed L2 evicts the previous
    # step's data by itself; a smaller one (cfg1) is timed step by step with L2 flushed before
    # each step by a write of twice its size, outside the timed events.
    footprint = sum(t.numel() * t.element_size() for t in ins + outs) + prog.arena_bytes
    flush = None
    if footprint < L2_BYTES:
        flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev)
    clk = Clocks(local)
    with clk:
        if flush is None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(a.steps):
                prog.run_into(ins, outs)
            end.record(stream)
            torch.cuda.synchronize(dev)
            ms = start.elapsed_time(end) / a.steps
        else:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(a.steps)]
            for s0, s1 in evs:
                flush.fill_(1.0)
                s0.record(stream)
                prog.run_into(ins, outs)
                s1.record(stream)
            torch.cuda.synchronize(dev)
            ms = sum(s0.elapsed_time(s1) for s0, s1 in evs) / a.steps
    l2_note = ("inputs, outputs and intermediates of a step exceed L2 (no flush needed)" if flush is None
               else f"L2 flushed before every timed step ({2 * L2_BYTES >> 20} MiB write, outside the events)")
    barrier()
    t = torch.tensor([ms], device=dev)
    if world > 1:
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
    ms_max = float(t.item())
    frac_rows = ((rows[1] - rows[0]) * world / w.rows) if sharded else world
    total_work = (w.flops or w.hbm_bytes) * frac_rows
    unit_scale, unit = (1e12, "TFLOP/s") if w.flops else (1e9, "GB/s")
    value = total_work / (ms_max * 1e-3) / unit_scale

    # per-kernel device times (events around every kernel, same stream) -> dominant kernel roofline
    kms = prog.time_kernels(ins, outs, iters=max(3, min(a.steps, 10)))
    pk = peaks()
    dom = max(range(len(kms)), key=lambda i: kms[i])
    ks = prog.kernel_sources[dom]
    if _tensor_family(ks.family):
        ach = ks.info["flops"] / (kms[dom] * 1e-3) / 1e12
        peak = pk["bf16_tflops_sustained"] if a.config in ("cfg4", "cfg5") else pk["bf16_tflops"]
        kind = ("sustained" if peak == pk["bf16_tflops_sustained"] else "burst") + " bf16"
        if ks.info.get("tf32x3"):
            # f32 GEMM on the TF32 tensor path: half the bf16 rate, three MMAs per product
            peak, kind = peak / 6.0, kind + " / 2 (TF32 rate) / 3 (3xTF32 products)"
        roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "kernel": ks.symbol, "ms": kms[dom],
                "peak_kind": kind + (", of measured" if pk["source"] == "measured" else ", of fallback")}
    else:
        ach = ks.info["bytes"] / (kms[dom] * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                "kernel": ks.symbol, "ms": kms[dom],
                "peak_kind": "copy bandwidth, " + ("of measured" if pk["source"] == "measured" else "of fallback")}
    roof["traffic"] = traffic_per_launch(a.config, ks)
    per_kernel = [{"kernel": k.symbol, "family": k.family, "ms": round(m, 4),
                   "rate": round((k.info["flops"] / (m * 1e-3) / 1e12) if _tensor_family(k.family)
                                 else (k.info["bytes"] / (m * 1e-3) / 1e9), 1) if m > 0 else None,
                   "rate_unit": "TFLOP/s" if _tensor_family(k.family) else "GB/s"}
                  for k, m in zip(prog.kernel_sources, kms)]

    # end to end through the public API with host data every step: HostPipeline streams the
    # row inputs in from pinned host memory and the result out, overlapping both copy
    # directions with compute across consecutive steps (weights stay resident)
    e2e = None
    if not a.no_e2e:
        from mlir_gpu_kernel_compiler_b200.pipeline import HostPipeline

        stream_idx = list(w.row_args) or list(range(len(ins)))
        resident = {i: t for i, t in enumerate(ins) if i not in stream_idx}
        host_in = {i: ins[i].cpu().pin_memory() for i in stream_idx}
        host_out = [[torch.empty(s, dtype=d).pin_memory() for s, d in prog.output_specs()] for _ in range(2)]
        h2d = sum(t.numel() * t.element_size() for t in host_in.values())
        d2h = sum(t.numel() * t.element_size() for t in host_out[0])
        pipe = HostPipeline(prog, stream_idx, resident, depth=2)
        for k in range(max(2, min(a.warmup, 3))):
            pipe.submit(host_in, host_out[k % 2])
        pipe.synchronize()
        barrier()
        s2, e2 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s2.record(pipe.s_h2d)
        for k in range(a.steps):
            pipe.submit(host_in, host_out[k % 2])
        pipe.s_d2h.wait_stream(pipe.s_comp)
        e2.record(pipe.s_d2h)
        pipe.synchronize()
        ems = s2.elapsed_time(e2) / a.steps
        t2 = torch.tensor([ems], device=dev)
        if world > 1:
            dist.all_reduce(t2, op=dist.ReduceOp.MAX)
        ems = float(t2.item())
        e2e = {"value": total_work / (ems * 1e-3) / unit_scale, "unit": unit, "ms_per_step": ems,
               "h2d_bytes_per_step": h2d, "d2h_bytes_per_step": d2h,
               "how": "HostPipeline: pinned host rows in, result out, copies overlapped with compute across steps"}
    prog.check()

    cpu = None
    if rank == 0 and world == 1 and not a.no_cpu_baseline:
        try:
            cpu = reference_baseline(a.config, steps=2, warmup=1)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}
    launches = sum(1 for L in prog.launches if all(g > 0 for g in L["grid"])) * a.steps
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32",
            "data": "synthetic: seeded CPU-generator inputs with the BASELINE shapes and distributions",
            "config": {"workload": f"{a.config}: {w.description}", "plan": plan_name, "rows_per_rank": (
                rows[1] - rows[0]) if rows else None, "global_rows": total_rows if sharded else None,
                "parallelism": f"rows{world}" if sharded else f"replicas{world}",
                "l2": l2_note, "graph": True},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
            "clocks": clk.summary(), "kernels": per_kernel,
        }
        print(json.dumps(line))
    del prog
    if world > 1:
        dist.destroy_process_group()


# dram read+write bytes per launch of the dominant kernel, from the committed ncu summaries
# (profiles/*.md)
TRAFFIC: dict = {
    ("cfg1", "tj_matmul_1"): 22.1e6,
    ("cfg1", "tj_matmul_2"): 31.5e6,
    ("cfg2", "tj_row_0"): 365.4e6,
    ("cfg3", "tj_matmul_0"): 1068.0e6,
    ("cfg4", "tj_attention_2"): 114.1e6,
}
# cfg5's launches (131072 rows at one GPU, 131072 / N per rank) are too large to capture, so
# its GEMMs were captured on 16384-row programs (profiles/gemm_traffic_cfg5_cfg1.md), once per
# tile kind (single CTA / CTA pair); a launch of M rows moves M / 16384 times those bytes (x, h
# and the per-row-group weight re-reads all grow in proportion to the rows)
CFG5_TRAFFIC_16K: dict = {
    ("tj_matmul_1", False): 1727.9e6,
    ("tj_matmul_2", False): 2822.8e6,
    ("tj_matmul_1", True): 1555.1e6,
    ("tj_matmul_2", True): 3272.9e6,
}


def traffic_per_launch(config: str, ks):
    if config == "cfg5":
        per = CFG5_TRAFFIC_16K.get((ks.symbol, bool(ks.info.get("pair"))))
        return per * ks.info["M"] / 16384 if per is not None and "M" in ks.info else None
    return TRAFFIC.get((config, ks.symbol))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg5", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--rows", type=int, default=None,
                    help="cfg5 only: run a leading slice of this many rows (for small profiling captures)")
    a = ap.parse_args()
    if a.warmup < 3 and a.impl == "b200":
        a.warmup = 3
    if a.impl == "reference":
        run_reference(a)
    else:
        run_b200(a)


if __name__ == "__main__":
    main()
