#!/usr/bin/env python
"""Benchmark of the tensorjit B200 backend on the BASELINE programs.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--config cfg5] [--impl b200|reference]
    torchrun --nproc-per-node N --master-addr 127.0.0.1 bench.py --gpus N ...

Headline workload: cfg5, the large-batch MLP x + linear(gelu(linear(rms_norm(x,g),w1,b1)),w2,b2)
in bf16 with x[131072,4096], w1[16384,4096], w2[4096,16384] — the program the reference's
north star runs at 1/2/4/8 GPUs.  Its rows are split across ranks (rank p owns rows
[p*R/N, (p+1)*R/N), weights replicated, no collective in the step), so the global batch is
fixed: strong scaling.  A step is one execution of the whole compiled program (RMSNorm row
kernel + two tcgen05 GEMMs with fused epilogues) over the rank's rows, as one CUDA graph.
Before the K timed steps every rank runs untimed steps for at least ``--soak-s`` seconds, so
that at every N the GPUs are timed in the same power-capped steady state.

``value``     whole-job algorithmic TFLOP/s with inputs resident in HBM (inputs are larger
              than L2, so no flush is needed between steps).
``e2e``       the same through the C ABI with host buffers: the rank's rows stream in from
              pinned host memory every step and the result streams back, overlapped with
              compute across steps (``HostPipeline``; weights stay resident, as a served
              model's would).  ``e2e_call`` beside it is the per-call latency of the public call
              ``program(*inputs)`` with the copies in sequence.
``roofline``  the dominant kernel's achieved rate from CUDA events around each kernel,
              against MEASURED_PEAKS.json.
``cpu_baseline`` the reference's own ``c`` backend (its generated C/OpenMP kernels, built for
              this host by oracle/ref_runner.py) on a bounded row sample, every host core.
``gather``    (N > 1) the optional NCCL all-gather of y to every rank, timed on its own, and
              ``gather.rows_on_root``: the step whose down projection stores its rows straight
              into rank 0's y over NVLink (no collective), timed in alternation with the
              ordinary step.
``configs``   (N = 1) cfg1-cfg4 measured the same way in the same run: program latency (graph
              replay), the dominant kernel's roofline, the reference baseline and clocks.

``--impl reference`` times that reference implementation alone, on the same metric, and
prints its own line (rank 0 only under torchrun).
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
# reference sample per config: (oracle/_ref program, rows of the row-sharded arguments or None = all)
REF_SAMPLE = {"cfg1": ("cfg1", None), "cfg2": ("cfg2", None), "cfg3": ("cfg3_m512", 512), "cfg4": ("cfg4", None),
              "cfg5": ("cfg5_m1024", 1024)}
SIDE_CONFIGS = ("cfg1", "cfg2", "cfg3", "cfg4")

L2_BYTES = 126 * 1024 * 1024  # B200 L2


def host_cores() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:  # pragma: no cover
        return os.cpu_count() or 1


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


# ---------------------------------------------------------------------------------------------
# the reference c backend on the host cores
# ---------------------------------------------------------------------------------------------
def reference_baseline(cfg: str, steps: int, warmup: int) -> dict | None:
    """Time the reference c backend's kernels on a bounded sample with every host core;
    None if its kernels were not prepared (oracle/_ref)."""
    import numpy as np

    from mlir_gpu_kernel_compiler_b200 import workloads as W
    from oracle import ref_runner

    name, rows = REF_SAMPLE[cfg]
    if not ref_runner.available(name):
        return None
    threads = ref_runner.set_threads(host_cores())
    w = W.WORKLOADS[cfg]
    ins = [t.float().numpy() for t in W.make_inputs(w, rows=(0, rows) if rows else None)]
    prog = ref_runner.RefProgram(name)
    for _ in range(max(warmup, 1)):
        prog.run(ins)
    ts = []
    for _ in range(max(steps, 1)):
        t0 = time.perf_counter()
        prog.run(ins)
        ts.append(time.perf_counter() - t0)
    sec = float(np.median(ts))
    frac = (rows / w.rows) if rows else 1.0
    work = (w.flops or w.hbm_bytes) * frac
    unit_scale = 1e12 if w.flops else 1e9
    out = {"value": work / sec / unit_scale, "unit": "TFLOP/s" if w.flops else "GB/s", "cores": threads,
           "kind": "reference",
           "sample": f"{name}: reference c backend (generated C/OpenMP, -O3 -march=native -fopenmp) on "
                     f"{rows or 'all'} rows, {threads} OpenMP threads, median of {len(ts)} runs, "
                     f"{sec * 1e3:.1f} ms per sample",
           "ms_per_sample": sec * 1e3}
    if rows:
        # rows are independent: the rate of a row slice is the rate of the whole program
        out.update(extrapolated=True, sample_rows=rows, program_rows=w.rows)
    return out


def run_reference(a) -> None:
    world, rank, _ = _dist()
    if rank != 0:
        return
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
    if res.get("extrapolated"):
        line["cpu_baseline"].update(extrapolated=True, sample_rows=res["sample_rows"])
    print(json.dumps(line))


# ---------------------------------------------------------------------------------------------
# DRAM traffic of the dominant kernels, from ncu captures (dram__bytes_read.sum + write.sum)
# ---------------------------------------------------------------------------------------------
# Keyed by (config, kernel symbol, tile signature); a run whose kernel has another signature (a
# different tile table) reports no traffic rather than a stale figure.  cfg5's launches are too
# large to capture, so its GEMMs were captured on 16384-row programs; a launch of M rows moves
# M / 16384 times those bytes (x, h and the per-row-group weight re-reads grow with the rows).
TRAFFIC: dict = {
    ("cfg1", "tj_matmul_1", "x3:BN128"): (22.1e6, None),
    ("cfg1", "tj_matmul_2", "x3:BN128"): (31.5e6, None),
    ("cfg2", "tj_row_0", "row"): (365.4e6, None),
    ("cfg3", "tj_matmul_0", "pair:BN256"): (1068.0e6, None),
    ("cfg4", "tj_attention_2", "attention"): (114.1e6, None),
    ("cfg5", "tj_matmul_1", "single:BN256"): (1727.9e6, 16384),
    ("cfg5", "tj_matmul_2", "single:BN256"): (2822.8e6, 16384),
    ("cfg5", "tj_matmul_1", "pair:BN256"): (1555.1e6, 16384),
    ("cfg5", "tj_matmul_2", "pair:BN256"): (3272.9e6, 16384),
}


def tile_signature(ks) -> str:
    if ks.family == "gemm_tc":
        kind = "x3" if ks.info.get("tf32x3") else ("pair" if ks.info.get("pair") else "single")
        return f"{kind}:BN{ks.info.get('BN')}"
    return ks.family


def traffic_per_launch(config: str, ks) -> tuple[float | None, str]:
    ent = TRAFFIC.get((config, ks.symbol, tile_signature(ks)))
    if ent is None:
        return None, f"no ncu capture of {ks.symbol} with tile {tile_signature(ks)}"
    per, rows = ent
    if rows is None:
        return per, f"ncu capture of this launch ({tile_signature(ks)})"
    return per * ks.info["M"] / rows, f"ncu capture at {rows} rows ({tile_signature(ks)}), scaled by M / {rows}"


# ---------------------------------------------------------------------------------------------
# one program, device-resident inputs
# ---------------------------------------------------------------------------------------------
def roofline_of(cfg: str, prog, kms: list[float], sustained: bool) -> tuple[dict, list[dict]]:
    pk = peaks()
    dom = max(range(len(kms)), key=lambda i: kms[i])
    ks = prog.kernel_sources[dom]
    of = ", of measured" if pk["source"] == "measured" else ", of fallback"
    if _tensor_family(ks.family):
        ach = ks.info["flops"] / (kms[dom] * 1e-3) / 1e12
        peak = pk["bf16_tflops_sustained"] if sustained else pk["bf16_tflops"]
        kind = ("sustained" if sustained else "burst") + " bf16"
        if ks.info.get("tf32x3"):
            # f32 GEMM on the TF32 tensor path: half the bf16 rate, three MMAs per product
            peak, kind = peak / 6.0, kind + " / 2 (TF32 rate) / 3 (3xTF32 products)"
        roof = {"bound": "tensor", "achieved": ach, "peak": peak, "unit": "TFLOP/s", "frac": ach / peak,
                "kernel": ks.symbol, "ms": kms[dom], "peak_kind": kind + of}
    else:
        ach = ks.info["bytes"] / (kms[dom] * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": ach, "peak": pk["hbm_gbs"], "unit": "GB/s", "frac": ach / pk["hbm_gbs"],
                "kernel": ks.symbol, "ms": kms[dom], "peak_kind": "copy bandwidth" + of}
    roof["traffic"], roof["traffic_source"] = traffic_per_launch(cfg, ks)
    roof["tile"] = tile_signature(ks)
    per_kernel = [{"kernel": k.symbol, "family": k.family, "ms": round(m, 4),
                   "rate": round((k.info["flops"] / (m * 1e-3) / 1e12) if _tensor_family(k.family)
                                 else (k.info["bytes"] / (m * 1e-3) / 1e9), 1) if m > 0 else None,
                   "rate_unit": "TFLOP/s" if _tensor_family(k.family) else "GB/s"}
                  for k, m in zip(prog.kernel_sources, kms)]
    return roof, per_kernel


def time_program(prog, ins, outs, steps: int, warmup: int, soak_s: float, dev, barrier) -> dict:
    """Warm up, soak (untimed steps for soak_s seconds), then time exactly ``steps`` graph
    replays with CUDA events on the launching stream.  A program whose inputs, outputs and
    intermediates fit in L2 is timed step by step with L2 flushed before each step by a write
    of twice its size, outside the events."""
    import torch

    stream = torch.cuda.current_stream(dev)
    for _ in range(warmup):
        prog.run_into(ins, outs)
    torch.cuda.synchronize(dev)
    prog.check()
    footprint = sum(t.numel() * t.element_size() for t in ins + outs) + prog.arena_bytes
    flush = torch.empty(2 * L2_BYTES // 4, dtype=torch.float32, device=dev) if footprint < L2_BYTES else None
    soaked = 0
    if soak_s > 0:
        t0 = time.perf_counter()
        while time.perf_counter() - t0 < soak_s:
            for _ in range(8):
                if flush is not None:
                    flush.fill_(1.0)
                prog.run_into(ins, outs)
                soaked += 1
            torch.cuda.synchronize(dev)
    barrier()
    torch.cuda.synchronize(dev)
    clk = Clocks(dev.index or 0)
    with clk:
        if flush is None:
            start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            start.record(stream)
            for _ in range(steps):
                prog.run_into(ins, outs)
            end.record(stream)
            torch.cuda.synchronize(dev)
            ms = start.elapsed_time(end) / steps
        else:
            evs = [(torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)) for _ in range(steps)]
            for s0, s1 in evs:
                flush.fill_(1.0)
                s0.record(stream)
                prog.run_into(ins, outs)
                s1.record(stream)
            torch.cuda.synchronize(dev)
            ms = sum(s0.elapsed_time(s1) for s0, s1 in evs) / steps
    l2 = ("inputs, outputs and intermediates of a step exceed L2 (no flush needed)" if flush is None
          else f"L2 flushed before every timed step ({2 * L2_BYTES >> 20} MiB write, outside the events)")
    return {"ms": ms, "clocks": clk.summary(), "l2": l2, "soak_steps": soaked, "soak_s": soak_s if soaked else 0.0}


def e2e_call(prog, host_ins: list, stream_idx: list[int], resident: dict, calls: int, dev) -> dict:
    """Per-call latency of the public call with host data: copy the streamed inputs from
    pinned host memory, ``program(*inputs)``, copy the outputs back; in sequence, one call at a
    time (CUDA events on the current stream around the whole call)."""
    import torch

    stream = torch.cuda.current_stream(dev)
    d_in = {i: torch.empty_like(host_ins[i], device=dev) for i in stream_idx}
    host_out = None
    h2d = sum(host_ins[i].numel() * host_ins[i].element_size() for i in stream_idx)

    def one():
        nonlocal host_out
        for i in stream_idx:
            d_in[i].copy_(host_ins[i], non_blocking=True)
        ins = [d_in[i] if i in d_in else resident[i] for i in range(len(host_ins))]
        outs = prog(*ins)
        if host_out is None:
            host_out = [torch.empty(o.shape, dtype=o.dtype).pin_memory() for o in outs]
        for h, o in zip(host_out, outs):
            h.copy_(o, non_blocking=True)

    one()
    torch.cuda.synchronize(dev)
    ts = []
    for _ in range(calls):
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s0.record(stream)
        one()
        s1.record(stream)
        torch.cuda.synchronize(dev)
        ts.append(s0.elapsed_time(s1))
    ts.sort()
    d2h = sum(h.numel() * h.element_size() for h in host_out)
    return {"ms_per_call": ts[len(ts) // 2], "calls": calls, "h2d_bytes_per_call": h2d, "d2h_bytes_per_call": d2h,
            "how": "program(*inputs) with the streamed inputs copied from pinned host memory and the outputs "
                   "copied back, in sequence (median call)"}


def measure_side_config(cfg: str, a, dev) -> dict:
    """cfg1-cfg4 on one GPU: program latency (graph replay), dominant-kernel roofline, per-call
    latency with host data, the reference c backend on the host cores, clocks."""
    import torch

    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200 import workloads as W
    from mlir_gpu_kernel_compiler_b200.plan import PProgram

    w = W.WORKLOADS[cfg]
    plan = PProgram.load(ROOT / "tests" / "golden" / "plans" / f"{w.plan}.json")
    host = W.make_inputs(w)
    ins = [t.to(dev) for t in host]
    prog = B200Program(plan, device=dev, use_graph=True)
    outs = [torch.empty(s, dtype=d, device=dev) for s, d in prog.output_specs()]
    t = time_program(prog, ins, outs, a.steps, a.warmup, 0.0, dev, lambda: None)
    ms = t["ms"]
    work = w.flops or w.hbm_bytes
    unit_scale, unit = (1e12, "TFLOP/s") if w.flops else (1e9, "GB/s")
    kms = prog.time_kernels(ins, outs, iters=max(3, min(a.steps, 10)))
    roof, per_kernel = roofline_of(cfg, prog, kms, sustained=False)
    rec = {"workload": f"{cfg}: {w.description}", "plan": w.plan, "value": work / (ms * 1e-3) / unit_scale,
           "unit": unit, "ms_per_step": ms, "steps": a.steps, "warmup": a.warmup, "l2": t["l2"], "graph": True,
           "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32", "roofline": roof, "kernels": per_kernel,
           "clocks": t["clocks"],
           "gpu_launches": sum(1 for L in prog.launches if all(g > 0 for g in L["grid"])) * a.steps}
    if not a.no_e2e:
        pinned = [h.pin_memory() for h in host]
        stream_idx = list(w.row_args) or list(range(len(host)))
        resident = {i: x for i, x in enumerate(ins) if i not in stream_idx}
        c = e2e_call(prog, pinned, stream_idx, resident, max(3, min(a.steps, 10)), dev)
        c["value"] = work / (c["ms_per_call"] * 1e-3) / unit_scale
        c["unit"] = unit
        rec["e2e_call"] = c
    prog.check()
    prog.close()
    del ins, outs, host
    torch.cuda.empty_cache()
    if not a.no_cpu_baseline:
        try:
            rec["cpu_baseline"] = reference_baseline(cfg, steps=3, warmup=1)
        except Exception as ex:  # the baseline is reported, never required
            rec["cpu_baseline"] = {"error": str(ex)[:200]}
    return rec


def rows_on_root_step(plan, prog, ins, outs, total_rows: int, steps: int, dev, barrier) -> dict:
    """The step with its output gathered on rank 0 without a collective: every rank's program
    (built with staged plain-store epilogues) is launched with its rows of rank 0's full-size y as the
    output, a CUDA IPC mapping on the other ranks, so the down projection's epilogue stores its
    tiles into rank 0's HBM over NVLink while the GEMM runs.  Timed in alternation with the
    ordinary step (local y), three rounds each (events, barrier + synchronize on both sides,
    max over ranks, median round); then rank 0 checks that every rank's rows equal what that
    rank's ordinary program stored locally."""
    import torch
    import torch.distributed as dist

    from mlir_gpu_kernel_compiler_b200 import B200Program
    from mlir_gpu_kernel_compiler_b200.distributed import RowsOnRoot

    world, rank = dist.get_world_size(), dist.get_rank()
    y_local = outs[0]
    peer = B200Program(plan, device=dev, use_graph=True, peer_outputs=True)
    try:
        target = RowsOnRoot((total_rows,) + tuple(y_local.shape[1:]), y_local.dtype, dev)
    except RuntimeError:
        peer.close()
        raise

    def timed(fn) -> float:
        torch.cuda.synchronize(dev)
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        for _ in range(steps):
            fn()
        e1.record()
        torch.cuda.synchronize(dev)
        barrier()
        ms = torch.tensor([e0.elapsed_time(e1) / steps], device=dev)
        dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    try:
        for _ in range(3):
            peer.run_into(ins, [target.dest])
        local_ms, peer_ms = [], []
        for _ in range(3):
            local_ms.append(timed(lambda: prog.run_into(ins, outs)))
            peer_ms.append(timed(lambda: peer.run_into(ins, [target.dest])))
        peer.check()
        # each rank's local rows, as its ordinary program stored them, against rank 0's copy
        sums = torch.zeros(world, 2, dtype=torch.float64, device=dev)
        sums[rank, 0] = y_local.double().sum()
        sums[rank, 1] = y_local.double().abs().sum()
        dist.all_reduce(sums)
        same = torch.zeros(1, device=dev)
        if rank == 0:
            parts = target.full.chunk(world, dim=0)
            ok = bool(torch.equal(parts[0], y_local))
            for r in range(world):
                ok &= bool(parts[r].double().sum() == sums[r, 0]) and bool(parts[r].double().abs().sum() == sums[r, 1])
            same[0] = float(ok)
        dist.broadcast(same, src=0)
        nbytes = total_rows * y_local[0].numel() * y_local.element_size()
        return {"ms_per_step": sorted(peer_ms)[1], "local_step_ms": sorted(local_ms)[1],
                "rounds_ms": {"local": local_ms, "rows_on_root": peer_ms},
                "bytes_to_rank0": nbytes * (world - 1) // world, "rows_identical": bool(same.item()),
                "how": "step whose last GEMM stores its rows into rank 0's y over NVLink (CUDA IPC mapping, "
                       f"staged plain-store epilogue), alternating with the ordinary step, 3 rounds x {steps} steps, "
                       "max over ranks, median round; rows_identical: rank 0's copy of every rank's rows has "
                       "the checksums of that rank's locally stored y (rank 0's: bit for bit)"}
    finally:
        target.close()
        peer.close()


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

    def barrier():
        if world > 1:
            dist.barrier(device_ids=[local])

    t = time_program(prog, ins, outs, a.steps, a.warmup, a.soak_s, dev, barrier)
    barrier()
    ms_t = torch.tensor([t["ms"]], device=dev)
    if world > 1:
        dist.all_reduce(ms_t, op=dist.ReduceOp.MAX)
    ms_max = float(ms_t.item())
    frac_rows = ((rows[1] - rows[0]) * world / w.rows) if sharded else world
    total_work = (w.flops or w.hbm_bytes) * frac_rows
    unit_scale, unit = (1e12, "TFLOP/s") if w.flops else (1e9, "GB/s")
    value = total_work / (ms_max * 1e-3) / unit_scale
    clocks_all = [t["clocks"]]
    if world > 1:
        clocks_all = [None] * world
        dist.all_gather_object(clocks_all, t["clocks"])

    # per-kernel device times (events around every kernel, same stream) -> dominant kernel roofline
    kms = prog.time_kernels(ins, outs, iters=max(3, min(a.steps, 10)))
    roof, per_kernel = roofline_of(a.config, prog, kms, sustained=a.soak_s > 0 or a.config in ("cfg4", "cfg5"))

    # the optional all-gather of y to every rank (N > 1), outside the compute step
    gather = None
    if world > 1 and sharded and not a.no_gather:
        from mlir_gpu_kernel_compiler_b200.distributed import gather_rows

        y = outs[0]
        for _ in range(2):
            gather_rows(y)
        torch.cuda.synchronize(dev)
        barrier()
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        reps = 5
        g0.record()
        for _ in range(reps):
            full = gather_rows(y)
        g1.record()
        torch.cuda.synchronize(dev)
        gms = torch.tensor([g0.elapsed_time(g1) / reps], device=dev)
        dist.all_reduce(gms, op=dist.ReduceOp.MAX)
        gms = float(gms.item())
        total_bytes = full.numel() * full.element_size()
        gather = {"ms": gms, "bytes_gathered": total_bytes,
                  "algbw_gbs": total_bytes / (gms * 1e-3) / 1e9,
                  "busbw_gbs": total_bytes * (world - 1) / world / (gms * 1e-3) / 1e9,
                  "how": "NCCL all_gather_into_tensor of every rank's y rows (bf16) to every rank, mean of "
                         f"{reps}, max over ranks; busbw = bytes x (N-1)/N / time, the bytes each GPU receives"}
        del full
        try:
            ror = rows_on_root_step(plan, prog, ins, outs, total_rows, a.steps, dev, barrier)
            ror["local_step_then_nccl_gather_ms"] = ror["local_step_ms"] + gms
        except RuntimeError as ex:   # raised on every rank together (RowsOnRoot set-up)
            ror = {"error": str(ex)[:300]}
        gather["rows_on_root"] = ror

    # end to end through the C ABI with host data every step: HostPipeline streams the row
    # inputs in from pinned host memory and the result out, overlapping both copy directions
    # with compute across consecutive steps (weights stay resident)
    e2e, e2e_c = None, None
    if not a.no_e2e:
        from mlir_gpu_kernel_compiler_b200.pipeline import HostPipeline

        stream_idx = list(w.row_args) or list(range(len(ins)))
        resident = {i: x for i, x in enumerate(ins) if i not in stream_idx}
        host_in = {i: ins[i].cpu().pin_memory() for i in stream_idx}
        host_out = [[torch.empty(s, dtype=d).pin_memory() for s, d in prog.output_specs()] for _ in range(2)]
        h2d = sum(x.numel() * x.element_size() for x in host_in.values())
        d2h = sum(x.numel() * x.element_size() for x in host_out[0])
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
        del pipe
        # per-call latency of the public call with host data, copies in sequence
        host_full = [ins[i].cpu().pin_memory() if i in stream_idx else ins[i] for i in range(len(ins))]
        barrier()
        e2e_c = e2e_call(prog, host_full, stream_idx, resident, max(3, min(a.steps, 5)), dev)
        ct = torch.tensor([e2e_c["ms_per_call"]], device=dev)
        if world > 1:
            dist.all_reduce(ct, op=dist.ReduceOp.MAX)
        e2e_c["ms_per_call"] = float(ct.item())
        e2e_c["value"] = total_work / (e2e_c["ms_per_call"] * 1e-3) / unit_scale
        e2e_c["unit"] = unit
        del host_full, host_in, host_out
    prog.check()
    launches = sum(1 for L in prog.launches if all(g > 0 for g in L["grid"])) * a.steps
    prog.close()
    del ins, outs
    torch.cuda.empty_cache()

    # cfg1-cfg4 in the same run (one GPU; rank 0 of a 1-GPU run)
    configs = None
    if world == 1 and a.side_configs:
        configs = {}
        for c in [x for x in a.side_configs.split(",") if x and x != a.config]:
            _trace("side config", c)
            try:
                configs[c] = measure_side_config(c, a, dev)
            except Exception as ex:  # a side record must not take the headline line with it
                configs[c] = {"error": f"{type(ex).__name__}: {str(ex)[:300]}"}

    cpu = None
    if rank == 0 and not a.no_cpu_baseline:
        try:
            cpu = reference_baseline(a.config, steps=3, warmup=1)
        except Exception as ex:  # the baseline is reported, never required
            cpu = {"error": str(ex)[:200]}
    barrier()
    if rank == 0:
        line = {
            "metric": METRIC, "value": value, "unit": unit, "n_gpus": world, "steps": a.steps, "warmup": a.warmup,
            "ms_per_step": ms_max, "higher_is_better": True, "scaling": "strong" if sharded else "weak",
            "vs_baseline": None, "dtype": "bf16" if w.dtype == torch.bfloat16 else "f32",
            "data": "synthetic: seeded CPU-generator inputs with the BASELINE shapes and distributions",
            "config": {"workload": f"{a.config}: {w.description}", "plan": plan_name, "rows_per_rank": (
                rows[1] - rows[0]) if rows else None, "global_rows": total_rows if sharded else None,
                "parallelism": f"rows{world}" if sharded else f"replicas{world}",
                "l2": t["l2"], "graph": True, "soak_s": t["soak_s"], "soak_steps_rank0": t["soak_steps"]},
            "roofline": roof, "cpu_baseline": cpu, "e2e": e2e, "e2e_call": e2e_c, "gpu_launches": launches,
            "clocks": t["clocks"], "kernels": per_kernel,
        }
        if world > 1:
            line["clocks_per_rank"] = clocks_all
            line["gather"] = gather
        if configs is not None:
            line["configs"] = configs
        print(json.dumps(line))
    if world > 1:
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--config", default="cfg5", choices=["cfg1", "cfg2", "cfg3", "cfg4", "cfg5"])
    ap.add_argument("--impl", default="b200", choices=["b200", "reference"])
    ap.add_argument("--soak-s", type=float, default=2.0,
                    help="untimed steps for this many seconds before the timed steps (power-capped steady state)")
    ap.add_argument("--side-configs", default=",".join(SIDE_CONFIGS),
                    help="1-GPU runs: also measure these configs into the line's 'configs' record ('' = none)")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-gather", action="store_true")
    ap.add_argument("--rows", type=int, default=None,
                    help="cfg5 only: run a leading slice of this many rows (for small profiling captures)")
    a = ap.parse_args()
    if a.warmup < 3 and a.impl == "b200":
        a.warmup = 3
    if a.config != "cfg5" and a.side_configs == ",".join(SIDE_CONFIGS):
        a.side_configs = ""          # a single-config run measures that config only
    if a.impl == "reference":
        run_reference(a)
    else:
        run_b200(a)


if __name__ == "__main__":
    main()
