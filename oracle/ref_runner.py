"""Runs the reference ``c`` backend's generated kernels (``oracle/_ref``) on the
host cores — BASELINE / TEST INFRASTRUCTURE ONLY (``bench.py``'s reference arm
and CPU-baseline leg).

``oracle/build_ref.py`` wrote ``<name>.c`` (the reference's own generated C/OpenMP
source) and ``<name>.json`` (symbols and INPUT/ARENA/OUTPUT argument references).
This module compiles the source for the current host with the reference's
flags (``tensorjit/backends/c_backend.py:317``) into ``oracle/_ref/<name>.<host>.so``
and runs the kernels in order, each called as ``void kernel_i(void** args)``
like ``csrc/runtime.cpp:88-110`` does, with a 64-byte aligned arena.
"""
from __future__ import annotations

import ctypes
import hashlib
import json
import os
import platform
import shutil
import subprocess
from pathlib import Path

import numpy as np

REF = Path(__file__).resolve().parent / "_ref"


def available(name: str) -> bool:
    return (REF / f"{name}.c").exists() and (REF / f"{name}.json").exists()


def _host_tag() -> str:
    cpu = platform.processor() or ""
    try:
        for line in open("/proc/cpuinfo"):
            if line.startswith("model name"):
                cpu = line.split(":", 1)[1].strip()
                break
    except OSError:
        pass
    return hashlib.sha256(cpu.encode()).hexdigest()[:10]


def set_threads(n: int) -> int:
    """Give the reference kernels' OpenMP runtime ``n`` threads and return the count it then
    reports.  Set explicitly (not only through OMP_NUM_THREADS, which a launcher such as
    torchrun pins to 1 before the process starts): the environment variable is updated for a
    libgomp that is not loaded yet, and ``omp_set_num_threads`` is called on the loaded one."""
    os.environ["OMP_NUM_THREADS"] = str(n)
    try:
        gomp = ctypes.CDLL("libgomp.so.1")
        gomp.omp_set_num_threads(ctypes.c_int(n))
        return int(gomp.omp_get_max_threads())
    except OSError:
        return n


class RefProgram:
    def __init__(self, name: str):
        self.manifest = json.loads((REF / f"{name}.json").read_text())
        src = REF / f"{name}.c"
        so = REF / f"{name}.{_host_tag()}.so"
        if not so.exists() or so.stat().st_mtime < src.stat().st_mtime:
            cc = "/usr/bin/gcc" if Path("/usr/bin/gcc").exists() else (shutil.which("gcc") or "gcc")
            tmp = so.with_suffix(f".{os.getpid()}.tmp")
            cmd = [cc, *self.manifest["flags"], str(src), "-o", str(tmp), "-lm"]
            r = subprocess.run(cmd, capture_output=True, text=True)
            if r.returncode != 0:
                raise RuntimeError(f"reference C build failed: {r.stderr[-2000:]}")
            os.replace(tmp, so)
        self.lib = ctypes.CDLL(str(so))
        self.fns = []
        for s in self.manifest["symbols"]:
            f = getattr(self.lib, s)
            f.argtypes = [ctypes.POINTER(ctypes.c_void_p)]
            f.restype = None
            self.fns.append(f)
        nb = max(int(self.manifest["arena_bytes"]), 64)
        self._arena_raw = np.empty(nb + 64, dtype=np.uint8)
        base = self._arena_raw.ctypes.data
        self.arena = base + (-base) % 64
        self.outputs = [np.empty(s, dtype=np.float32) for s in self.manifest["output_shapes"]]

    def run(self, inputs: list[np.ndarray]) -> list[np.ndarray]:
        ins = [np.ascontiguousarray(x, dtype=np.float32) for x in inputs]
        ip = [x.ctypes.data for x in ins]
        op = [o.ctypes.data for o in self.outputs]
        for fn, args in zip(self.fns, self.manifest["args"]):
            ptrs = (ctypes.c_void_p * max(len(args), 1))()
            for i, (kind, val) in enumerate(args):
                ptrs[i] = ip[val] if kind == 0 else (self.arena + val if kind == 1 else op[val])
            fn(ptrs)
        return [self.outputs[j] for j in self.manifest["graph_outputs"]]
