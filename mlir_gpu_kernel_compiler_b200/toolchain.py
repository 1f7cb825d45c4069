"""Build steps: the C++ runtime library and the per-kernel sm_100a cubins.

* ``runtime_library()`` — ``libtj_b200.so`` (the C ABI of ``include/tj_b200.h``),
  built in-tree with g++ from ``csrc/tj_b200_runtime.cpp``.  It links no CUDA
  library; libcuda is opened at run time.
* ``compile_cubins(sources)`` — nvcc ``-gencode arch=compute_100a,code=sm_100a``
  per kernel translation unit, in parallel, cached on disk by a hash of the
  source, the kernel headers, the flags and the nvcc version (the reference
  caches NVRTC output by content hash the same way, ``cuda_backend.py:470-479``).

Cache root: ``$TENSORJIT_B200_CACHE_DIR``, else ``<repo>/_build/cubin`` (in-tree so a
warmed cache travels with the checkout), else ``~/.cache/tensorjit_b200``.
"""
from __future__ import annotations

import hashlib
import os
import shutil
import subprocess
import tempfile
import threading
from concurrent.futures import ThreadPoolExecutor
from functools import lru_cache
from pathlib import Path

PKG = Path(__file__).resolve().parent
REPO = PKG.parent
CSRC = PKG / "csrc"
KDIR = CSRC / "kernels"
INCLUDE = REPO / "include"
LIB_PATH = PKG / "_lib" / "libtj_b200.so"
ARCH_FLAGS = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "--expt-relaxed-constexpr", "-Xptxas=-warn-spills"]

# the failure-path test build: the GEMM producers skip their first stage and every bounded
# wait gives up after 20 ms, so the timeout reporting can be tested without a GPU fault
STALL_TEST_FLAGS = ("-DTJ_TEST_STALL_FIRST_LOAD", "-DTJ_WAIT_NS=20000000ull")

# the checked kernel build (every global access and TMA coordinate bounds-checked on the device)
CHECKED_FLAGS = ("-DTJ_CHECKED",)

_lock = threading.Lock()


class BuildError(RuntimeError):
    pass


def cuda_home() -> Path:
    return Path(os.environ.get("CUDA_HOME") or os.environ.get("CUDA_PATH") or "/usr/local/cuda")


def nvcc() -> str:
    p = cuda_home() / "bin" / "nvcc"
    if p.exists():
        return str(p)
    w = shutil.which("nvcc")
    if not w:
        raise BuildError("nvcc not found (set CUDA_HOME)")
    return w


@lru_cache(maxsize=None)
def nvcc_version() -> str:
    """nvcc's version line for the cache key.  It is remembered in the cache
    directory per nvcc binary (size, mtime), so a cache hit spawns no process:
    a process under a profiler should not start tool subprocesses."""
    exe = Path(nvcc())
    st = exe.stat()
    stamp = cache_dir() / f"nvcc_version.{st.st_size}.{int(st.st_mtime)}.txt"
    try:
        v = stamp.read_text().strip()
        if v:
            return v
    except OSError:
        pass
    r = subprocess.run([str(exe), "--version"], capture_output=True, text=True)
    v = r.stdout.strip().splitlines()[-1] if r.returncode == 0 else "unknown"
    try:
        stamp.write_text(v + "\n")
    except OSError:
        pass
    return v


def cache_dir() -> Path:
    env = os.environ.get("TENSORJIT_B200_CACHE_DIR", "")
    return _cache_dir(env)


@lru_cache(maxsize=None)
def _cache_dir(env: str) -> Path:
    cands = [Path(env)] if env else [REPO / "_build" / "cubin", Path.home() / ".cache" / "tensorjit_b200"]
    for d in cands:
        try:
            d.mkdir(parents=True, exist_ok=True)
            probe = d / f".w{os.getpid()}.{threading.get_ident()}"
            probe.write_text("")
            probe.unlink()
            return d
        except OSError:
            continue
    raise BuildError("no writable cubin cache directory")


@lru_cache(maxsize=None)
def _headers_hash() -> str:
    h = hashlib.sha256()
    for f in sorted(KDIR.glob("*.cuh")):
        h.update(f.name.encode())
        h.update(f.read_bytes())
    return h.hexdigest()


def source_key(source: str, extra_flags: tuple = ()) -> str:
    h = hashlib.sha256()
    for part in (source, _headers_hash(), " ".join(ARCH_FLAGS + NVCC_FLAGS + list(extra_flags)), nvcc_version(), "v1"):
        h.update(part.encode())
        h.update(b"\0")
    return h.hexdigest()[:24]


def compile_cubin(source: str, name: str = "kernel", extra_flags: tuple = ()) -> bytes:
    key = source_key(source, extra_flags)
    d = cache_dir()
    out = d / f"{key}.cubin"
    if os.environ.get("TJ_TRACE") == "1":
        import sys

        print(f"[b200] cubin {name} {key} cached={out.exists()}", file=sys.stderr, flush=True)
    if out.exists():
        try:
            data = out.read_bytes()
            if len(data) > 64 and data[:4] == b"\x7fELF":
                return data
        except OSError:
            pass
        out.unlink(missing_ok=True)          # corrupt cache entry: rebuild
    with tempfile.TemporaryDirectory(prefix="tjb200_") as td:
        src = Path(td) / f"{name}.cu"
        src.write_text(source)
        tmp = Path(td) / "k.cubin"
        cmd = [nvcc(), "-cubin", *ARCH_FLAGS, *NVCC_FLAGS, *extra_flags, f"-I{KDIR}", "-o", str(tmp), str(src)]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise BuildError(f"nvcc failed for {name}:\n{r.stderr[-4000:]}\n--- source ---\n{source[:6000]}")
        data = tmp.read_bytes()
        part = d / f"{key}.{os.getpid()}.{threading.get_ident()}.tmp"
        part.write_bytes(data)
        os.replace(part, out)
        (d / f"{key}.cu").write_text(source)
    return data


def compile_cubins(sources: list[tuple[str, str]], extra_flags: tuple = ()) -> list[bytes]:
    """Compile ``[(name, source), ...]`` in parallel; returns the cubin images in order."""
    if not sources:
        return []
    unique: dict[str, str] = {}            # each distinct source is compiled once
    for n, s in sources:
        unique.setdefault(s, n)
    workers = max(1, min(len(unique), os.cpu_count() or 4, 16))
    if workers == 1:
        done = {s: compile_cubin(s, n, extra_flags) for s, n in unique.items()}
    else:
        with ThreadPoolExecutor(max_workers=workers) as ex:
            futs = {s: ex.submit(compile_cubin, s, n, extra_flags) for s, n in unique.items()}
            done = {s: f.result() for s, f in futs.items()}
    return [done[s] for _, s in sources]


def build_runtime(force: bool = False, extra_flags: tuple = (), variant: str = "") -> Path:
    """Compile ``libtj_b200.so`` in-tree: the driver-API runtime (host C++; libcuda is opened
    at run time) plus the allocation-free linear entry point (``tj_b200_noalloc.cu``, sm_100a,
    static CUDA runtime).  The library loads on machines without a GPU.  ``variant`` names a
    separately built copy with ``extra_flags`` (``libtj_b200_<variant>.so``; e.g. the
    failure-path test build); the product library is the one without."""
    with _lock:
        src = CSRC / "tj_b200_runtime.cpp"
        na = CSRC / "tj_b200_noalloc.cu"
        hdr = INCLUDE / "tj_b200.h"
        out = LIB_PATH if not variant else LIB_PATH.with_name(f"libtj_b200_{variant}.so")
        stamp = out.with_suffix(".hash")
        h = hashlib.sha256(src.read_bytes() + na.read_bytes() + hdr.read_bytes() + _headers_hash().encode()
                           + " ".join(extra_flags).encode()).hexdigest()
        if not force and out.exists() and stamp.exists() and stamp.read_text() == h:
            return out
        out.parent.mkdir(parents=True, exist_ok=True)
        tmp = out.with_suffix(f".{os.getpid()}.tmp")
        cmd = [nvcc(), "-O2", "-std=c++17", "-shared", *ARCH_FLAGS, "-Xcompiler", "-fPIC,-fvisibility=hidden,-Wall",
               "--expt-relaxed-constexpr", *extra_flags, f"-I{INCLUDE}", f"-I{KDIR}", str(src), str(na), "-o",
               str(tmp), "-ldl", "-lpthread"]
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise BuildError(f"runtime build failed:\n{r.stderr[-4000:]}")
        os.replace(tmp, out)
        stamp.write_text(h)
        return out
