"""The C ABI library: builds, loads without a GPU, exports every symbol the
header declares, matches the header's struct layouts, and validates its inputs
before touching the driver."""
import ctypes
import re
import subprocess
from pathlib import Path

from mlir_gpu_kernel_compiler_b200 import runtime as rt
from mlir_gpu_kernel_compiler_b200 import toolchain

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "tj_b200.h"


def declared_functions():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"TJ_API\s+[\w\s\*]+?\b(tj_b200_\w+)\s*\(", text)))


def test_library_exports_every_declared_symbol():
    lib_path = toolchain.build_runtime()
    out = subprocess.run(["nm", "-D", "--defined-only", str(lib_path)], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (tj_b200_\w+)", out))
    decl = declared_functions()
    assert decl, "no declarations parsed"
    missing = [d for d in decl if d not in exported]
    assert not missing, missing
    assert set(decl) == set(rt.EXPORTS)
    lib = rt.library()
    for name in decl:
        assert hasattr(lib, name)


def test_struct_layouts_match_header(tmp_path):
    src = tmp_path / "sz.c"
    src.write_text(f'#include "{HEADER}"\n#include <stdio.h>\n#include <stddef.h>\n'
                   "int main(){printf(\"%zu %zu %zu %zu %zu %zu %zu\\n\", sizeof(tj_argref), sizeof(tj_tmap), "
                   "sizeof(tj_launch), sizeof(tj_program_info), offsetof(tj_launch, first_arg), "
                   "offsetof(tj_tmap, param_offset), sizeof(tj_ipc_handle)); return 0;}\n")
    exe = tmp_path / "sz"
    subprocess.run(["gcc", str(src), "-o", str(exe)], check=True)
    vals = [int(x) for x in subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split()]
    assert vals == [ctypes.sizeof(rt.TjArgRef), ctypes.sizeof(rt.TjTMap), ctypes.sizeof(rt.TjLaunch),
                    ctypes.sizeof(rt.TjProgramInfo), rt.TjLaunch.first_arg.offset, rt.TjTMap.param_offset.offset,
                    ctypes.sizeof(rt.TjIpcHandle)]


def test_abi_version_and_errors_without_gpu():
    lib = rt.library()
    assert lib.tj_b200_abi_version() == 1
    out = ctypes.c_void_p()
    # NULL out pointer
    rc = lib.tj_b200_program_create(None, None, 0, None, 0, None, 0, None, 0, 0, 0, 0, 0, None)
    assert rc == rt.TJ_ERR_INVALID and b"out_program" in lib.tj_b200_last_error()
    # argument reference out of range is rejected before the driver is used
    L = (rt.TjLaunch * 1)()
    L[0].symbol = b"k"
    L[0].module = 0
    L[0].block[0] = L[0].block[1] = L[0].block[2] = 1
    L[0].grid[0] = L[0].grid[1] = L[0].grid[2] = 1
    L[0].param_bytes = 8
    L[0].num_args = 1
    A = (rt.TjArgRef * 1)()
    A[0].kind = rt.ARG_INPUT
    A[0].value = 5
    img = ctypes.create_string_buffer(b"\x7fELF" + b"\0" * 60)
    imgs = (ctypes.c_void_p * 1)(ctypes.cast(img, ctypes.c_void_p))
    sizes = (ctypes.c_size_t * 1)(64)
    rc = lib.tj_b200_program_create(imgs, sizes, 1, L, 1, A, 1, None, 0, 0, 1, 1, 0, ctypes.byref(out))
    assert rc == rt.TJ_ERR_INVALID and b"input index out of range" in lib.tj_b200_last_error()
    A[0].kind = rt.ARG_ARENA
    A[0].value = 128
    rc = lib.tj_b200_program_create(imgs, sizes, 1, L, 1, A, 1, None, 0, 64, 1, 1, 0, ctypes.byref(out))
    assert rc == rt.TJ_ERR_INVALID and b"arena offset" in lib.tj_b200_last_error()
    A[0].kind = 9
    rc = lib.tj_b200_program_create(imgs, sizes, 1, L, 1, A, 1, None, 0, 64, 1, 1, 0, ctypes.byref(out))
    assert rc == rt.TJ_ERR_INVALID and b"bad argument kind" in lib.tj_b200_last_error()
    # valid table but no driver in this container -> TJ_ERR_NO_DRIVER (or a CUDA error on a GPU host)
    A[0].kind = rt.ARG_INPUT
    A[0].value = 0
    if not lib.tj_b200_driver_available():
        rc = lib.tj_b200_program_create(imgs, sizes, 1, L, 1, A, 1, None, 0, 0, 1, 1, 0, ctypes.byref(out))
        assert rc == rt.TJ_ERR_NO_DRIVER
    assert lib.tj_b200_run(None, None, None, None) == rt.TJ_ERR_INVALID
    assert lib.tj_b200_destroy(None) == rt.TJ_OK
    # peer-memory entry points: NULL arguments are rejected before the driver is used
    h, off, p = rt.TjIpcHandle(), ctypes.c_uint64(), ctypes.c_void_p()
    assert lib.tj_b200_ipc_export(None, 0, ctypes.byref(h), ctypes.byref(off)) == rt.TJ_ERR_INVALID
    assert lib.tj_b200_ipc_open(None, 0, 0, ctypes.byref(p)) == rt.TJ_ERR_INVALID
    assert lib.tj_b200_ipc_close(None, 0, 0) == rt.TJ_ERR_INVALID
    if not lib.tj_b200_driver_available():
        assert lib.tj_b200_ipc_export(ctypes.c_void_p(1 << 20), 0, ctypes.byref(h), ctypes.byref(off)) in (
            rt.TJ_ERR_NO_DRIVER, rt.TJ_ERR_NOT_SUPPORTED)


def test_tmap_validation():
    lib = rt.library()
    out = ctypes.c_void_p()
    L = (rt.TjLaunch * 1)()
    L[0].symbol = b"k"
    L[0].block[0] = L[0].block[1] = L[0].block[2] = 1
    L[0].grid[0] = L[0].grid[1] = L[0].grid[2] = 1
    L[0].param_bytes = 64 + 128
    L[0].num_args = 1
    L[0].num_tmaps = 1
    A = (rt.TjArgRef * 1)()
    T = (rt.TjTMap * 1)()
    T[0].arg = 0
    T[0].rank = 2
    T[0].param_offset = 32          # not 64-byte aligned
    img = ctypes.create_string_buffer(b"\x7fELF" + b"\0" * 60)
    imgs = (ctypes.c_void_p * 1)(ctypes.cast(img, ctypes.c_void_p))
    sizes = (ctypes.c_size_t * 1)(64)
    rc = lib.tj_b200_program_create(imgs, sizes, 1, L, 1, A, 1, T, 1, 0, 1, 1, 0, ctypes.byref(out))
    assert rc == rt.TJ_ERR_INVALID and b"parameter offset" in lib.tj_b200_last_error()
