"""ctypes binding of the C ABI in ``include/tj_b200.h`` (``libtj_b200.so``).

The structures below mirror the header field for field; ``tests/test_abi.py``
checks their sizes and every exported symbol.
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path

from . import toolchain

TJ_OK = 0
TJ_ERR_INVALID = -1
TJ_ERR_CUDA = -2
TJ_ERR_NO_DRIVER = -3
TJ_ERR_DEVICE_STATUS = -4
TJ_ERR_NOT_SUPPORTED = -5

ARG_INPUT, ARG_ARENA, ARG_OUTPUT, ARG_STATUS = 0, 1, 2, 3

EXPORTS = (
    "tj_b200_program_create", "tj_b200_run", "tj_b200_set_graph", "tj_b200_check_status",
    "tj_b200_program_info", "tj_b200_destroy", "tj_b200_last_error", "tj_b200_abi_version",
    "tj_b200_driver_available", "tj_b200_time_kernels", "tj_b200_linear_f32_noalloc",
    "tj_b200_linear_f32_noalloc_status", "tj_b200_ipc_export", "tj_b200_ipc_open", "tj_b200_ipc_close",
    "tj_b200_set_pdl",
)


class TjArgRef(ctypes.Structure):
    _fields_ = [("kind", ctypes.c_int32), ("reserved", ctypes.c_int32), ("value", ctypes.c_int64)]


class TjTMap(ctypes.Structure):
    _fields_ = [
        ("arg", ctypes.c_int32), ("dtype", ctypes.c_int32), ("rank", ctypes.c_int32), ("swizzle", ctypes.c_int32),
        ("dims", ctypes.c_uint64 * 5), ("strides", ctypes.c_uint64 * 4), ("box", ctypes.c_uint32 * 5),
        ("param_offset", ctypes.c_uint32), ("l2_promotion", ctypes.c_int32), ("reserved", ctypes.c_int32),
    ]


class TjLaunch(ctypes.Structure):
    _fields_ = [
        ("symbol", ctypes.c_char_p), ("module", ctypes.c_int32),
        ("grid", ctypes.c_uint32 * 3), ("block", ctypes.c_uint32 * 3), ("cluster", ctypes.c_uint32 * 3),
        ("smem_bytes", ctypes.c_uint32), ("param_bytes", ctypes.c_uint32),
        ("first_arg", ctypes.c_int32), ("num_args", ctypes.c_int32),
        ("first_tmap", ctypes.c_int32), ("num_tmaps", ctypes.c_int32),
    ]


class TjIpcHandle(ctypes.Structure):
    _fields_ = [("bytes", ctypes.c_ubyte * 64)]


class TjProgramInfo(ctypes.Structure):
    _fields_ = [
        ("arena", ctypes.c_void_p), ("arena_bytes", ctypes.c_uint64), ("num_kernels", ctypes.c_int32),
        ("num_inputs", ctypes.c_int32), ("num_outputs", ctypes.c_int32), ("graph_enabled", ctypes.c_int32),
        ("calls", ctypes.c_uint64), ("launches", ctypes.c_uint64), ("graph_replays", ctypes.c_uint64),
        ("graph_node_updates", ctypes.c_uint64), ("graph_instantiations", ctypes.c_uint64),
        ("host_us_total", ctypes.c_double),
    ]


class RuntimeError_(RuntimeError):
    """A failure reported by the B200 runtime (driver error, bad launch table, device status)."""

    def __init__(self, code: int, msg: str):
        super().__init__(f"tj_b200 error {code}: {msg}")
        self.code = code


CudaError = RuntimeError_

_lib = None
_lib_lock = threading.Lock()


def library(path: str | Path | None = None) -> ctypes.CDLL:
    """Load ``libtj_b200.so`` (building it in-tree first if it is missing)."""
    global _lib
    with _lib_lock:
        if _lib is not None and path is None:
            return _lib
        p = Path(path) if path else toolchain.build_runtime()
        lib = ctypes.CDLL(str(p))
        vp, i32, u64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_uint64
        lib.tj_b200_program_create.argtypes = [
            ctypes.POINTER(vp), ctypes.POINTER(ctypes.c_size_t), i32, ctypes.POINTER(TjLaunch), i32,
            ctypes.POINTER(TjArgRef), i32, ctypes.POINTER(TjTMap), i32, u64, i32, i32, i32, ctypes.POINTER(vp)]
        lib.tj_b200_program_create.restype = ctypes.c_int
        lib.tj_b200_run.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(vp), vp]
        lib.tj_b200_run.restype = ctypes.c_int
        lib.tj_b200_time_kernels.argtypes = [vp, ctypes.POINTER(vp), ctypes.POINTER(vp), vp, i32,
                                             ctypes.POINTER(ctypes.c_float)]
        lib.tj_b200_time_kernels.restype = ctypes.c_int
        lib.tj_b200_linear_f32_noalloc.argtypes = [vp, vp, vp, i32, i32, i32, vp]
        lib.tj_b200_linear_f32_noalloc.restype = ctypes.c_int
        lib.tj_b200_linear_f32_noalloc_status.argtypes = [ctypes.POINTER(i32), ctypes.POINTER(i32), vp]
        lib.tj_b200_linear_f32_noalloc_status.restype = ctypes.c_int
        lib.tj_b200_ipc_export.argtypes = [vp, i32, ctypes.POINTER(TjIpcHandle), ctypes.POINTER(u64)]
        lib.tj_b200_ipc_export.restype = ctypes.c_int
        lib.tj_b200_ipc_open.argtypes = [ctypes.POINTER(TjIpcHandle), u64, i32, ctypes.POINTER(vp)]
        lib.tj_b200_ipc_open.restype = ctypes.c_int
        lib.tj_b200_ipc_close.argtypes = [vp, u64, i32]
        lib.tj_b200_ipc_close.restype = ctypes.c_int
        lib.tj_b200_set_pdl.argtypes = [vp, i32]
        lib.tj_b200_set_pdl.restype = ctypes.c_int
        lib.tj_b200_set_graph.argtypes = [vp, i32]
        lib.tj_b200_set_graph.restype = ctypes.c_int
        lib.tj_b200_check_status.argtypes = [vp, ctypes.POINTER(i32), ctypes.POINTER(i32)]
        lib.tj_b200_check_status.restype = ctypes.c_int
        lib.tj_b200_program_info.argtypes = [vp, ctypes.POINTER(TjProgramInfo)]
        lib.tj_b200_program_info.restype = ctypes.c_int
        lib.tj_b200_destroy.argtypes = [vp]
        lib.tj_b200_destroy.restype = ctypes.c_int
        lib.tj_b200_last_error.argtypes = []
        lib.tj_b200_last_error.restype = ctypes.c_char_p
        lib.tj_b200_abi_version.restype = ctypes.c_int
        lib.tj_b200_driver_available.restype = ctypes.c_int
        if path is None:
            _lib = lib
        return lib


def check(rc: int, what: str = "") -> None:
    if rc != TJ_OK:
        msg = library().tj_b200_last_error().decode(errors="replace")
        raise RuntimeError_(rc, f"{what}: {msg}" if what else msg)


def ipc_export(ptr: int, device: int) -> tuple[bytes, int]:
    """(64-byte handle, offset) that lets another process of this node map the device
    allocation holding ``ptr``."""
    h, off = TjIpcHandle(), ctypes.c_uint64()
    check(library().tj_b200_ipc_export(ctypes.c_void_p(ptr), device, ctypes.byref(h), ctypes.byref(off)),
          "tj_b200_ipc_export")
    return bytes(h.bytes), off.value


def ipc_open(handle: bytes, offset: int, device: int) -> int:
    """Device address, valid on ``device``, of the exported allocation plus ``offset``."""
    if len(handle) != 64:
        raise ValueError(f"an IPC handle has 64 bytes, got {len(handle)}")
    h = TjIpcHandle()
    ctypes.memmove(h.bytes, handle, 64)
    out = ctypes.c_void_p()
    check(library().tj_b200_ipc_open(ctypes.byref(h), offset, device, ctypes.byref(out)), "tj_b200_ipc_open")
    return int(out.value)


def ipc_close(ptr: int, offset: int, device: int) -> None:
    check(library().tj_b200_ipc_close(ctypes.c_void_p(ptr), offset, device), "tj_b200_ipc_close")


class NativeProgram:
    """Owns one runtime program handle (modules, arena, status word, graph)."""

    def __init__(self, cubins: list[bytes], launches: list[dict], args: list[tuple[int, int]],
                 tmaps: list[dict], arena_bytes: int, num_inputs: int, num_outputs: int, device: int):
        lib = library()
        self._lib = lib
        self._images = [ctypes.create_string_buffer(c, len(c)) for c in cubins]
        n_mod = len(cubins)
        img_ptrs = (ctypes.c_void_p * max(n_mod, 1))(*[ctypes.cast(b, ctypes.c_void_p) for b in self._images])
        sizes = (ctypes.c_size_t * max(n_mod, 1))(*[len(c) for c in cubins])
        self._symbols = [ctypes.create_string_buffer(L["symbol"].encode()) for L in launches]
        L_arr = (TjLaunch * max(len(launches), 1))()
        for i, L in enumerate(launches):
            t = L_arr[i]
            t.symbol = ctypes.cast(self._symbols[i], ctypes.c_char_p)
            t.module = L["module"]
            for d in range(3):
                t.grid[d] = L["grid"][d]
                t.block[d] = L["block"][d]
                t.cluster[d] = L.get("cluster", (1, 1, 1))[d]
            t.smem_bytes = L.get("smem", 0)
            t.param_bytes = L["param_bytes"]
            t.first_arg, t.num_args = L["first_arg"], L["num_args"]
            t.first_tmap, t.num_tmaps = L["first_tmap"], L["num_tmaps"]
        A_arr = (TjArgRef * max(len(args), 1))()
        for i, (kind, value) in enumerate(args):
            A_arr[i].kind = kind
            A_arr[i].value = value
        T_arr = (TjTMap * max(len(tmaps), 1))()
        for i, tm in enumerate(tmaps):
            t = T_arr[i]
            t.arg, t.dtype, t.rank, t.swizzle = tm["arg"], tm["dtype"], tm["rank"], tm["swizzle"]
            for d, v in enumerate(tm["dims"]):
                t.dims[d] = v
            for d, v in enumerate(tm["strides"]):
                t.strides[d] = v
            for d, v in enumerate(tm["box"]):
                t.box[d] = v
            t.param_offset = tm["param_offset"]
            t.l2_promotion = tm.get("l2_promotion", 2)
        self._launch_arr, self._arg_arr, self._tmap_arr = L_arr, A_arr, T_arr
        handle = ctypes.c_void_p()
        rc = lib.tj_b200_program_create(img_ptrs, sizes, n_mod, L_arr, len(launches), A_arr, len(args), T_arr,
                                        len(tmaps), arena_bytes, num_inputs, num_outputs, device,
                                        ctypes.byref(handle))
        check(rc, "tj_b200_program_create")
        self.handle = handle
        self.num_inputs, self.num_outputs = num_inputs, num_outputs
        self._in = (ctypes.c_void_p * max(num_inputs, 1))()
        self._out = (ctypes.c_void_p * max(num_outputs, 1))()

    def set_pdl(self, enable: bool) -> None:
        check(self._lib.tj_b200_set_pdl(self.handle, 1 if enable else 0), "tj_b200_set_pdl")

    def set_graph(self, enable: bool) -> None:
        check(self._lib.tj_b200_set_graph(self.handle, 1 if enable else 0), "tj_b200_set_graph")

    def run(self, in_ptrs: list[int], out_ptrs: list[int], stream: int) -> None:
        for i, p in enumerate(in_ptrs):
            self._in[i] = p
        for j, p in enumerate(out_ptrs):
            self._out[j] = p
        rc = self._lib.tj_b200_run(self.handle, self._in, self._out, stream or None)
        if rc != TJ_OK:
            check(rc, "tj_b200_run")

    def time_kernels(self, in_ptrs: list[int], out_ptrs: list[int], stream: int, iters: int,
                     num_kernels: int) -> list[float]:
        for i, p in enumerate(in_ptrs):
            self._in[i] = p
        for j, p in enumerate(out_ptrs):
            self._out[j] = p
        ms = (ctypes.c_float * max(num_kernels, 1))()
        check(self._lib.tj_b200_time_kernels(self.handle, self._in, self._out, stream or None, iters, ms),
              "tj_b200_time_kernels")
        return [ms[i] for i in range(num_kernels)]

    def check_status(self) -> tuple[int, int]:
        code, where = ctypes.c_int32(), ctypes.c_int32()
        rc = self._lib.tj_b200_check_status(self.handle, ctypes.byref(code), ctypes.byref(where))
        if rc == TJ_ERR_DEVICE_STATUS:
            return code.value, where.value
        check(rc, "tj_b200_check_status")
        return 0, 0

    def info(self) -> dict:
        inf = TjProgramInfo()
        check(self._lib.tj_b200_program_info(self.handle, ctypes.byref(inf)), "tj_b200_program_info")
        return {f: getattr(inf, f) for f, _ in TjProgramInfo._fields_}

    def close(self) -> None:
        if getattr(self, "handle", None):
            self._lib.tj_b200_destroy(self.handle)
            self.handle = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass
