"""B200-native execution backend for tensorjit's fused kernel plan.

Drop-in for the reference's backend plugin interface
(``tensorjit/compiler.py:45-73`` -> ``<backend>.compile_program(program, device, tune)``):

    import tensorjit as tj
    import mlir_gpu_kernel_compiler_b200 as tjb

    tjb.register()                      # adds backend "b200" to tensorjit (and makes it the cuda default)
    f = tj.jit(fn, backend="b200")      # or tensors on cuda with no backend given
    y = f(*cuda_tensors)

or, with a plan produced elsewhere (a ``tensorjit.passes.Program`` or its JSON form):

    prog = tjb.compile_program(plan, device="cuda")
    outs = prog(*cuda_tensors)

The package holds: ``plan`` (the plan data model), ``memory`` (arena planner),
``codegen`` (plan -> sm_100a CUDA sources), ``csrc`` (hand-written kernel
templates and the C++ runtime behind ``include/tj_b200.h``), ``toolchain``
(nvcc / g++ builds and the cubin cache), ``runtime`` (ctypes binding of the C
ABI), ``program`` (``B200Program``), ``autotune`` (tcgen05 tile search),
``distributed`` (row-sharded execution over NCCL) and ``workloads`` (the
benchmark programs' seeded inputs).
"""
from __future__ import annotations

from .plan import PProgram, as_plan, from_tensorjit
from .program import B200Program, compile_program

ROW_FUSION_MAX_N = 8192
__version__ = "0.1.0"


def register(make_default: bool = True) -> None:
    """Register backend ``"b200"`` with an importable tensorjit.

    Mirrors the four edits the reference's dispatch needs (``compiler.py:21,24-31,34,61-68``):
    the name in ``BACKENDS``, ``ROW_FUSION_MAX_N["b200"] = 8192`` (so the plan is
    identical to the one the ``cuda`` backend gets), a ``compile_graph`` branch that
    calls this package's ``compile_program``, and (optionally) ``"b200"`` as the
    default backend for cuda tensors.
    """
    import tensorjit.compiler as C

    if getattr(C, "_b200_registered", False):
        return
    if "b200" not in C.BACKENDS:
        C.BACKENDS = tuple(C.BACKENDS) + ("b200",)
    C.ROW_FUSION_MAX_N["b200"] = ROW_FUSION_MAX_N
    orig_compile_graph = C.compile_graph
    orig_pick = C.pick_backend

    def compile_graph(graph, backend, device="cpu", tune=True):
        if backend == "b200":
            program = C.lower(graph, backend)
            return compile_program(program, device="cuda" if device == "cpu" else device, tune=tune)
        return orig_compile_graph(graph, backend, device=device, tune=tune)

    def pick_backend(device, requested=None):
        import os

        requested = requested or os.environ.get("TENSORJIT_BACKEND")
        if requested:
            assert requested in C.BACKENDS, f"unknown backend {requested}"
            return requested
        if make_default and device == "cuda":
            return "b200"
        return orig_pick(device, None)

    C.compile_graph = compile_graph
    C.pick_backend = pick_backend
    # modules that imported the two functions by name keep their own bindings: the package
    # re-exports (tensorjit/__init__.py:17) and the torch.compile backend
    # (tensorjit/frontend/torch_backend.py:22), which calls them in torch_compile_backend
    import sys

    for mod in ("tensorjit", "tensorjit.frontend.torch_backend"):
        m = sys.modules.get(mod)
        if m is not None:
            if getattr(m, "compile_graph", None) is orig_compile_graph:
                m.compile_graph = compile_graph
            if getattr(m, "pick_backend", None) is orig_pick:
                m.pick_backend = pick_backend
    C._b200_registered = True


__all__ = ["B200Program", "compile_program", "register", "PProgram", "as_plan", "from_tensorjit",
           "ROW_FUSION_MAX_N"]
