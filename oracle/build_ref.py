"""Recipe for ``oracle/_ref``: the reference ``c`` backend's own kernels for the
benchmark programs — TEST / BASELINE INFRASTRUCTURE ONLY.

Step 1 (here, where the reference tensorjit sources are importable; writes only
into ``oracle/_ref``):

    CC=/usr/bin/gcc CXX=/usr/bin/g++ python oracle/build_ref.py --ref <tensorjit checkout>

traces each benchmark program in f32, lowers it with the reference's own passes,
and lets the reference's ``c_backend`` generate its C/OpenMP source
(``tensorjit/backends/c_backend.py:344-416``, autotune off so the analytic tile
choice of ``autotune.py:48-80`` is used).  It writes ``<name>.c`` (the generated
source, untouched) and ``<name>.json`` (kernel symbols and, per kernel argument,
INPUT/ARENA/OUTPUT references resolved against the reference memory planner,
exactly as ``tensorjit/runtime/native.py:70-96`` resolves them).

Step 2 (on the machine that runs the baseline, see ``oracle/ref_runner.py``):
compile ``<name>.c`` with the reference's flags (``c_backend.py:317``:
``-O3 -shared -fPIC -ffast-math -march=native -fopenmp -std=c11``) for that
host's CPU and run the kernels in plan order the way the reference's native
runtime does (``csrc/runtime.cpp:88-110``).
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import tempfile
from pathlib import Path

HERE = Path(__file__).resolve().parent
OUT = HERE / "_ref"
REPO = HERE.parent
sys.path.insert(0, str(REPO))

from oracle import reference_checkout  # noqa: E402

# (name, workload, rows of the row-sharded arguments or None for the full program)
SAMPLES = [("cfg1", "cfg1", None), ("cfg2", "cfg2", None), ("cfg3_m512", "cfg3", 512), ("cfg4", "cfg4", None),
           ("cfg5_m1024", "cfg5", 1024)]


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", default=str(reference_checkout()))
    a = ap.parse_args()
    if not Path(a.ref).exists():
        print(f"reference not found at {a.ref}; nothing to do")
        return
    sys.path.insert(0, a.ref)
    os.environ.setdefault("TENSORJIT_NO_AUTOTUNE", "1")
    os.environ.setdefault("TENSORJIT_CACHE_DIR", tempfile.mkdtemp(prefix="tjref_"))
    import tensorjit as tj
    import tensorjit.compiler as C
    from tensorjit.backends import c_backend
    from tensorjit.ir import TensorType
    from tensorjit.passes.memory_planner import plan_memory

    sys.path.insert(0, str(REPO / "tests" / "golden"))
    from make_fixtures import config_fns

    from mlir_gpu_kernel_compiler_b200 import workloads as W

    fns = config_fns(tj)
    OUT.mkdir(exist_ok=True)
    for name, wname, rows in SAMPLES:
        w = W.WORKLOADS[wname]
        shapes = [tuple(ar.shape) for ar in w.args]
        if rows is not None:
            for i in w.row_args:
                shapes[i] = (rows,) + shapes[i][1:]
        g = tj.trace(fns[wname], [TensorType(s) for s in shapes])
        program = C.lower(g, "c")
        cp = c_backend.compile_program(program, tune=False)
        plan = plan_memory(program)
        aliases = program.aliases

        def resolve(n):
            while id(n) in aliases:
                n = aliases[id(n)][0]
            return n

        in_index = {id(n): i for i, n in enumerate(g.inputs)}
        escaping = {id(resolve(o)) for o in g.outputs}
        out_nodes = []
        for k in program.kernels:
            for o in k.outputs:
                if id(o) in escaping and o not in out_nodes:
                    out_nodes.append(o)
        out_index = {id(o): j for j, o in enumerate(out_nodes)}

        def ref(n):
            src = resolve(n)
            if id(src) in in_index:
                return [0, in_index[id(src)]]
            if id(src) in out_index:
                return [2, out_index[id(src)]]
            return [1, plan.offset(src)]

        manifest = {
            "name": name, "workload": wname, "rows": rows,
            "input_shapes": [list(s) for s in shapes],
            "output_shapes": [list(o.shape) for o in out_nodes],
            "graph_outputs": [out_index[id(resolve(o))] for o in g.outputs],
            "arena_bytes": plan.arena_bytes,
            "symbols": list(cp.symbols),
            "args": [[ref(i) for i in k.inputs] + [ref(o) for o in k.outputs] for k in program.kernels],
            "flags": ["-O3", "-shared", "-fPIC", "-ffast-math", "-march=native", "-fopenmp", "-std=c11"],
        }
        (OUT / f"{name}.c").write_text(cp.source)
        (OUT / f"{name}.json").write_text(json.dumps(manifest, indent=1))
        print(f"{name}: {len(cp.symbols)} kernels, arena {plan.arena_bytes} B")


if __name__ == "__main__":
    main()
