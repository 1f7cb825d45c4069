"""The fused kernel plan this backend consumes, as a self-contained data model.

tensorjit's fusion pass hands a backend a ``Program``: a straight-line list of
``Kernel`` objects whose nodes are IR ``Node``s (``tensorjit/passes/fusion.py:24-61``,
``tensorjit/ir/graph.py:113-147``).  This module mirrors exactly the fields a backend
reads from those objects, so the B200 backend works both on a live tensorjit
``Program`` (``from_tensorjit``) and on a plan serialised to JSON (``to_json`` /
``from_json``), which is how plans travel to machines where tensorjit itself is
not installed.

Field meanings follow the reference:

* ``PNode``: one SSA value.  ``op`` is a key of ``OPS`` (``graph.py:71-110``),
  ``shape``/``dtype`` its static ``TensorType``; ``attrs`` carries ``value`` (const),
  ``trans_b`` (matmul), ``axis``/``keepdim`` (reductions), ``shape`` (reshape,
  broadcast_to) and ``perm`` (transpose).  ``users`` lists every consumer in the
  whole graph (``graph.py:119,129-130``).
* ``PKernel``: ``kind`` in {elementwise, copy, matmul, reduce, row}; ``nodes`` in
  topological order, ``anchor`` (matmul/reduce/movement node), ``inputs`` (values
  read from outside the kernel, consts excluded) and ``outputs`` (values that
  escape) exactly as ``_finalize`` computes them (``fusion.py:64-75``).  Row kernels
  also carry ``stages`` (the per-row sub-kernels in order), ``rows`` and ``n``
  (``fusion.py:326-328``).
* ``PProgram.aliases``: reshape node id -> (source node, shape); reshapes of
  materialised values are free views (``fusion.py:96-102``).
"""
from __future__ import annotations

import json
import math
from dataclasses import dataclass, field
from typing import Any, Optional

DTYPES = ("f32", "f16", "bf16", "i32")
ITEMSIZE = {"f32": 4, "f16": 2, "bf16": 2, "i32": 4}

ELEMENTWISE_OPS = {
    "neg": 1, "exp": 1, "log": 1, "sqrt": 1, "rsqrt": 1, "tanh": 1, "relu": 1, "sigmoid": 1,
    "gelu": 1, "silu": 1, "abs": 1,
    "add": 2, "sub": 2, "mul": 2, "div": 2, "pow": 2, "maximum": 2, "minimum": 2,
    "where": 3,
}
REDUCE_OPS = ("sum", "max", "mean")
MOVEMENT_OPS = ("reshape", "transpose", "broadcast_to")


@dataclass(eq=False)
class PNode:
    id: int
    op: str
    inputs: list["PNode"]
    shape: tuple
    dtype: str
    attrs: dict[str, Any] = field(default_factory=dict)
    name: str = ""
    users: list["PNode"] = field(default_factory=list, repr=False)

    @property
    def numel(self) -> int:
        return math.prod(self.shape) if self.shape else 1

    @property
    def nbytes(self) -> int:
        return self.numel * ITEMSIZE[self.dtype]

    @property
    def is_elementwise(self) -> bool:
        return self.op in ELEMENTWISE_OPS

    def __repr__(self) -> str:
        return f"{self.name}={self.op}({', '.join(i.name for i in self.inputs)}):{self.dtype}{list(self.shape)}"


@dataclass(eq=False)
class PKernel:
    kind: str
    nodes: list[PNode]
    anchor: Optional[PNode]
    inputs: list[PNode]
    outputs: list[PNode]
    iter_shape: tuple
    stages: list["PKernel"] = field(default_factory=list)
    rows: tuple = ()
    n: int = 0
    attrs: dict = field(default_factory=dict)   # backend-side rewrites (fuse.py) describe their kernels here

    def __repr__(self) -> str:
        return f"PKernel<{self.kind} {[x.op for x in self.nodes]} -> {[o.name for o in self.outputs]}>"


@dataclass(eq=False)
class PProgram:
    name: str
    nodes: list[PNode]
    inputs: list[PNode]
    outputs: list[PNode]
    kernels: list[PKernel]
    aliases: dict[int, tuple[PNode, tuple]]     # reshape node id -> (source node, shape)
    meta: dict[str, Any] = field(default_factory=dict)

    def resolve(self, n: PNode) -> PNode:
        """Follow reshape aliases to the materialised value (``fusion.py:88-92``)."""
        while n.id in self.aliases:
            n = self.aliases[n.id][0]
        return n

    def __str__(self) -> str:
        lines = [f"program {self.name}: {len(self.kernels)} kernels"]
        for k in self.kernels:
            lines.append(f"  {k.kind:12s} {[x.op for x in k.nodes]} -> {[o.name for o in k.outputs]}")
        return "\n".join(lines)

    # -- serialisation -------------------------------------------------------
    def to_dict(self) -> dict:
        def kd(k: PKernel) -> dict:
            d = {
                "kind": k.kind,
                "nodes": [x.id for x in k.nodes],
                "anchor": k.anchor.id if k.anchor is not None else None,
                "inputs": [x.id for x in k.inputs],
                "outputs": [x.id for x in k.outputs],
                "iter_shape": list(k.iter_shape),
            }
            if k.kind == "row":
                d["stages"] = [kd(s) for s in k.stages]
                d["rows"] = list(k.rows)
                d["n"] = k.n
            return d

        return {
            "format": "tensorjit-plan/1",
            "name": self.name,
            "nodes": [
                {"id": x.id, "op": x.op, "name": x.name, "inputs": [i.id for i in x.inputs],
                 "shape": list(x.shape), "dtype": x.dtype, "attrs": _attrs_to_json(x.attrs)}
                for x in self.nodes
            ],
            "inputs": [x.id for x in self.inputs],
            "outputs": [x.id for x in self.outputs],
            "kernels": [kd(k) for k in self.kernels],
            "aliases": {str(a): [src.id, list(shape)] for a, (src, shape) in self.aliases.items()},
            "meta": self.meta,
        }

    def to_json(self, **kw) -> str:
        return json.dumps(self.to_dict(), **kw)

    @staticmethod
    def from_dict(d: dict) -> "PProgram":
        if d.get("format") != "tensorjit-plan/1":
            raise ValueError(f"not a tensorjit plan (format={d.get('format')!r})")
        by_id: dict[int, PNode] = {}
        for nd in d["nodes"]:
            by_id[nd["id"]] = PNode(nd["id"], nd["op"], [], tuple(nd["shape"]), nd["dtype"],
                                    _attrs_from_json(nd["attrs"]), nd["name"])
        for nd in d["nodes"]:
            node = by_id[nd["id"]]
            node.inputs = [by_id[i] for i in nd["inputs"]]
        _link_users(list(by_id.values()))

        def kern(kd_: dict) -> PKernel:
            k = PKernel(
                kind=kd_["kind"],
                nodes=[by_id[i] for i in kd_["nodes"]],
                anchor=by_id[kd_["anchor"]] if kd_["anchor"] is not None else None,
                inputs=[by_id[i] for i in kd_["inputs"]],
                outputs=[by_id[i] for i in kd_["outputs"]],
                iter_shape=tuple(kd_["iter_shape"]),
            )
            if k.kind == "row":
                k.stages = [kern(s) for s in kd_["stages"]]
                k.rows = tuple(kd_["rows"])
                k.n = int(kd_["n"])
            return k

        return PProgram(
            name=d["name"],
            nodes=[by_id[nd["id"]] for nd in d["nodes"]],
            inputs=[by_id[i] for i in d["inputs"]],
            outputs=[by_id[i] for i in d["outputs"]],
            kernels=[kern(k) for k in d["kernels"]],
            aliases={int(a): (by_id[v[0]], tuple(v[1])) for a, v in d["aliases"].items()},
            meta=dict(d.get("meta", {})),
        )

    @staticmethod
    def from_json(text: str) -> "PProgram":
        return PProgram.from_dict(json.loads(text))

    @staticmethod
    def load(path) -> "PProgram":
        with open(path) as f:
            return PProgram.from_json(f.read())


def _attrs_to_json(attrs: dict) -> dict:
    out = {}
    for k, v in attrs.items():
        if isinstance(v, tuple):
            v = list(v)
        if isinstance(v, float) and (v != v or v in (float("inf"), float("-inf"))):
            v = {"float": repr(v)}
        out[k] = v
    return out


def _attrs_from_json(attrs: dict) -> dict:
    out = {}
    for k, v in attrs.items():
        if isinstance(v, dict) and "float" in v:
            v = float(v["float"])
        elif isinstance(v, list):
            v = tuple(v)
        out[k] = v
    return out


def _link_users(nodes: list[PNode]) -> None:
    for x in nodes:
        x.users = []
    for x in nodes:
        for i in x.inputs:
            i.users.append(x)


def from_tensorjit(program) -> PProgram:
    """Convert a live ``tensorjit.passes.Program`` into a ``PProgram``.

    Only attribute reads on the reference objects: ``Node.op/inputs/type/attrs/name``,
    ``Kernel.kind/nodes/anchor/inputs/outputs/iter_shape`` and the row-kernel extras
    ``stages/rows/n``, ``Program.graph/kernels/aliases``.
    """
    g = program.graph
    order: list = []
    seen: dict[int, int] = {}

    def visit(n):
        if id(n) in seen:
            return
        for i in n.inputs:
            visit(i)
        seen[id(n)] = len(order)
        order.append(n)

    for n in list(g.inputs) + list(g.nodes):
        visit(n)
    for k in program.kernels:
        for n in list(k.nodes) + list(k.inputs) + list(k.outputs):
            visit(n)
    for a, (src, _shape) in program.aliases.items():
        visit(src)
    for o in g.outputs:
        visit(o)
    pn: dict[int, PNode] = {}
    for i, n in enumerate(order):
        dt = n.type.dtype
        dt = dt.value if hasattr(dt, "value") else str(dt)
        pn[id(n)] = PNode(i, n.op, [], tuple(n.type.shape), dt, dict(n.attrs), n.name)
    for n in order:
        pn[id(n)].inputs = [pn[id(i)] for i in n.inputs]
    nodes = [pn[id(n)] for n in order]
    _link_users(nodes)

    def kern(k) -> PKernel:
        pk = PKernel(
            kind=k.kind,
            nodes=[pn[id(n)] for n in k.nodes],
            anchor=pn[id(k.anchor)] if k.anchor is not None else None,
            inputs=[pn[id(n)] for n in k.inputs],
            outputs=[pn[id(n)] for n in k.outputs],
            iter_shape=tuple(k.iter_shape),
        )
        if k.kind == "row":
            pk.stages = [kern(s) for s in k.stages]
            pk.rows = tuple(k.rows)
            pk.n = int(k.n)
        return pk

    # alias keys in the reference are id(node) of reshape nodes
    aliases = {}
    for n in order:
        if id(n) in program.aliases:
            src, shape = program.aliases[id(n)]
            aliases[pn[id(n)].id] = (pn[id(src)], tuple(shape))
    return PProgram(
        name=g.name,
        nodes=nodes,
        inputs=[pn[id(n)] for n in g.inputs],
        outputs=[pn[id(n)] for n in g.outputs],
        kernels=[kern(k) for k in program.kernels],
        aliases=aliases,
    )


def as_plan(program) -> PProgram:
    """Accept a ``PProgram``, a plan dict/JSON string, or a live tensorjit ``Program``."""
    if isinstance(program, PProgram):
        return program
    if isinstance(program, dict):
        return PProgram.from_dict(program)
    if isinstance(program, str):
        return PProgram.from_json(program)
    if hasattr(program, "kernels") and hasattr(program, "graph") and hasattr(program, "aliases"):
        return from_tensorjit(program)
    raise TypeError(f"cannot interpret {type(program).__name__} as a kernel plan")


# -- stride helpers (same definitions as tensorjit/backends/common.py:11-35) --------------
def contiguous_strides(shape: tuple) -> tuple:
    strides, acc = [], 1
    for s in reversed(shape):
        strides.append(acc)
        acc *= s
    return tuple(reversed(strides))


def broadcast_strides(in_shape: tuple, iter_shape: tuple) -> tuple:
    """Element strides to read a contiguous ``in_shape`` tensor at every point of
    ``iter_shape``; broadcast dimensions get stride 0 (``common.py:18-26``)."""
    cs = contiguous_strides(in_shape)
    pad = len(iter_shape) - len(in_shape)
    out = [0] * pad
    for d in range(len(in_shape)):
        out.append(0 if in_shape[d] == 1 and iter_shape[pad + d] != 1 else cs[d])
    return tuple(out)


def access_strides(inp: PNode, consumer: PNode, iter_shape: tuple) -> tuple:
    """How ``consumer`` reads ``inp`` over ``iter_shape``: a transpose reads with
    permuted strides, everything else with broadcast strides (``common.py:29-35``)."""
    if consumer.op == "transpose":
        perm = consumer.attrs["perm"]
        cs = contiguous_strides(inp.shape)
        return tuple(cs[p] for p in perm)
    return broadcast_strides(inp.shape, iter_shape)


def first_consumer(n: PNode, candidates: list[PNode], default: PNode) -> PNode:
    """The node through which a kernel reads input ``n`` (reference idiom
    ``next((c for c in nodes if n in c.inputs), nodes[0])``)."""
    for c in candidates:
        if any(i is n for i in c.inputs):
            return c
    return default
