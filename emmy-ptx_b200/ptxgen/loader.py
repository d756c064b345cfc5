"""Load a Kernel IR json plus its sibling ``meta.json`` into a ``KernelSpec``.

Same contract as the reference's ``load_kernel`` (``ptxgen/loader.py:32-119``):

* the first ``KernelOp`` node of the graph is the kernel; its ``name`` is the
  entry point;
* ``meta.json`` next to the IR file is the launch contract: the kernel entry
  whose ``entry`` matches (or the only one) gives ``arg_order``, ``args``,
  ``grid``, ``block``, ``smem_bytes`` and ``zero_outputs``;
* without ``meta.json`` the signature is the node's inputs followed by its
  outputs, with shapes and dtypes from the graph and a 1x1x1 launch;
* names in ``arg_order`` missing from meta's ``args`` are filled from the
  graph (``ZeroPrologue`` destinations are the known case).

The IR itself is deserialised by ``ptxgen.ir`` instead of ``emmy-ml``.
"""

from __future__ import annotations

import json
from pathlib import Path

from . import ir
from .model import ArgSpec, KernelSpec


def _graph_tensor(g: ir.Graph, name: str):
    for node in g.nodes.values():
        for t in node.outputs:
            if t.name == name:
                return t
    return None


def _arg_from_meta(a: dict) -> ArgSpec:
    data = a.get("data")
    value = a.get("value")
    if value is None and data:
        value = data[0]
    return ArgSpec(
        name=a["name"],
        dtype=a.get("dtype", "f32"),
        shape=tuple(int(x) for x in (a.get("shape") or ())),
        scalar=bool(a.get("scalar", False)),
        value=value,
        output=bool(a.get("output", False)),
        seed=a.get("seed"),
        data=list(data) if data is not None else None,
        intermediate=bool(a.get("intermediate", False)),
    )


def _arg_from_graph(g: ir.Graph, name: str, outputs) -> ArgSpec:
    t = _graph_tensor(g, name)
    if t is None:
        return ArgSpec(name=name, dtype="f32", shape=(), output=name in outputs)
    return ArgSpec(name=name, dtype=t.dtype.name, shape=tuple(int(d) for d in t.shape),
                   output=name in outputs)


def load_kernel_data(data: dict, meta: dict | None, source: str = "<memory>") -> KernelSpec:
    graph = ir.Graph.from_dict(data)
    kernels = [n.op for n in graph.nodes.values() if isinstance(n.op, ir.KernelOp)]
    if not kernels:
        raise ValueError(f"{source}: the graph holds no KernelOp to compile")
    op = kernels[0]
    entry = op.name or ""
    if not entry:
        raise ValueError(f"{source}: the KernelOp names no entry point")

    kmeta = None
    if meta is not None:
        cands = meta.get("kernels", [])
        kmeta = next((k for k in cands if k.get("entry") == entry), None)
        if kmeta is None and len(cands) == 1:
            kmeta = cands[0]

    args: dict[str, ArgSpec] = {}
    if kmeta is not None:
        arg_order = list(kmeta.get("arg_order") or [])
        for a in kmeta.get("args", []):
            args[a["name"]] = _arg_from_meta(a)
        grid = tuple(int(x) for x in (kmeta.get("grid") or (1, 1, 1)))
        block = tuple(int(x) for x in (kmeta.get("block") or (1, 1, 1)))
        smem = int(kmeta.get("smem_bytes") or 0)
        zero = list(kmeta.get("zero_outputs") or [])
    else:
        arg_order = list(op.inputs) + list(op.outputs)
        for name in arg_order:
            args[name] = _arg_from_graph(graph, name, op.outputs)
        grid, block, smem, zero = (1, 1, 1), (1, 1, 1), 0, []

    if not arg_order:
        arg_order = list(args)
    for name in arg_order:
        if name not in args:
            args[name] = _arg_from_graph(graph, name, op.outputs)

    return KernelSpec(op=op, entry=entry, arg_order=arg_order, args=args, grid=grid,
                      block=block, smem_bytes=smem, zero_outputs=zero, source=source)


def load_kernel(path: str | Path) -> KernelSpec:
    path = Path(path)
    data = json.loads(path.read_text())
    meta_path = path.parent / "meta.json"
    meta = json.loads(meta_path.read_text()) if meta_path.exists() else None
    return load_kernel_data(data, meta, source=str(path))
