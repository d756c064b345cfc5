"""Kernel IR generator: the problem families of the open set at any shape.

Emmy's tracer (``tools/generate.py:57-71``) is not available, so this module
writes Kernel IR directly, in the repr grammar ``ptxgen.ir`` parses.  For each
family it follows the schedule of the shipped problem of that family and only
re-derives the shape-dependent literals:

* ``pointwise``   -- p00..p03 (``Tile[a0]``, ``U`` elements per cell, grouped
                     vector write);
* ``reduce_full`` -- r01..r03 (one CTA of ``T`` threads strides the array;
                     optional mean epilogue);
* ``reduce_rows`` -- r04 (one row per CTA);
* ``rmsnorm``, ``softmax``, ``l2norm`` -- f01..f03 (reduce, then a second
                     strided pass over the row);
* ``matmul``      -- m01 (32x64x64 tiles, 3-stage ``cp.async`` ring,
                     512 threads, 2x2 outputs per thread);
* ``matmul_splitk`` -- m02 (16x32x8 tiles, K split into slices reduced with
                     atomic writes into a zeroed C);
* ``attention``   -- a02 (one output element per thread, online softmax)
                     and its ``[B, H, S, D]`` generalisation with K given
                     untransposed;
* ``attention_tiled`` -- a01 (the same online softmax, a 4 x 2 output tile
                     per thread);
* ``tma_box_copy``, ``matmul_tma`` -- kernels written with the bulk-async
                     transport nodes (``TmaDescriptor``, ``TmaLoad``,
                     ``Mbarrier*``, ``SetMaxNReg``), which no shipped problem
                     uses: a box copy with zero fill and swizzle, and the m02
                     tile schedule fed by box copies instead of ``cp.async``;
* ``matmul_mma``  -- a 16-bit matmul on warp-level tensor-core fragments
                     (``RegFragment``, ``LdmatrixLoad``, ``MmaSyncPtx``,
                     ``RegStore``) fed by box copies;
* ``attention_mma`` -- softmax(Q K^T / sqrt(D)) V in fragments: S cells
                     by ``mma.sync``, row max and sum by
                     ``FragmentRowReduce``, scaling and exp by
                     ``FragmentApply``, P turned into A cells by
                     ``FragmentRepack`` for the P V products;
* ``carry_scan``  -- a per-row recurrence on carried state (``Pre`` /
                     ``Carry``): two cells updated from each other's previous
                     values, a counter set only under a condition, the
                     carrying loop run twice inside an outer loop;
* ``matmul_wgmma`` -- C = A.B^T (B given K-major, [N][K]) on warpgroup
                     products (``WgmmaDescriptor``, ``WgmmaMma``,
                     ``WgmmaFence/Commit/Wait``) over 128-byte-swizzled box
                     copies.

At the shipped shapes the generated bodies equal the shipped ones byte for
byte (``tests/test_irgen.py``); that pins the generator to the reference's
schedule.  Every generator returns ``(graph_json, meta_json)``.
"""

from __future__ import annotations

import json
import math

from .ir import (Accum, Assign, Axis, BinaryExpr, Cond, CpAsyncCommit, CpAsyncCopy,
                 CpAsyncWait, Dim, ElementwiseImpl, Init, Let, Literal, Load, Loop,
                 LdmatrixLoad, MbarrierArriveExpectTx, MbarrierInit, MbarrierWait, MmaSyncPtx,
                 RegFragment, RegStore, SetMaxNReg, Smem, StridedLoop, Sync, TernaryExpr, Tile,
                 TmaDescriptor, TmaLoad, TreeHalve, Var, WarpShuffle, WgmmaCommit,
                 WgmmaDescriptor, WgmmaFence, WgmmaMma, WgmmaWait, Window, Write, datatype,
                 FragmentApply, FragmentPromote, FragmentRepack, FragmentRowReduce, Pre, Carry)

F32 = datatype("f32")


def L(v: int) -> Literal:
    return Literal(value=int(v), dtype="int")


def Lf(v: float) -> Literal:
    return Literal(value=float(v), dtype="float")


def V(n: str) -> Var:
    return Var(name=n)


def _b(op):
    return lambda a, b: BinaryExpr(op=op, left=a, right=b)


ADD, SUB, MUL, DIV, MOD, LT, EQ = (_b(o) for o in ("+", "-", "*", "/", "%", "<", "=="))


def EW(name: str) -> ElementwiseImpl:
    return ElementwiseImpl(name)


def ax(name: str, extent: int, window=None) -> Axis:
    return Axis(name=name, extent=Dim(extent), window=window)


def win(parent: str, extent: int) -> Window:
    return Window(parent=ax(parent, extent), base=None, bound=None, partition=False)


def tile(axes, body, block_threads=None, raster_axes=None, raster_group=None) -> Tile:
    return Tile(axes=tuple(axes), body=tuple(body), block_threads=block_threads, aux_threads=0,
                raster_axes=raster_axes, raster_group=raster_group, raster_orient="m")


def load(names, buf, index, dtype=F32) -> Load:
    if isinstance(names, str):
        names = (names,)
    return Load(names=tuple(names), input=buf, index=tuple(index), dtype=dtype)


def assign(name, op, *args, dtype=F32) -> Assign:
    return Assign(name=name, op=EW(op), args=tuple(args), dtype=dtype)


def accum(name, value, op, axes, base=None, dtype=F32) -> Accum:
    return Accum(name=name, value=value, op=EW(op), dtype=dtype, axes=tuple(axes), base=base)


def write(out, index, values, atomic=False, dtype=F32) -> Write:
    if isinstance(values, str):
        values = (values,)
    return Write(output=out, index=tuple(index), values=tuple(values), value_dtype=dtype,
                 atomic=atomic, swizzle="NONE")


def strided(axis, extent, start, step, body) -> StridedLoop:
    return StridedLoop(axis=ax(axis, extent), start=start, step=step, body=tuple(body),
                       unroll=False, end=None, seed=True)


def loop(axis, extent, body, unroll=False, seed=True) -> Loop:
    return Loop(axis=ax(axis, extent), body=tuple(body), unroll=unroll, seed=seed)


# ---------------------------------------------------------------------------
# graph + meta packaging
# ---------------------------------------------------------------------------


def package(entry: str, node: str, body, inputs: list[tuple], constants: list[tuple],
            output: tuple, arg_order: list[str], grid, block, smem_bytes=0,
            zero_outputs=(), rtol=1e-3, atol=1e-4, code="", pid="generated",
            kernel_inputs: list[str] | None = None, graph_out_shape=None):
    """Build the graph json and meta json the loader reads.

    ``inputs``: (name, shape, dtype, seed); ``constants``: (name, value);
    ``output``: (name, shape, dtype)."""
    nodes: dict = {}
    for name, value in constants:
        nodes[name] = {"op": "ConstantOp",
                       "op_fields": {"name": name, "value": value, "context_value": None,
                                     "load_ops": [], "source_path": None, "source_parts": [],
                                     "source_shape": None, "source_dtype": None,
                                     "source_graph": None},
                       "inputs": [], "outputs": [{"name": name, "shape": [1], "dtype": "f32"}]}
    for name, shape, dt, _seed in inputs:
        nodes[name] = {"op": "InputOp", "op_fields": {}, "inputs": [],
                       "outputs": [{"name": name, "shape": list(shape), "dtype": dt}]}
    nodes = dict(sorted(nodes.items()))
    oname, oshape, odt = output
    kin = kernel_inputs if kernel_inputs is not None else [n for n in arg_order if n != oname]
    nodes[node] = {"op": "KernelOp",
                   "op_fields": {"body": [repr(s) for s in body], "name": entry,
                                 "zero_delegated": [], "serial": []},
                   "inputs": list(kin),
                   "outputs": [{"name": oname,
                                "shape": list(oshape if graph_out_shape is None else graph_out_shape),
                                "dtype": odt}]}
    graph = {"inputs": [i[0] for i in inputs], "outputs": [oname], "nodes": nodes}
    args = []
    for name in arg_order:
        c = next((c for c in constants if c[0] == name), None)
        i = next((i for i in inputs if i[0] == name), None)
        if c is not None:
            args.append({"name": name, "dtype": "f32", "shape": [1], "data": [c[1]]})
        elif i is not None:
            args.append({"name": name, "dtype": i[2], "shape": list(i[1]), "seed": i[3]})
        else:
            args.append({"name": name, "dtype": odt, "shape": list(oshape), "output": True})
    meta = {"id": pid, "code": code, "rtol": rtol, "atol": atol,
            "graph_inputs": [i[0] for i in inputs], "graph_outputs": [oname],
            "kernels": [{"node": node, "entry": entry, "arg_order": list(arg_order),
                         "grid": [int(g) for g in grid], "block": [int(b) for b in block],
                         "smem_bytes": int(smem_bytes), "zero_outputs": list(zero_outputs),
                         "args": args, "final": True}]}
    return graph, meta


# ---------------------------------------------------------------------------
# category 1: pointwise
# ---------------------------------------------------------------------------

# A pointwise program: per-element steps, in emission order.
#   ("load", base, buffer, "vec"|"const")   ("op", base, opname, argbases...)
PROGRAMS = {
    "add": [("load", "in0", "x0", "vec"), ("load", "in1", "x1", "vec"),
            ("op", "v0", "add", "in0", "in1")],
    "scale_shift": [("load", "in1", "mul_c1", "const"), ("load", "in2", "x", "vec"),
                    ("op", "v0", "multiply", "in1", "in2"), ("load", "in0", "add_c1", "const"),
                    ("op", "v1", "add", "in0", "v0")],
    "relu_mul": [("load", "in0", "x", "vec"), ("op", "v0", "relu", "in0"),
                 ("load", "in1", "y", "vec"), ("op", "v1", "multiply", "in1", "v0")],
    # "scalar": element 0 of a one-element input (an earlier kernel's result)
    "center": [("load", "in0", "x", "vec"), ("load", "in1", "mean", "scalar"),
               ("op", "v0", "subtract", "in0", "in1")],
}


def pointwise(n: int, unroll: int, program="add", block: int = 256,
              out: str = "add", arg_order=None, constants=(), entry="k_add_pointwise",
              rtol=0.0, atol=0.0, pid="pointwise", dtype="f32"):
    """``program``: a name in PROGRAMS or a list of steps in that format.
    ``dtype`` is the element type of the vector inputs, of every op (each
    result is coerced to it, as ``Assign.dtype`` asks) and of the output;
    constants stay f32 as the graph's ConstantOps are."""
    steps = PROGRAMS[program] if isinstance(program, str) else list(program)
    dt = datatype(dtype)
    if n % unroll:
        raise ValueError("n must be a multiple of the unroll factor")
    cells = n // unroll
    body = []
    for k in range(unroll):
        idx = ADD(MUL(V("a0"), L(unroll)), L(k))
        for st in steps:
            if st[0] == "load":
                _, base, buf, kind = st
                body.append(load(f"{base}__u{k}", buf, (idx,) if kind == "vec" else (L(0),),
                                 dtype=dt if kind == "vec" else F32))
            else:
                _, base, opname, *args = st
                body.append(assign(f"{base}__u{k}", opname, *[f"{a}__u{k}" for a in args],
                                   dtype=dt))
    last = [s for s in steps if s[0] == "op"][-1][1]
    body.append(write(out, (ADD(MUL(V("a0"), L(unroll)), L(0)),),
                      tuple(f"{last}__u{k}" for k in range(unroll)), dtype=dt))
    t = tile([ax("a0", cells)], body)
    vec_inputs = []
    seen = set()
    for st in steps:
        if st[0] == "load" and st[3] == "vec" and st[2] not in seen:
            seen.add(st[2])
            vec_inputs.append(st[2])
    scalar_inputs = sorted({st[2] for st in steps if st[0] == "load" and st[3] == "scalar"})
    if arg_order is None:
        arg_order = [c[0] for c in constants] + vec_inputs + scalar_inputs + [out]
    inputs = [(b, (n,), dtype, i) for i, b in enumerate(sorted(vec_inputs))]
    inputs += [(b, (1,), "f32", len(inputs) + i) for i, b in enumerate(scalar_inputs)]
    grid = (math.ceil(cells / block), 1, 1)
    return package(entry, out, [t], inputs, list(constants), (out, (n,), dtype), arg_order,
                   grid, (block, 1, 1), rtol=rtol, atol=atol, pid=pid)


# ---------------------------------------------------------------------------
# category 2: reductions
# ---------------------------------------------------------------------------


def _combine(state=("acc0",), kind="add"):
    if kind == "add":
        return (Assign(name="acc0", op=EW("add"), args=("acc0", "acc0__o"), dtype=None),)
    if kind == "maximum":
        return (Assign(name="acc0", op=EW("maximum"), args=("acc0", "acc0__o"), dtype=None),)
    if kind == "online_softmax":
        return (
            Assign(name="acc0__o__gn", op=EW("maximum"), args=("acc0", "acc0__o"), dtype=None),
            Assign(name="acc0__o__dg", op=EW("subtract"), args=("acc0", "acc0__o__gn"), dtype=None),
            Assign(name="acc0__o__alpha", op=EW("exp"), args=("acc0__o__dg",), dtype=None),
            Assign(name="acc0__o__dg_o", op=EW("subtract"), args=("acc0__o", "acc0__o__gn"),
                   dtype=None),
            Assign(name="acc0__o__beta", op=EW("exp"), args=("acc0__o__dg_o",), dtype=None),
            Assign(name="acc0__o__acc1_sa", op=EW("multiply"), args=("acc0__o__alpha", "acc1"),
                   dtype=None),
            Assign(name="acc0__o__acc1_sb", op=EW("multiply"), args=("acc0__o__beta", "acc1__o"),
                   dtype=None),
            Assign(name="acc1", op=EW("add"), args=("acc0__o__acc1_sa", "acc0__o__acc1_sb"),
                   dtype=None),
            Assign(name="acc0", op=EW("copy"), args=("acc0__o__gn",), dtype=None),
        )
    raise ValueError(kind)


def _block_combine(tid_axis: str, threads: int, states=("acc0",), kind="add"):
    """WarpShuffle + per-warp smem slots + TreeHalve, as r01..f03 write it."""
    comb = _combine(states, kind)
    sb = tuple(f"{s}__o" for s in states)
    warps = threads // 32
    out = [WarpShuffle(state=tuple(states), state_b=sb, combine_states=comb, length=32,
                       dtype=F32)]
    out += [Smem(name=f"{s}_smem", extents=(warps,), dtype="float", align=0) for s in states]
    out.append(Cond(cond=EQ(V("lane"), L(0)),
                    body=tuple(write(f"{s}_smem", (V("warp"),), s) for s in states),
                    else_body=()))
    out.append(Sync(barrier_id=0, count=None, warp=False))
    out.append(TreeHalve(bufs=tuple(f"{s}_smem" for s in states), state=tuple(states),
                         state_b=sb, combine_states=comb, length=warps, tid_var="warp",
                         dtype=F32, barrier_id=0, barrier_count=None, inner=None))
    return out


def reduce_full(n: int, threads: int = 128, mean: bool = False, entry=None, pid="reduce_full",
                dtype="f32", acc_dtype="f32"):
    """Full-array sum (r01/r02) or mean (r03) by one CTA of ``threads``.
    ``dtype`` is the input's and the result's element type, ``acc_dtype``
    the per-thread accumulator's: f32 or f16, the float states the
    reference's WarpShuffle takes (``ptxgen/emit.py:1385-1395``; the combine
    itself promotes to f32)."""
    body = [strided("a0", n, V("a0_co"), L(threads),
                    [load("in0", "x", (V("a0"),), dtype=datatype(dtype)),
                     accum("acc0", "in0", "add", ("a0",), dtype=datatype(acc_dtype))])]
    body += _block_combine("a0_co", threads)
    if mean:
        tail = [load("in1", "mean_keepdim_count", (L(0),)),
                assign("v0", "divide", "acc0", "in1"),
                write("mean", (), "v0", dtype=datatype(dtype))]
        out, entry = "mean", entry or "k_mean_ffcca3"
        constants = [("mean_keepdim_count", float(n))]
        arg_order = ["x", "mean_keepdim_count", "mean"]
    else:
        tail = [write("sum_1", (), "acc0", dtype=datatype(dtype))]
        out, entry = "sum_1", entry or "k_sum_1_reduce"
        constants = []
        arg_order = ["x", "sum_1"]
    body.append(Cond(cond=EQ(V("a0_co"), L(0)), body=tuple(tail), else_body=()))
    t = tile([ax("a0_co", threads)], body, block_threads=threads)
    return package(entry, out, [t], [("x", (n,), dtype, 0)], constants, (out, (1,), dtype),
                   arg_order, (1, 1, 1), (threads, 1, 1), rtol=1e-4, atol=1e-4, pid=pid,
                   graph_out_shape=())


def scalar_affine(n: int, s: float, t: float, lim: int, block: int = 256,
                  entry="k_affine_scalar", pid="scalar_affine"):
    """``out[i] = x[i] * s + t`` for ``i < lim``, else ``x[i]``, with ``s``,
    ``t`` (f32) and ``lim`` (s32) passed by value -- the runner's
    ``"scalar": true`` argument form (``docs/API.md:49``), which the kernel
    body names like any SSA value."""
    body = [load("in0", "x", (V("a0"),)),
            Cond(cond=LT(V("a0"), V("lim")),
                 body=(assign("v0", "multiply", "in0", "s"), assign("v1", "add", "v0", "t"),
                       write("out", (V("a0"),), "v1")),
                 else_body=(write("out", (V("a0"),), "in0"),))]
    tl = tile([ax("a0", n)], body)
    graph, meta = package(entry, "out", [tl], [("x", (n,), "f32", 0)], [],
                          ("out", (n,), "f32"), ["x", "s", "t", "lim", "out"],
                          (math.ceil(n / block), 1, 1), (block, 1, 1), rtol=0.0, atol=0.0,
                          pid=pid, kernel_inputs=["x", "s", "t", "lim"])
    scal = {"s": ("f32", float(s)), "t": ("f32", float(t)), "lim": ("i32", int(lim))}
    k0 = meta["kernels"][0]
    k0["args"] = [({"name": a["name"], "dtype": scal[a["name"]][0], "shape": [],
                    "scalar": True, "value": scal[a["name"]][1]} if a["name"] in scal else a)
                  for a in k0["args"]]
    return graph, meta


def center(n: int, threads: int = 128, unroll: int = 4, pid="center"):
    """A two-kernel problem: ``mean = sum(x) / n`` (r03 schedule), then
    ``y = x - mean`` (pointwise) with ``mean`` an intermediate the runner
    chains from the first kernel (``submit.py:112-122``).  Returns
    ``({entry: graph}, meta)``; both kernels read ``x`` from seed 0."""
    g1, m1 = reduce_full(n, threads=threads, mean=True, pid=pid)
    g2, m2 = pointwise(n, unroll, program="center", out="y", entry="k_sub_pointwise",
                       rtol=1e-5, atol=1e-5, pid=pid)
    k1, k2 = dict(m1["kernels"][0]), dict(m2["kernels"][0])
    k1["final"] = False
    k2["args"] = [({"name": a["name"], "dtype": a["dtype"], "shape": a["shape"],
                    "intermediate": True} if a["name"] == "mean" else a) for a in k2["args"]]
    meta = {"id": pid, "code": "", "rtol": 1e-4, "atol": 1e-4, "graph_inputs": ["x"],
            "graph_outputs": ["y"], "kernels": [k1, k2]}
    return {k1["entry"]: g1, k2["entry"]: g2}, meta


def zero_chain(n: int, m: int, c: float = 0.75, block: int = 256, pid="zero_chain"):
    """A two-kernel problem with a delegated zero-init (``TASK.md:95``,
    ``ptxgen/emit.py:1518-1540``): the first kernel computes ``y = x * c``
    and, with a ``ZeroPrologue``, clears ``acc`` (m words) for the second,
    which adds ``y[i]`` into ``acc[i % m]`` with atomic writes and lists
    ``acc`` under ``zero_delegated`` -- so neither the runner nor the second
    kernel clears it.  ``y`` and ``acc`` are intermediates chained from the
    first kernel.  Returns ``({entry: graph}, meta)``."""
    from .ir import ZeroPrologue
    b1 = [load("in0", "x", (V("a0"),)), load("in1", "c", (L(0),)),
          assign("v0", "multiply", "in0", "in1"), write("y", (V("a0"),), "v0")]
    g1, m1 = package("k_scale_zero", "y", [ZeroPrologue(dst="acc", words=m),
                                           tile([ax("a0", n)], b1)],
                     [("x", (n,), "f32", 0)], [("c", float(c))], ("y", (n,), "f32"),
                     ["x", "c", "y", "acc"], (math.ceil(n / block), 1, 1), (block, 1, 1),
                     rtol=1e-5, atol=1e-5, pid=pid, kernel_inputs=["x", "c"])
    k1 = m1["kernels"][0]
    k1["final"] = False
    k1["args"] = [a for a in k1["args"] if a["name"] != "acc"] + [
        {"name": "acc", "dtype": "f32", "shape": [m], "output": True}]
    b2 = [load("in0", "y", (V("a0"),)),
          write("acc", (MOD(V("a0"), L(m)),), "in0", atomic=True)]
    g2, m2 = package("k_accum_into", "acc", [tile([ax("a0", n)], b2)], [], [],
                     ("acc", (m,), "f32"), ["y", "acc"], (math.ceil(n / block), 1, 1),
                     (block, 1, 1), rtol=1e-5, atol=1e-5, pid=pid, kernel_inputs=["y", "acc"])
    g2["nodes"]["acc"]["op_fields"]["zero_delegated"] = ["acc"]
    k2 = m2["kernels"][0]
    k2["args"] = [{"name": "y", "dtype": "f32", "shape": [n], "intermediate": True},
                  {"name": "acc", "dtype": "f32", "shape": [m], "intermediate": True,
                   "output": True}]
    meta = {"id": pid, "code": "", "rtol": 1e-5, "atol": 1e-5, "graph_inputs": ["x"],
            "graph_outputs": ["acc"], "kernels": [k1, k2]}
    return {k1["entry"]: g1, k2["entry"]: g2}, meta


def write_problem(pdir, graphs: dict, meta: dict) -> None:
    """Write ``<entry>.ir.json`` per kernel and ``meta.json`` into ``pdir``."""
    import json
    from pathlib import Path
    pdir = Path(pdir)
    pdir.mkdir(parents=True, exist_ok=True)
    for entry, g in graphs.items():
        (pdir / f"{entry}.ir.json").write_text(json.dumps(g, indent=1))
    (pdir / "meta.json").write_text(json.dumps(meta, indent=1))


def reduce_rows(rows: int, cols: int, threads: int = 128, entry="k_sum_1_reduce",
                pid="reduce_rows", dtype="f32"):
    """Row sum (r04): one row per CTA; ``dtype`` as in ``reduce_full``."""
    dt = datatype(dtype)
    body = [strided("a1", cols, V("a1_co"), L(threads),
                    [load("in0", "x", (V("a0"), V("a1")), dtype=dt),
                     accum("acc0", "in0", "add", ("a1",))])]
    body += _block_combine("a1_co", threads)
    body.append(Cond(cond=EQ(V("a1_co"), L(0)),
                     body=(write("sum_1", (V("a0"),), "acc0", dtype=dt),), else_body=()))
    t = tile([ax("a0", rows), ax("a1_co", threads)], body, block_threads=threads)
    return package(entry, "sum_1", [t], [("x", (rows, cols), dtype, 0)], [],
                   ("sum_1", (rows,), dtype), ["x", "sum_1"], (rows, 1, 1), (threads, 1, 1),
                   rtol=1e-4, atol=1e-4, pid=pid)


def reduce_cols(rows: int, cols: int, block: int = 128, dtype="f64", entry="k_sum_0_reduce",
                pid="reduce_cols"):
    """Column sum with a per-thread accumulator: one column per thread, a
    ``Loop`` over the rows folding into an ``Accum`` of ``dtype`` -- the form
    an f64 reduction takes, since no cross-lane combine is needed."""
    dt = datatype(dtype)
    body = [loop("a0", rows, [load("in0", "x", (V("a0"), V("a1")), dtype=dt),
                              accum("acc0", "in0", "add", ("a0",), dtype=dt)]),
            write("sum_0", (V("a1"),), "acc0", dtype=dt)]
    t = tile([ax("a1", cols)], body)
    return package(entry, "sum_0", [t], [("x", (rows, cols), dtype, 0)], [],
                   ("sum_0", (cols,), dtype), ["x", "sum_0"], (math.ceil(cols / block), 1, 1),
                   (block, 1, 1), rtol=1e-5, atol=1e-5, pid=pid)


# ---------------------------------------------------------------------------
# category 4: fused rows
# ---------------------------------------------------------------------------


def rmsnorm(rows: int, cols: int, eps: float = 1e-5, threads: int = 128,
            entry="k_mean_cbd1de", pid="rmsnorm"):
    body = [strided("a1", cols, V("a1_co"), L(threads),
                    [load("in2", "x", (V("a0"), V("a1"))), assign("v1", "multiply", "in2", "in2"),
                     accum("acc0", "v1", "add", ("a1",))])]
    body += _block_combine("a1_co", threads)
    body += [load("in1", "mean_count", (L(0),)), assign("v0", "reciprocal", "in1"),
             assign("v2", "multiply", "acc0", "v0"), load("in0", "add_c1", (L(0),)),
             assign("v3", "add", "in0", "v2"), assign("v4", "sqrt", "v3"),
             assign("v5", "reciprocal", "v4"),
             strided("a2", cols, V("a1_co"), L(threads),
                     [load("in3", "x", (V("a0"), V("a2"))), assign("v6", "multiply", "in3", "v5"),
                      load("in4", "w", (V("a2"),)), assign("v7", "multiply", "in4", "v6"),
                      write("mul_1", (V("a0"), V("a2")), "v7")])]
    t = tile([ax("a0", rows), ax("a1_co", threads)], body, block_threads=threads)
    return package(entry, "mul_1", [t], [("w", (cols,), "f32", 1), ("x", (rows, cols), "f32", 0)],
                   [("add_c1", eps), ("mean_count", float(cols))],
                   ("mul_1", (rows, cols), "f32"), ["mean_count", "add_c1", "x", "w", "mul_1"],
                   (rows, 1, 1), (threads, 1, 1), rtol=1e-3, atol=1e-4, pid=pid)


def softmax(rows: int, cols: int, threads: int = 128, entry="k_softmax_05263d", pid="softmax"):
    step = [Let(name="one", value=Lf(1.0), dtype=F32),
            load("in0", "x", (V("a0"), V("a1"))),
            assign("in0__gn", "maximum", "acc0", "in0"),
            assign("in0__dg", "subtract", "acc0", "in0__gn"),
            assign("in0__alpha", "exp", "in0__dg"),
            assign("in0__dg_o", "subtract", "in0", "in0__gn"),
            assign("in0__beta", "exp", "in0__dg_o"),
            assign("in0__acc1_sa", "multiply", "acc1", "in0__alpha"),
            assign("in0__acc1_sb", "multiply", "in0__beta", "one"),
            accum("acc1", "in0__acc1_sb", "add", ("a1",), base="in0__acc1_sa"),
            accum("acc0", "in0", "maximum", ("a1",))]
    body = [strided("a1", cols, V("a1_co"), L(threads), step)]
    body += _block_combine("a1_co", threads, states=("acc0", "acc1"), kind="online_softmax")
    body += [assign("v2", "reciprocal", "acc1"),
             strided("a3", cols, V("a1_co"), L(threads),
                     [load("in2", "x", (V("a0"), V("a3"))), assign("v3", "subtract", "in2", "acc0"),
                      assign("v4", "exp", "v3"), assign("v5", "multiply", "v2", "v4"),
                      write("softmax", (V("a0"), V("a3")), "v5")])]
    t = tile([ax("a0", rows), ax("a1_co", threads)], body, block_threads=threads)
    return package(entry, "softmax", [t], [("x", (rows, cols), "f32", 0)], [],
                   ("softmax", (rows, cols), "f32"), ["x", "softmax"], (rows, 1, 1),
                   (threads, 1, 1), rtol=1e-3, atol=1e-5, pid=pid)


def l2norm(rows: int, cols: int, threads: int = 128, entry="k_div_reduce", pid="l2norm"):
    body = [strided("a1", cols, V("a1_co"), L(threads),
                    [load("in0", "x", (V("a0"), V("a1"))), assign("v0", "multiply", "in0", "in0"),
                     accum("acc0", "v0", "add", ("a1",))])]
    body += _block_combine("a1_co", threads)
    body += [assign("v1", "sqrt", "acc0"), assign("v2", "reciprocal", "v1"),
             strided("a2", cols, V("a1_co"), L(threads),
                     [load("in1", "x", (V("a0"), V("a2"))), assign("v3", "multiply", "in1", "v2"),
                      write("div", (V("a0"), V("a2")), "v3")])]
    t = tile([ax("a0", rows), ax("a1_co", threads)], body, block_threads=threads)
    return package(entry, "div", [t], [("x", (rows, cols), "f32", 0)], [],
                   ("div", (rows, cols), "f32"), ["x", "div"], (rows, 1, 1), (threads, 1, 1),
                   rtol=1e-3, atol=1e-4, pid=pid)


# ---------------------------------------------------------------------------
# category 3: matmul
# ---------------------------------------------------------------------------


def _m01_copy(smem, rowbase, src, src_row, src_col, lane_rows, tidl):
    lr = DIV(MUL(tidl, L(4)), L(64))
    lc = MOD(MUL(tidl, L(4)), L(64))
    return CpAsyncCopy(smem=smem, smem_index=(rowbase, L(0)), src=src,
                       src_index=(src_row(lr), src_col(lc)), nbytes=16, swizzle="NONE",
                       lane_index=(lr, lc), lane_rows=lane_rows)


def matmul(m: int, n: int, k: int, entry="k_matmul_2967be", pid="matmul"):
    """C = A.B with the m01 schedule: 32x64 C tile per CTA, K in steps of 64
    through a 3-stage cp.async ring, 16x32 threads with 2x2 outputs each."""
    BM, BN, BK, ST = 32, 64, 64, 3
    if m % BM or n % BN or k % BK or k < 2 * BK:
        raise ValueError("matmul shape must tile by 32x64x64 with K >= 128")
    tidl = ADD(MUL(V("a0_u"), L(32)), V("a1_u"))
    body = [Init(name=f"acc0__c{i}_{j}", identity=0.0, dtype=F32) for i in (0, 1) for j in (0, 1)]
    body += [Smem(name="_a_smem", extents=(BM * ST, BK), dtype="float", align=16),
             Smem(name="_b_smem", extents=(BK * ST, BN), dtype="float", align=16)]

    def a_row(lr):
        return ADD(MUL(V("a0_b"), L(BM)), ADD(lr, L(0)))

    def b_col(lc):
        return ADD(MUL(V("a1_b"), L(BN)), lc)

    for s in range(2):
        koff = L(s * BK)
        abase = L(0) if s == 0 else ADD(MUL(L(s), L(BM)), L(0))
        body.append(_m01_copy("_a_smem", abase, "x0", a_row, lambda lc, ko=koff: ADD(ko, lc),
                               32, tidl))
        for half in (0, 32):
            bbase = L(half) if s == 0 else ADD(MUL(L(s), L(BK)), L(half))
            body.append(_m01_copy("_b_smem", bbase, "x1",
                                  lambda lr, ko=koff, h=half: ADD(ko, ADD(lr, L(h))), b_col, 32,
                                  tidl))
        body.append(CpAsyncCommit())
    kn = TernaryExpr(cond=LT(ADD(V("_ks"), L(2 * BK)), L(k)), if_true=ADD(V("_ks"), L(2 * BK)),
                     if_false=L(k - BK))
    slot = MOD(ADD(DIV(V("_ks"), L(BK)), L(2)), L(ST))
    cur = MOD(DIV(V("_ks"), L(BK)), L(ST))
    inner = [
        _m01_copy("_a_smem", ADD(MUL(slot, L(BM)), L(0)), "x0", a_row,
                  lambda lc: ADD(kn, lc), 32, tidl),
        _m01_copy("_b_smem", ADD(MUL(slot, L(BK)), L(0)), "x1",
                  lambda lr: ADD(kn, ADD(lr, L(0))), b_col, 32, tidl),
        _m01_copy("_b_smem", ADD(MUL(slot, L(BK)), L(32)), "x1",
                  lambda lr: ADD(kn, ADD(lr, L(32))), b_col, 32, tidl),
        CpAsyncCommit(), CpAsyncWait(group=2), Sync(barrier_id=0, count=None, warp=False),
    ]

    def bcol(j):
        return SUB(ADD(ADD(MUL(V("a1_b"), L(BN)), MUL(V("a1_u"), L(2))), L(j)),
                   MUL(V("a1_b"), L(BN)))

    def arow(i):
        return SUB(ADD(ADD(MUL(V("a0_b"), L(BM)), MUL(V("a0_u"), L(2))), L(i)),
                   MUL(V("a0_b"), L(BM)))

    ki = [
        Load(names=("in1__c0_0",), input="_b_smem",
             index=(ADD(MUL(cur, L(BK)), V("_ki")), bcol(0)), dtype=None),
        Load(names=("in0__c0_0",), input="_a_smem",
             index=(ADD(MUL(cur, L(BM)), arow(0)), V("_ki")), dtype=None),
        assign("acc0__v__c0_0", "multiply", "in1__c0_0", "in0__c0_0"),
        accum("acc0__c0_0", "acc0__v__c0_0", "add", ("_ki",)),
        Load(names=("in1__c0_1",), input="_b_smem",
             index=(ADD(MUL(cur, L(BK)), V("_ki")), bcol(1)), dtype=None),
        assign("acc0__v__c0_1", "multiply", "in1__c0_1", "in0__c0_0"),
        accum("acc0__c0_1", "acc0__v__c0_1", "add", ("_ki",)),
        Load(names=("in0__c1_0",), input="_a_smem",
             index=(ADD(MUL(cur, L(BM)), arow(1)), V("_ki")), dtype=None),
        assign("acc0__v__c1_0", "multiply", "in1__c0_0", "in0__c1_0"),
        accum("acc0__c1_0", "acc0__v__c1_0", "add", ("_ki",)),
        assign("acc0__v__c1_1", "multiply", "in1__c0_1", "in0__c1_0"),
        accum("acc0__c1_1", "acc0__v__c1_1", "add", ("_ki",)),
    ]
    inner.append(loop("_ki", BK, ki, unroll=True, seed=False))
    inner.append(Sync(barrier_id=0, count=None, warp=False))
    body.append(strided("_ks", k, L(0), L(BK), inner))

    def orow(i):
        return ADD(ADD(MUL(V("a0_b"), L(BM)), MUL(V("a0_u"), L(2))), L(i))

    def ocol(j):
        return ADD(ADD(MUL(V("a1_b"), L(BN)), MUL(V("a1_u"), L(2))), L(j))

    body.append(write("matmul", (orow(0), ocol(0)), ("acc0__c0_0", "acc0__c0_1")))
    body.append(write("matmul", (orow(1), ocol(0)), ("acc0__c1_0", "acc0__c1_1")))
    t = tile([ax("a0_b", m // BM, win("a0", m)), ax("a1_b", n // BN, win("a1", n)),
              ax("a0_u", 16), ax("a1_u", 32)], body, block_threads=512,
             raster_axes=("a0_b", "a1_b"))
    smem = (BM * ST * BK + BK * ST * BN) * 4
    return package(entry, "matmul", [t], [("x0", (m, k), "f32", 0), ("x1", (k, n), "f32", 1)],
                   [], ("matmul", (m, n), "f32"), ["x1", "x0", "matmul"],
                   ((m // BM) * (n // BN), 1, 1), (512, 1, 1), smem_bytes=smem,
                   rtol=1e-3, atol=1e-3, pid=pid, kernel_inputs=["x1", "x0"])


def matmul_splitk(m: int, n: int, k: int, slice_k: int = 8, entry="k_matmul",
                  pid="matmul_splitk"):
    """C += A.B over K slices of ``slice_k`` with atomic writes (m02): 16x32 C
    tile per CTA, 8x32 threads, 2 rows x 1 column each, K step 8."""
    BM, BN, BK, TH = 16, 32, 8, 256
    if m % BM or n % BN or k % slice_k or slice_k % BK:
        raise ValueError("split-K shape must tile by 16x32 with K slices of multiple of 8")
    tidl = ADD(MUL(V("a0_u"), L(32)), V("a1_u"))
    body = [Init(name="acc0__c0_0", identity=0.0, dtype=F32),
            Init(name="acc0__c1_0", identity=0.0, dtype=F32),
            Smem(name="_a_smem", extents=(BM, BK), dtype="float", align=16),
            Smem(name="_b_smem", extents=(BK, BN), dtype="float", align=16)]
    fa4 = MUL(V("_fa"), L(4))
    fb4 = MUL(V("_fb"), L(4))
    ca = CpAsyncCopy(smem="_a_smem", smem_index=(DIV(fa4, L(BK)), MOD(fa4, L(BK))), src="x0",
                     src_index=(ADD(MUL(V("a0_b"), L(BM)), DIV(fa4, L(BK))),
                                ADD(MUL(V("_a2_ks"), L(slice_k)), ADD(V("_ks"), MOD(fa4, L(BK))))),
                     nbytes=16, swizzle="NONE", lane_index=None, lane_rows=0)
    cb = CpAsyncCopy(smem="_b_smem", smem_index=(DIV(fb4, L(BN)), MOD(fb4, L(BN))), src="x1",
                     src_index=(ADD(MUL(V("_a2_ks"), L(slice_k)), ADD(V("_ks"), DIV(fb4, L(BN)))),
                                ADD(MUL(V("a1_b"), L(BN)), MOD(fb4, L(BN)))),
                     nbytes=16, swizzle="NONE", lane_index=None, lane_rows=0)

    def bcol():
        return SUB(ADD(ADD(MUL(V("a1_b"), L(BN)), MUL(V("a1_u"), L(1))), L(0)),
                   MUL(V("a1_b"), L(BN)))

    def arow(i):
        return SUB(ADD(ADD(MUL(V("a0_b"), L(BM)), MUL(V("a0_u"), L(2))), L(i)),
                   MUL(V("a0_b"), L(BM)))

    ki = [Load(names=("in1__c0_0",), input="_b_smem", index=(V("_ki"), bcol()), dtype=None),
          Load(names=("in0__c0_0",), input="_a_smem", index=(arow(0), V("_ki")), dtype=None),
          assign("acc0__v__c0_0", "multiply", "in1__c0_0", "in0__c0_0"),
          accum("acc0__c0_0", "acc0__v__c0_0", "add", ("_ki",)),
          Load(names=("in0__c1_0",), input="_a_smem", index=(arow(1), V("_ki")), dtype=None),
          assign("acc0__v__c1_0", "multiply", "in1__c0_0", "in0__c1_0"),
          accum("acc0__c1_0", "acc0__v__c1_0", "add", ("_ki",))]
    ks = [strided("_fa", BM * BK // 4, tidl, L(TH), [ca]),
          strided("_fb", BK * BN // 4, tidl, L(TH), [cb]),
          CpAsyncCommit(), CpAsyncWait(group=0), Sync(barrier_id=0, count=None, warp=False),
          loop("_ki", BK, ki, unroll=True, seed=False),
          Sync(barrier_id=0, count=None, warp=False)]
    body.append(strided("_ks", slice_k, L(0), L(BK), ks))

    def orow(i):
        return ADD(ADD(MUL(V("a0_b"), L(BM)), MUL(V("a0_u"), L(2))), L(i))

    ocol = ADD(ADD(MUL(V("a1_b"), L(BN)), MUL(V("a1_u"), L(1))), L(0))
    body.append(write("matmul", (orow(0), ocol), "acc0__c0_0", atomic=True))
    body.append(write("matmul", (orow(1), ocol), "acc0__c1_0", atomic=True))
    slices = k // slice_k
    t = tile([ax("_a2_ks", slices), ax("a0_b", m // BM, win("a0", m)),
              ax("a1_b", n // BN, win("a1", n)), ax("a0_u", 8), ax("a1_u", 32)], body,
             block_threads=TH, raster_axes=("a0_b", "a1_b"))
    return package(entry, "matmul", [t], [("x0", (m, k), "f32", 0), ("x1", (k, n), "f32", 1)],
                   [], ("matmul", (m, n), "f32"), ["x1", "x0", "matmul"],
                   (slices * (m // BM) * (n // BN), 1, 1), (TH, 1, 1),
                   zero_outputs=["matmul"], rtol=1e-3, atol=1e-3, pid=pid,
                   kernel_inputs=["x1", "x0"])


# ---------------------------------------------------------------------------
# category 5: attention
# ---------------------------------------------------------------------------


def _online_step(score_name: str, vload: Load | None, key_axis: str, cell=(0, 0),
                 vname: str = "in7__bc0"):
    """The per-key online-softmax update of a02 for one output element; with
    ``cell`` = (r, c) the update of output (row r, column c) of a01's
    register tile, whose ``v`` row is loaded once, in cell (0, 0)."""
    s = f"__c{cell[0]}_{cell[1]}"
    return [
        assign(f"v4{s}", "multiply", score_name, "v1"),
        Let(name=f"one{s}", value=Lf(1.0), dtype=F32),
        assign(f"v4__gn{s}", "maximum", f"acc1{s}", f"v4{s}"),
        assign(f"v4__dg{s}", "subtract", f"acc1{s}", f"v4__gn{s}"),
        assign(f"v4__alpha{s}", "exp", f"v4__dg{s}"),
        assign(f"v4__dg_o{s}", "subtract", f"v4{s}", f"v4__gn{s}"),
        assign(f"v4__beta{s}", "exp", f"v4__dg_o{s}"),
        assign(f"v4__acc3_sa{s}", "multiply", f"acc3{s}", f"v4__alpha{s}"),
        assign(f"v4__acc3_sb{s}", "multiply", f"one{s}", f"v4__beta{s}"),
        accum(f"acc3{s}", f"v4__acc3_sb{s}", "add", (key_axis,), base=f"v4__acc3_sa{s}"),
        assign(f"v4__acc5__sum_sa{s}", "multiply", f"acc5__sum{s}", f"v4__alpha{s}"),
    ] + ([vload] if vload is not None else []) + [
        assign(f"v4__acc5__sum_sb{s}", "multiply", vname, f"v4__beta{s}"),
        accum(f"acc5__sum{s}", f"v4__acc5__sum_sb{s}", "add", (key_axis,),
              base=f"v4__acc5__sum_sa{s}"),
        accum(f"acc1{s}", f"v4{s}", "maximum", (key_axis,)),
    ]


def attention(s: int, d: int, scale_div: float | None = None,
              entry="k_matmul_softmax_reduce_6f0029", pid="attention"):
    """softmax(q.kt / c) . v for one head, q,v [S,D], kt [D,S] (a02)."""
    if d % 32:
        raise ValueError("head dim must be a multiple of 32")
    c = float(scale_div) if scale_div is not None else math.sqrt(d)
    row = ADD(ADD(MUL(V("a0_b"), L(1)), MUL(V("a0_u"), L(1))), L(0))
    col = ADD(ADD(MUL(V("a5_b"), L(32)), MUL(V("a5_u"), L(1))), L(0))
    dot = loop("a2", d, [load("in2__ar0", "q", (row, V("a2"))),
                         load("in1__ar0", "kt", (V("a2"), V("a1"))),
                         assign("v3__ar0", "multiply", "in1__ar0", "in2__ar0"),
                         accum("acc0__ar0", "v3__ar0", "add", ("a2",))])
    vload = load("in7__bc0", "v", (V("a1"), col))
    body = [load("in0", "div_c1", (L(0),)), assign("v1", "reciprocal", "in0"),
            loop("a1", s, [dot] + _online_step("acc0__ar0", vload, "a1")),
            assign("v9__c0_0", "reciprocal", "acc3__c0_0"),
            assign("acc5__c0_0", "multiply", "acc5__sum__c0_0", "v9__c0_0"),
            write("matmul_1", (row, col), "acc5__c0_0")]
    t = tile([ax("a0_b", s, win("a0", s)), ax("a5_b", d // 32, win("a5", d)),
              ax("a0_u", 1), ax("a5_u", 32)], body, block_threads=32,
             raster_axes=("a0_b", "a5_b"), raster_group=8)
    return package(entry, "matmul_1", [t],
                   [("kt", (d, s), "f32", 1), ("q", (s, d), "f32", 0), ("v", (s, d), "f32", 2)],
                   [("div_c1", c)], ("matmul_1", (s, d), "f32"),
                   ["div_c1", "q", "kt", "v", "matmul_1"], (s * d // 32, 1, 1), (32, 1, 1),
                   rtol=1e-3, atol=1e-4, pid=pid)


def attention_tiled(s: int, d: int, scale_div: float | None = None,
                    entry="k_matmul_softmax_reduce_b55365", pid="attention_tiled"):
    """softmax(q.kt / c) . v for one head (a01,
    ``problems/a01_attention/k_matmul_softmax_reduce_b55365.ir.json``): the
    a02 online softmax with
    each of a CTA's 128 threads holding a 4 x 2 register tile of the output
    (8 x 16 threads over a 32 x 32 block), one q.kt dot product per tile row,
    one paired ``v`` load per key and the key loop unrolled."""
    if s % 32 or d % 32:
        raise ValueError("sequence length and head dim must be multiples of 32")
    c = float(scale_div) if scale_div is not None else math.sqrt(d)
    rows = [ADD(ADD(MUL(V("a0_b"), L(32)), MUL(V("a0_u"), L(4))), L(r)) for r in range(4)]
    cols = [ADD(ADD(MUL(V("a5_b"), L(32)), MUL(V("a5_u"), L(2))), L(j)) for j in range(2)]
    key = []
    for r in range(4):
        key.append(loop("a2", d, [load(f"in2__ar{r}", "q", (rows[r], V("a2"))),
                                  load(f"in1__ar{r}", "kt", (V("a2"), V("a1"))),
                                  assign(f"v3__ar{r}", "multiply", f"in1__ar{r}", f"in2__ar{r}"),
                                  accum(f"acc0__ar{r}", f"v3__ar{r}", "add", ("a2",))]))
    vload = load(("in7__bc0", "in7__bc1"), "v", (V("a1"), cols[0]))
    for r in range(4):
        for j in range(2):
            key += _online_step(f"acc0__ar{r}", vload if (r, j) == (0, 0) else None, "a1",
                                cell=(r, j), vname=f"in7__bc{j}")
    body = [load("in0", "div_c1", (L(0),)), assign("v1", "reciprocal", "in0"),
            loop("a1", s, key, unroll=True)]
    for r in range(4):
        for j in range(2):
            cs = f"__c{r}_{j}"
            body += [assign(f"v9{cs}", "reciprocal", f"acc3{cs}"),
                     assign(f"acc5{cs}", "multiply", f"acc5__sum{cs}", f"v9{cs}"),
                     write("matmul_1", (rows[r], cols[j]), f"acc5{cs}")]
    t = tile([ax("a0_b", s // 32, win("a0", s)), ax("a5_b", d // 32, win("a5", d)),
              ax("a0_u", 8), ax("a5_u", 16)], body, block_threads=128,
             raster_axes=("a0_b", "a5_b"))
    return package(entry, "matmul_1", [t],
                   [("kt", (d, s), "f32", 1), ("q", (s, d), "f32", 0), ("v", (s, d), "f32", 2)],
                   [("div_c1", c)], ("matmul_1", (s, d), "f32"),
                   ["div_c1", "q", "kt", "v", "matmul_1"], ((s // 32) * (d // 32), 1, 1),
                   (128, 1, 1), rtol=1e-3, atol=1e-4, pid=pid)


def attention_bhsd(b: int, h: int, s: int, d: int, dtype: str = "f32",
                   entry="k_attention_bhsd", pid="attention_bhsd"):
    """softmax(q.k^T / sqrt(d)) . v over ``[B, H, S, D]`` q, k, v (k NOT
    transposed), one output element per thread; the a02 schedule with batch
    and head axes added.  ``dtype='bf16'`` stores q, k, v and the output as
    bf16 while the arithmetic stays f32."""
    if d % 32:
        raise ValueError("head dim must be a multiple of 32")
    dt = datatype(dtype)
    row = ADD(ADD(MUL(V("a0_b"), L(1)), MUL(V("a0_u"), L(1))), L(0))
    col = ADD(ADD(MUL(V("a5_b"), L(32)), MUL(V("a5_u"), L(1))), L(0))
    bh = (V("ab"), V("ah"))
    dot = loop("a2", d, [load("in2__ar0", "q", bh + (row, V("a2"))),
                         load("in1__ar0", "k", bh + (V("a1"), V("a2"))),
                         assign("v3__ar0", "multiply", "in1__ar0", "in2__ar0"),
                         accum("acc0__ar0", "v3__ar0", "add", ("a2",))])
    vload = load("in7__bc0", "v", bh + (V("a1"), col))
    body = [load("in0", "div_c1", (L(0),)), assign("v1", "reciprocal", "in0"),
            loop("a1", s, [dot] + _online_step("acc0__ar0", vload, "a1")),
            assign("v9__c0_0", "reciprocal", "acc3__c0_0"),
            assign("acc5__c0_0", "multiply", "acc5__sum__c0_0", "v9__c0_0"),
            write("out", bh + (row, col), "acc5__c0_0")]
    t = tile([ax("ab", b), ax("ah", h), ax("a0_b", s, win("a0", s)),
              ax("a5_b", d // 32, win("a5", d)), ax("a0_u", 1), ax("a5_u", 32)], body,
             block_threads=32, raster_axes=("a0_b", "a5_b"), raster_group=8)
    shp = (b, h, s, d)
    tol = (2e-2, 2e-2) if dtype == "bf16" else (1e-3, 1e-4)
    return package(entry, "out", [t],
                   [("k", shp, dtype, 1), ("q", shp, dtype, 0), ("v", shp, dtype, 2)],
                   [("div_c1", math.sqrt(d))], ("out", shp, dtype),
                   ["div_c1", "q", "k", "v", "out"], (b * h * s * d // 32, 1, 1), (32, 1, 1),
                   rtol=tol[0], atol=tol[1], pid=pid)


# ---------------------------------------------------------------------------
# the benchmark configurations
# ---------------------------------------------------------------------------

# ---------------------------------------------------------------------------
# bulk-async transport: box copies into shared memory under an mbarrier
# ---------------------------------------------------------------------------

_SMEM_C = {"f32": "float", "f16": "half", "bf16": "__nv_bfloat16", "f64": "double"}
_EB = {"f32": 4, "f16": 2, "bf16": 2, "f64": 8}
_MBAR = "unsigned long long"


def _tma_issue(tid, loads, nbytes):
    """Thread ``tid == 0`` announces ``nbytes`` on mbarrier ``bar`` slot 0 and
    issues the box copies ``loads``."""
    return Cond(cond=EQ(tid, L(0)),
                body=(MbarrierArriveExpectTx(mbar="bar", bytes_=L(nbytes), slot=L(0)),) +
                tuple(loads), else_body=())


def _swizzled(e, dtype: str, swizzle: str):
    """Shared-memory element index of box element ``e`` under a TMA swizzle:
    byte o moves to o ^ (((o >> 7) & m) << 4)."""
    span = {"NONE": 0, "B32": 32, "B64": 64, "B128": 128}[swizzle]
    if not span:
        return e
    eb = _EB[dtype]
    sh, cs = 7 - int(math.log2(eb)), 4 - int(math.log2(eb))
    rowbits = _b("&")(_b(">>")(e, L(sh)), L(span // 16 - 1))
    return _b("^")(e, _b("<<")(rowbits, L(cs)))


def tma_box_copy(rows: int, cols: int, br: int, bc: int, nbr: int, nbc: int, dtype="f32",
                 swizzle="NONE", off_r=0, off_c=0, threads=128, maxnreg=None, view3=False,
                 entry="k_tma_box_copy", pid="tma_box_copy"):
    """out[i*br + r, j*bc + c] = x[i*br + off_r + r, j*bc + off_c + c] (zero
    outside x): one CTA per (i, j) box; thread 0 initialises the mbarrier,
    announces the bytes and issues the box copy; every thread waits for phase
    0, then copies the box out of shared memory (undoing the swizzle).
    ``view3``: the same copy through a rank-3 view (rows/2, 2, cols) of x
    and a (br/2, 2, bc) box (rows, br and off_r even)."""
    eb = _EB[dtype]
    t = V("t")
    r0 = ADD(MUL(V("bi"), L(br)), L(off_r))
    c0 = ADD(MUL(V("bj"), L(bc)), L(off_c))
    if view3:
        if rows % 2 or br % 2 or off_r % 2:
            raise ValueError("view3 needs even rows, br and off_r")
        view, box = (rows // 2, 2, cols), (br // 2, 2, bc)
        coords = (ADD(MUL(V("bi"), L(br // 2)), L(off_r // 2)), L(0), c0)
    else:
        view, box, coords = (rows, cols), (br, bc), (r0, c0)
    body = [TmaDescriptor(name="dx", src_buf="x0", src_shape=view, box_extents=box,
                          swizzle=swizzle, dtype=dtype),
            Smem(name="tile", extents=(br * bc,), dtype=_SMEM_C[dtype], align=1024),
            Smem(name="bar", extents=(1,), dtype=_MBAR, align=8)]
    if maxnreg:
        body.append(SetMaxNReg(count=maxnreg, direction="dec"))
    body += [
        Cond(cond=EQ(t, L(0)), body=(MbarrierInit(mbar="bar", count=L(1), slot=L(0)),),
             else_body=()),
        Sync(barrier_id=0, count=None, warp=False),
        _tma_issue(t, [TmaLoad(smem="tile", smem_index=L(0), desc="dx", coords=coords,
                               mbar="bar", mbar_slot=L(0))], br * bc * eb),
        MbarrierWait(mbar="bar", phase=L(0), slot=L(0)),
        strided("e", br * bc, t, L(threads), [
            Load(names=("v",), input="tile", index=(_swizzled(V("e"), dtype, swizzle),),
                 dtype=None),
            write("out", (ADD(MUL(V("bi"), L(br)), DIV(V("e"), L(bc))),
                          ADD(MUL(V("bj"), L(bc)), MOD(V("e"), L(bc)))), "v",
                  dtype=datatype(dtype))]),
    ]
    tl = tile([ax("bi", nbr), ax("bj", nbc), ax("t", threads)], body, block_threads=threads)
    return package(entry, "copy", [tl], [("x0", (rows, cols), dtype, 0)], [],
                   ("out", (nbr * br, nbc * bc), dtype), ["x0", "out"], (nbr * nbc, 1, 1),
                   (threads, 1, 1), rtol=0.0, atol=0.0, pid=pid)


def matmul_tma(m: int, n: int, k: int, entry="k_matmul_tma", pid="matmul_tma"):
    """C = A.B with m02's 16x32 tile, 8x32 threads and K step of 8, each K
    step's A (16x8) and B (8x32) boxes brought by two box copies that
    complete on one mbarrier (phase = step number); the products are summed
    in K order per output as in m02, and C is written once (no slices)."""
    BM, BN, BK, TH = 16, 32, 8, 256
    if m % BM or n % BN or k % BK:
        raise ValueError("matmul_tma shape must tile by 16x32 with K a multiple of 8")
    tidl = ADD(MUL(V("a0_u"), L(32)), V("a1_u"))
    body = [Init(name="acc0__c0_0", identity=0.0, dtype=F32),
            Init(name="acc0__c1_0", identity=0.0, dtype=F32),
            TmaDescriptor(name="dA", src_buf="x0", src_shape=(m, k), box_extents=(BM, BK),
                          swizzle="NONE", dtype="f32"),
            TmaDescriptor(name="dB", src_buf="x1", src_shape=(k, n), box_extents=(BK, BN),
                          swizzle="NONE", dtype="f32"),
            Smem(name="_a_smem", extents=(BM, BK), dtype="float", align=128),
            Smem(name="_b_smem", extents=(BK, BN), dtype="float", align=128),
            Smem(name="bar", extents=(1,), dtype=_MBAR, align=8),
            Cond(cond=EQ(tidl, L(0)), body=(MbarrierInit(mbar="bar", count=L(1), slot=L(0)),),
                 else_body=()),
            Sync(barrier_id=0, count=None, warp=False)]

    def bcol():
        return V("a1_u")

    def arow(i):
        return ADD(MUL(V("a0_u"), L(2)), L(i))

    ki = [Load(names=("in1__c0_0",), input="_b_smem", index=(V("_ki"), bcol()), dtype=None),
          Load(names=("in0__c0_0",), input="_a_smem", index=(arow(0), V("_ki")), dtype=None),
          assign("acc0__v__c0_0", "multiply", "in1__c0_0", "in0__c0_0"),
          accum("acc0__c0_0", "acc0__v__c0_0", "add", ("_ki",)),
          Load(names=("in0__c1_0",), input="_a_smem", index=(arow(1), V("_ki")), dtype=None),
          assign("acc0__v__c1_0", "multiply", "in1__c0_0", "in0__c1_0"),
          accum("acc0__c1_0", "acc0__v__c1_0", "add", ("_ki",))]
    copies = [TmaLoad(smem="_a_smem", smem_index=L(0), desc="dA",
                      coords=(MUL(V("a0_b"), L(BM)), V("_ks")), mbar="bar", mbar_slot=L(0)),
              TmaLoad(smem="_b_smem", smem_index=L(0), desc="dB",
                      coords=(V("_ks"), MUL(V("a1_b"), L(BN))), mbar="bar", mbar_slot=L(0))]
    ks = [_tma_issue(tidl, copies, (BM * BK + BK * BN) * 4),
          MbarrierWait(mbar="bar", phase=DIV(V("_ks"), L(BK)), slot=L(0)),
          loop("_ki", BK, ki, unroll=True, seed=False),
          Sync(barrier_id=0, count=None, warp=False)]
    body.append(strided("_ks", k, L(0), L(BK), ks))

    def orow(i):
        return ADD(ADD(MUL(V("a0_b"), L(BM)), MUL(V("a0_u"), L(2))), L(i))

    ocol = ADD(MUL(V("a1_b"), L(BN)), V("a1_u"))
    body.append(write("matmul", (orow(0), ocol), "acc0__c0_0"))
    body.append(write("matmul", (orow(1), ocol), "acc0__c1_0"))
    t = tile([ax("a0_b", m // BM, win("a0", m)), ax("a1_b", n // BN, win("a1", n)),
              ax("a0_u", 8), ax("a1_u", 32)], body, block_threads=TH)
    return package(entry, "matmul", [t], [("x0", (m, k), "f32", 0), ("x1", (k, n), "f32", 1)],
                   [], ("matmul", (m, n), "f32"), ["x1", "x0", "matmul"],
                   ((m // BM) * (n // BN), 1, 1), (TH, 1, 1), rtol=1e-3, atol=1e-3, pid=pid,
                   kernel_inputs=["x1", "x0"])


def matmul_mma(m: int, n: int, k: int, dtype="bf16", m_valid=None, n_valid=None,
               promote_every=0, entry="k_matmul_mma", pid="matmul_mma"):
    """C = A.B (A [m, k], B [k, n] in bf16 or f16, C in f32) on m16n8k16
    fragments: a 64 x 32 C tile per CTA of four warps, warp w owning rows
    16w..16w+15 as four 16 x 8 cells; per K step of 16 thread 0 brings the
    A (64 x 16) and B (16 x 32) boxes with two box copies on one mbarrier,
    each warp loads its A cell and the four B cells (``ldmatrix``, B [K][N]
    transposed) and accumulates four products.  ``m_valid`` / ``n_valid``:
    rows and columns of C stored (the guards of ``RegStore``).
    ``promote_every`` (f16 only): the products accumulate in f16 cells that
    ``FragmentPromote`` adds into the f32 cells every that many K steps and
    once after the loop."""
    if promote_every and dtype != "f16":
        raise ValueError("f16 accumulators take f16 operands")
    BM, BN, BK, TH = 64, 32, 16, 128
    if m % BM or n % BN or k % BK:
        raise ValueError("matmul_mma shape must tile by 64x32 with K a multiple of 16")
    t = V("t")
    nb = (BM * BK + BK * BN) * 2
    body = [TmaDescriptor(name="dA", src_buf="x0", src_shape=(m, k), box_extents=(BM, BK),
                          swizzle="NONE", dtype=dtype),
            TmaDescriptor(name="dB", src_buf="x1", src_shape=(k, n), box_extents=(BK, BN),
                          swizzle="NONE", dtype=dtype),
            Smem(name="_a_smem", extents=(BM, BK), dtype=_SMEM_C[dtype], align=128),
            Smem(name="_b_smem", extents=(BK, BN), dtype=_SMEM_C[dtype], align=128),
            Smem(name="bar", extents=(1,), dtype=_MBAR, align=8),
            RegFragment(name="fa", role="a", shape="m16n8k16", dtype=dtype, count=1, nregs=4),
            RegFragment(name="fb", role="b", shape="m16n8k16", dtype=dtype, count=4, nregs=2),
            RegFragment(name="fc", role="c", shape="m16n8k16", dtype="f32", count=4, nregs=4),
            Cond(cond=EQ(t, L(0)), body=(MbarrierInit(mbar="bar", count=L(1), slot=L(0)),),
                 else_body=()),
            Sync(barrier_id=0, count=None, warp=False)]
    acc = "fc"
    if promote_every:
        body.insert(-2, RegFragment(name="fh", role="c", shape="m16n8k16", dtype="f16", count=4,
                                    nregs=2))
        acc = "fh"
    copies = [TmaLoad(smem="_a_smem", smem_index=L(0), desc="dA",
                      coords=(MUL(V("bm"), L(BM)), V("_ks")), mbar="bar", mbar_slot=L(0)),
              TmaLoad(smem="_b_smem", smem_index=L(0), desc="dB",
                      coords=(V("_ks"), MUL(V("bn"), L(BN))), mbar="bar", mbar_slot=L(0))]
    ks = [_tma_issue(t, copies, nb),
          MbarrierWait(mbar="bar", phase=DIV(V("_ks"), L(BK)), slot=L(0)),
          LdmatrixLoad(frag="fa", src_buffer="_a_smem", src_index=(MUL(V("warp"), L(16)), L(0)),
                       role="a")]
    for j in range(BN // 8):
        ks += [LdmatrixLoad(frag="fb", src_buffer="_b_smem", src_index=(L(0), L(8 * j)),
                            role="b", b_trans=True, fragment_index=L(j)),
               MmaSyncPtx(c_frag=f"{acc}[{j}]", a_frag="fa", b_frag=f"fb[{j}]",
                          shape="m16n8k16", ab_dtype=dtype,
                          c_dtype="f16" if promote_every else "f32")]
    promote = [FragmentPromote(dst=f"fc[{j}]", src=f"fh[{j}]") for j in range(BN // 8)]
    if promote_every:
        step = DIV(V("_ks"), L(BK))
        ks.append(Cond(cond=EQ(MOD(step, L(promote_every)), L(promote_every - 1)),
                       body=tuple(promote), else_body=()))
    ks.append(Sync(barrier_id=0, count=None, warp=False))
    body.append(strided("_ks", k, L(0), L(BK), ks))
    if promote_every:
        body += promote
    for j in range(BN // 8):
        body.append(RegStore(dst_buffer="matmul",
                             dst_index=(ADD(MUL(V("bm"), L(BM)), MUL(V("warp"), L(16))),
                                        ADD(MUL(V("bn"), L(BN)), L(8 * j))),
                             frag="fc", fragment_index=L(j),
                             m_guard=None if m_valid is None else L(m_valid),
                             n_guard=None if n_valid is None else L(n_valid)))
    tl = tile([ax("bm", m // BM), ax("bn", n // BN), ax("t", TH)], body, block_threads=TH)
    return package(entry, "matmul", [tl], [("x0", (m, k), dtype, 0), ("x1", (k, n), dtype, 1)],
                   [], ("matmul", (m, n), "f32"), ["x0", "x1", "matmul"],
                   ((m // BM) * (n // BN), 1, 1), (TH, 1, 1), rtol=1e-3, atol=1e-3, pid=pid)


def matmul_wgmma(m: int, n: int, k: int, dtype="bf16", bn=64, groups=1, swizzle="B128",
                 m_valid=None, n_valid=None, entry="k_matmul_wgmma", pid="matmul_wgmma"):
    """C[m, n] = sum_k A[m, k] * Bt[n, k] (A, Bt bf16 or f16, C f32): each
    warpgroup owns a 64 x ``bn`` C tile (``groups`` warpgroups per CTA, tiles
    stacked along M); per K step of 64 thread 0 brings A (64*groups x 64)
    and Bt (bn x 64) with two box copies (``swizzle``), then each group
    issues four k16 products from descriptors that advance 32 bytes along
    the swizzled rows, commits and waits."""
    BK, TH = 64, 128 * groups
    BM = 64 * groups
    if m % BM or n % bn or k % BK:
        raise ValueError("matmul_wgmma shape must tile by (64*groups) x bn x 64")
    t = V("t")
    nb = (BM * BK + bn * BK) * 2
    cshape = f"m64n{bn}k16"
    body = [TmaDescriptor(name="dA", src_buf="x0", src_shape=(m, k), box_extents=(BM, BK),
                          swizzle=swizzle, dtype=dtype),
            TmaDescriptor(name="dB", src_buf="x1", src_shape=(n, k), box_extents=(bn, BK),
                          swizzle=swizzle, dtype=dtype),
            Smem(name="_a_smem", extents=(BM, BK), dtype=_SMEM_C[dtype], align=1024),
            Smem(name="_b_smem", extents=(bn, BK), dtype=_SMEM_C[dtype], align=1024),
            Smem(name="bar", extents=(1,), dtype=_MBAR, align=8),
            RegFragment(name="fc", role="c", shape=cshape, dtype="f32", count=1,
                        nregs=bn // 2),
            Cond(cond=EQ(t, L(0)), body=(MbarrierInit(mbar="bar", count=L(1), slot=L(0)),),
                 else_body=()),
            Sync(barrier_id=0, count=None, warp=False)]
    copies = [TmaLoad(smem="_a_smem", smem_index=L(0), desc="dA",
                      coords=(MUL(V("bm"), L(BM)), V("_ks")), mbar="bar", mbar_slot=L(0)),
              TmaLoad(smem="_b_smem", smem_index=L(0), desc="dB",
                      coords=(MUL(V("bn"), L(bn)), V("_ks")), mbar="bar", mbar_slot=L(0))]
    grp = DIV(V("t"), L(128))
    ks = [_tma_issue(t, copies, nb),
          MbarrierWait(mbar="bar", phase=DIV(V("_ks"), L(BK)), slot=L(0)),
          WgmmaFence()]
    for j in range(BK // 16):
        ks += [WgmmaDescriptor(name="da", smem="_a_smem",
                               smem_index=ADD(MUL(grp, L(64 * BK)), L(16 * j)),
                               swizzle=swizzle, lbo_bytes=16, sbo_bytes=1024),
               WgmmaDescriptor(name="db", smem="_b_smem", smem_index=L(16 * j), swizzle=swizzle,
                               lbo_bytes=16, sbo_bytes=1024),
               WgmmaMma(c_frags="fc", b_desc="db", shape=cshape, ab_dtype=dtype, a_desc="da",
                        scale_d=BinaryExpr(op=">", left=ADD(V("_ks"), L(16 * j)), right=L(0)))]
    ks += [WgmmaCommit(), WgmmaWait(group=0), Sync(barrier_id=0, count=None, warp=False)]
    body.append(strided("_ks", k, L(0), L(BK), ks))
    body.append(RegStore(dst_buffer="matmul",
                         dst_index=(ADD(MUL(V("bm"), L(BM)), MUL(grp, L(64))),
                                    MUL(V("bn"), L(bn))),
                         frag="fc", shape=cshape,
                         m_guard=None if m_valid is None else L(m_valid),
                         n_guard=None if n_valid is None else L(n_valid)))
    tl = tile([ax("bm", m // BM), ax("bn", n // bn), ax("t", TH)], body, block_threads=TH)
    return package(entry, "matmul", [tl], [("x0", (m, k), dtype, 0), ("x1", (n, k), dtype, 1)],
                   [], ("matmul", (m, n), "f32"), ["x0", "x1", "matmul"],
                   ((m // BM) * (n // bn), 1, 1), (TH, 1, 1), rtol=1e-3, atol=1e-3, pid=pid)


def attention_mma(bh: int, s: int, d: int, dtype="bf16", entry="k_attention_mma",
                  pid="attention_mma"):
    """out = softmax(q k^T / sqrt(d)) v per batch*head (q, k, v [bh, s, d] in
    bf16 or f16, out f32), flash style on m16n8k16 fragments: a CTA of four
    warps owns 64 query rows (16 per warp, Q cells loaded once); per block
    of 64 keys thread 0 brings K and V with two box copies, each warp forms
    its 16 x 64 S in eight c cells, takes the row max (``FragmentRowReduce``),
    rescales its running max, sum and O cells (``FragmentApply`` with row
    pairs), exponentiates S in place, repacks it into four A cells
    (``FragmentRepack``) and accumulates P V; O / l is stored at the end."""
    BQ, BKV, TH = 64, 64, 128
    if s % BQ or d % 16 or d > 128:
        raise ValueError("attention_mma needs s a multiple of 64 and d a multiple of 16, <= 128")
    t = V("t")
    nk, no = d // 16, d // 8
    row0 = ADD(MUL(V("bh"), L(s)), MUL(V("qb"), L(BQ)))
    body = [TmaDescriptor(name=f"d{x}", src_buf=x, src_shape=(bh * s, d), box_extents=(BQ, d),
                          swizzle="NONE", dtype=dtype) for x in ("q", "k", "v")]
    body += [Smem(name=f"_{x}", extents=(BQ, d), dtype=_SMEM_C[dtype], align=128)
             for x in ("q", "k", "v")]
    body += [Smem(name="bar", extents=(1,), dtype=_MBAR, align=8),
             RegFragment(name="fq", role="a", shape="m16n8k16", dtype=dtype, count=nk, nregs=4),
             RegFragment(name="fk", role="b", shape="m16n8k16", dtype=dtype, count=1, nregs=2),
             RegFragment(name="fv", role="b", shape="m16n8k16", dtype=dtype, count=1, nregs=2),
             RegFragment(name="fp", role="a", shape="m16n8k16", dtype=dtype, count=4, nregs=4),
             RegFragment(name="fo", role="c", shape="m16n8k16", dtype="f32", count=no, nregs=4),
             Let(name="sc", value=Lf(1.0 / math.sqrt(d)), dtype=F32)]
    for nm, v0 in (("m_t", -1e30), ("m_b", -1e30), ("l_t", 0.0), ("l_b", 0.0)):
        body.append(Init(name=nm, identity=v0, dtype=F32))
    body += [Cond(cond=EQ(t, L(0)), body=(MbarrierInit(mbar="bar", count=L(1), slot=L(0)),),
                  else_body=()),
             Sync(barrier_id=0, count=None, warp=False),
             _tma_issue(t, [TmaLoad(smem="_q", smem_index=L(0), desc="dq", coords=(row0, L(0)),
                                    mbar="bar", mbar_slot=L(0))], BQ * d * 2),
             MbarrierWait(mbar="bar", phase=L(0), slot=L(0))]
    body += [LdmatrixLoad(frag="fq", src_buffer="_q", src_index=(MUL(V("warp"), L(16)), L(16 * i)),
                          role="a", fragment_index=L(i)) for i in range(nk)]
    krow = ADD(MUL(V("bh"), L(s)), V("_j"))
    blk = [_tma_issue(t, [TmaLoad(smem=f"_{x}", smem_index=L(0), desc=f"d{x}",
                                  coords=(krow, L(0)), mbar="bar", mbar_slot=L(0))
                          for x in ("k", "v")], 2 * BKV * d * 2),
           MbarrierWait(mbar="bar", phase=ADD(L(1), DIV(V("_j"), L(BKV))), slot=L(0)),
           RegFragment(name="fs", role="c", shape="m16n8k16", dtype="f32", count=8, nregs=4)]
    for n in range(BKV // 8):
        for i in range(nk):
            blk += [LdmatrixLoad(frag="fk", src_buffer="_k", src_index=(L(8 * n), L(16 * i)),
                                 role="b", b_trans=False),
                    MmaSyncPtx(c_frag=f"fs[{n}]", a_frag=f"fq[{i}]", b_frag="fk",
                               shape="m16n8k16", ab_dtype=dtype, c_dtype="f32")]
    cells = tuple(f"fs[{n}]" for n in range(BKV // 8))
    blk += [FragmentApply(out=c, op="multiply", args=("sc",), kinds=("scalar",)) for c in cells]
    blk.append(FragmentRowReduce(top="bm_t", bot="bm_b", frags=cells, op="maximum"))
    for h in ("t", "b"):
        blk += [assign(f"mn_{h}", "maximum", f"m_{h}", f"bm_{h}"),
                assign(f"dm_{h}", "subtract", f"m_{h}", f"mn_{h}"),
                assign(f"al_{h}", "exp", f"dm_{h}")]
    blk += [FragmentApply(out=c, op="subtract", args=(("mn_t", "mn_b"),), kinds=("row",))
            for c in cells]
    blk += [FragmentApply(out=c, op="exp", args=(), kinds=()) for c in cells]
    blk.append(FragmentRowReduce(top="rs_t", bot="rs_b", frags=cells, op="add"))
    for h in ("t", "b"):
        blk += [assign(f"ls_{h}", "multiply", f"l_{h}", f"al_{h}"),
                assign(f"l_{h}", "add", f"ls_{h}", f"rs_{h}"),
                assign(f"m_{h}", "copy", f"mn_{h}")]
    blk += [FragmentApply(out=f"fo[{c}]", op="multiply", args=(("al_t", "al_b"),),
                          kinds=("row",)) for c in range(no)]
    blk += [FragmentRepack(frag=f"fp[{i}]", srcs=(f"fs[{2 * i}]", f"fs[{2 * i + 1}]"),
                           ab_dtype=dtype) for i in range(BKV // 16)]
    for c in range(no):
        for i in range(BKV // 16):
            blk += [LdmatrixLoad(frag="fv", src_buffer="_v", src_index=(L(16 * i), L(8 * c)),
                                 role="b", b_trans=True),
                    MmaSyncPtx(c_frag=f"fo[{c}]", a_frag=f"fp[{i}]", b_frag="fv",
                               shape="m16n8k16", ab_dtype=dtype, c_dtype="f32")]
    blk.append(Sync(barrier_id=0, count=None, warp=False))
    body.append(strided("_j", s, L(0), L(BKV), blk))
    body += [FragmentApply(out=f"fo[{c}]", op="divide", args=(("l_t", "l_b"),), kinds=("row",))
             for c in range(no)]
    body += [RegStore(dst_buffer="out", dst_index=(ADD(row0, MUL(V("warp"), L(16))), L(8 * c)),
                      frag="fo", fragment_index=L(c), ldm=d) for c in range(no)]
    tl = tile([ax("bh", bh), ax("qb", s // BQ), ax("t", TH)], body, block_threads=TH)
    return package(entry, "attention", [tl],
                   [("q", (bh, s, d), dtype, 0), ("k", (bh, s, d), dtype, 1),
                    ("v", (bh, s, d), dtype, 2)], [], ("out", (bh, s, d), "f32"),
                   ["q", "k", "v", "out"], (bh * (s // BQ), 1, 1), (TH, 1, 1),
                   rtol=1e-2, atol=1e-3, pid=pid)


def carry_scan(rows: int, cols: int, threads: int = 128, entry="k_carry_scan",
               pid="carry_scan"):
    """One thread per row of x [rows, cols], carried cells st[0], st[1]
    (seed 1) and cnt (seed 0).  Per column: y[r, c] = st[1] as the previous
    step left it; st[0] <- st[1], st[1] <- st[0] * 0.5 + st[1] * x[r, c]
    (both from the previous state); cnt <- cnt + 1 where x[r, c] > 0.  The
    column loop runs twice inside an outer loop (the cells are seeded again
    each time); y[r, cols + 3 + rep] = st[1] after run rep, and after both
    y[r, cols .. cols + 2] = st[0], st[1], cnt."""
    r = V("r")
    zero = L(0)
    inner = [load("xv", "x", (r, V("c"))),
             Pre(name="p0", carrier="st", index=(zero,)),
             Pre(name="p1", carrier="st", index=(L(1),)),
             Pre(name="q", carrier="cnt", index=()),
             assign("a", "multiply", "p0", "half"),
             assign("b", "multiply", "p1", "xv"),
             assign("n1", "add", "a", "b"),
             assign("q1", "add", "q", "one"),
             write("y", (r, V("c")), "p1"),
             Carry(name="st", value="p1", index=(zero,), seed=1.0, dtype=F32),
             Carry(name="st", value="n1", index=(L(1),), seed=1.0, dtype=F32),
             Cond(cond=BinaryExpr(op=">", left=V("xv"), right=Lf(0.0)),
                  body=(Carry(name="cnt", value="q1", index=(), seed=0.0, dtype=F32),),
                  else_body=())]
    outer = [loop("c", cols, inner, seed=False),
             Pre(name="g1", carrier="st", index=(L(1),)),
             write("y", (r, ADD(L(cols + 3), V("rep"))), "g1")]
    body = [Let(name="half", value=Lf(0.5), dtype=F32), Let(name="one", value=Lf(1.0), dtype=F32),
            loop("rep", 2, outer, seed=False),
            Pre(name="f0", carrier="st", index=(zero,)),
            Pre(name="f1", carrier="st", index=(L(1),)),
            Pre(name="fc", carrier="cnt", index=()),
            write("y", (r, L(cols)), "f0"), write("y", (r, L(cols + 1)), "f1"),
            write("y", (r, L(cols + 2)), "fc")]
    tl = tile([ax("r", rows)], body, block_threads=threads)
    return package(entry, "scan", [tl], [("x", (rows, cols), "f32", 0)], [],
                   ("y", (rows, cols + 5), "f32"), ["x", "y"],
                   ((rows + threads - 1) // threads, 1, 1), (threads, 1, 1), rtol=0.0, atol=0.0,
                   pid=pid)


def bench_kernels():
    """IR + meta for every BASELINE configuration, keyed by a short name."""
    return {
        "vector_add": lambda: pointwise(1 << 28, 4, "add", pid="vector_add_2p28"),
        "sum": lambda: reduce_full(1 << 26, pid="sum_2p26"),
        "mean": lambda: reduce_full(1 << 26, mean=True, pid="mean_2p26"),
        "row_sum": lambda: reduce_rows(8192, 8192, pid="row_sum_8192"),
        "rmsnorm": lambda: rmsnorm(65536, 4096, eps=1e-6, pid="rmsnorm_65536x4096"),
        "softmax": lambda: softmax(65536, 4096, pid="softmax_65536x4096"),
        "l2norm": lambda: l2norm(65536, 4096, pid="l2norm_65536x4096"),
        "matmul_square": lambda: matmul(8192, 8192, 8192, pid="matmul_8192"),
        "matmul_rect": lambda: matmul(16384, 4096, 1024, pid="matmul_16384x4096x1024"),
        "matmul_splitk8": lambda: matmul_splitk(16384, 4096, 1024, slice_k=128,
                                                pid="matmul_splitk8"),
        "attention_f32": lambda: attention_bhsd(16, 32, 4096, 128, "f32", pid="attn_f32"),
        "attention_bf16": lambda: attention_bhsd(16, 32, 4096, 128, "bf16", pid="attn_bf16"),
    }


def golden_cases():
    """Small generated kernels the reference interpreter is run on to make
    golden vectors: (name, graph, meta, seed_offset, distribution)."""
    cases = []

    def add(name, gm, off=0, dist="normal"):
        cases.append((name, gm[0], gm[1], off, dist))

    add("gen_add_u4_4096", pointwise(4096, 4, "add", pid="gen_add"), 0, "uniform")
    add("gen_relu_mul_u2_1000", pointwise(1000, 2, "relu_mul", out="mul", entry="k_mul_pointwise",
                                          pid="gen_relu_mul"))
    add("gen_sum_5000", reduce_full(5000, pid="gen_sum"), 0, "uniform01")
    add("gen_mean_8192_t256", reduce_full(8192, threads=256, mean=True, pid="gen_mean"), 0,
        "uniform01")
    add("gen_rowsum_48x300", reduce_rows(48, 300, pid="gen_rowsum"))
    add("gen_rmsnorm_32x640", rmsnorm(32, 640, eps=1e-6, pid="gen_rmsnorm"))
    add("gen_softmax_40x1000", softmax(40, 1000, pid="gen_softmax"))
    add("gen_l2norm_24x256_t64", l2norm(24, 256, threads=64, pid="gen_l2norm"))
    add("gen_matmul_64x128x192", matmul(64, 128, 192, pid="gen_matmul"), 0, "uniform")
    add("gen_splitk_32x64x64_s16", matmul_splitk(32, 64, 64, slice_k=16, pid="gen_splitk"))
    add("gen_attn_64x32", attention(64, 32, pid="gen_attn"))
    add("gen_attn_tiled_96x64", attention_tiled(96, 64, pid="gen_attn_tiled"))
    add("gen_attn_bhsd_2x2x32x32", attention_bhsd(2, 2, 32, 32, pid="gen_attn_bhsd"))
    # f16 and f64 data paths (``ptxgen/model.py:8-31``, ``ptxgen/interp.py:115-141``)
    add("gen_add_f64_u2_1000", pointwise(1000, 2, "add", dtype="f64", pid="gen_add_f64"))
    add("gen_relu_mul_f64_u2_1000", pointwise(1000, 2, "relu_mul", out="mul", dtype="f64",
                                              entry="k_mul_pointwise", pid="gen_relu_mul_f64"))
    add("gen_add_f16_u4_4096", pointwise(4096, 4, "add", dtype="f16", pid="gen_add_f16"), 0,
        "uniform")
    add("gen_relu_mul_f16_u2_1000", pointwise(1000, 2, "relu_mul", out="mul", dtype="f16",
                                              entry="k_mul_pointwise", pid="gen_relu_mul_f16"))
    add("gen_scalar_affine_3000", scalar_affine(3000, 1.75, -0.5, 2222, pid="gen_scalar"))
    add("gen_sum_f16_5000", reduce_full(5000, dtype="f16", pid="gen_sum_f16"), 0, "uniform01")
    add("gen_sum_f16acc_f16_3000", reduce_full(3000, dtype="f16", acc_dtype="f16",
                                               pid="gen_sum_f16acc"))
    add("gen_mean_f16_8192_t256", reduce_full(8192, threads=256, mean=True, dtype="f16",
                                              pid="gen_mean_f16"), 0, "uniform01")
    add("gen_rowsum_f16_48x300", reduce_rows(48, 300, dtype="f16", pid="gen_rowsum_f16"))
    add("gen_colsum_f64_64x300", reduce_cols(64, 300, dtype="f64", pid="gen_colsum_f64"))
    add("gen_colsum_f16_64x300", reduce_cols(64, 300, dtype="f16", pid="gen_colsum_f16"), 0,
        "uniform01")
    return cases


def dumps(obj) -> str:
    return json.dumps(obj, indent=1) + "\n"
