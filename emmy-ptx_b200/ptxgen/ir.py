"""Emmy Kernel IR object model and a safe deserialiser.

The reference loads IR through ``emmy-ml`` (``Graph.from_dict``,
``ptxgen/loader.py:35``).  That package is not available here, so this module
rebuilds the same object model from the JSON on its own:

* ``KernelOp.op_fields.body`` holds one Python-repr string per top-level
  statement, e.g. ``Tile(axes=(Axis(name='a0', extent=Dim(64), ...),), ...)``.
  Each string is parsed with ``ast.parse(mode="eval")`` and rebuilt by walking
  the tree.  Only ``Call``, ``Constant``, ``Tuple``, ``List`` and ``Name``
  nodes are accepted and every constructor must be a known class, so nothing
  in the file is ever executed.
* The classes carry the attribute names the IR vocabulary defines
  (``TASK.md:89-187``) and the small protocol the reference code relies on:
  ``nested()`` for child bodies, ``Dim.as_static()``, ``ElementwiseImpl.name``,
  ``DataType.name``, ``Literal.dtype`` as the strings ``'int'``/``'float'``,
  ``free_vars`` on expressions, and no ``swizzle`` attribute on ``Load``
  (``ptxgen/interp.py:702`` reads it with a ``getattr`` default).

The model is also used to *write* IR (``repr`` of every node reproduces the
constructor syntax the JSON uses), which is how ``ptxgen.irgen`` emits new
kernels at the benchmark shapes.
"""

from __future__ import annotations

import ast
import json
from dataclasses import dataclass, field, fields
from pathlib import Path
from typing import Any

import numpy as np

# ---------------------------------------------------------------------------
# leaf helpers
# ---------------------------------------------------------------------------


class Dim:
    """A static extent; ``Dim(512)`` in the repr grammar."""

    __slots__ = ("value",)

    def __init__(self, value: int):
        self.value = int(value)

    def as_static(self) -> int:
        return self.value

    def __int__(self) -> int:
        return self.value

    def __eq__(self, other) -> bool:
        return isinstance(other, Dim) and other.value == self.value

    def __hash__(self) -> int:
        return hash(("Dim", self.value))

    def __repr__(self) -> str:
        return f"Dim({self.value})"


class ElementwiseImpl:
    """An elementwise op handle; ``ElementwiseImpl('add')``."""

    __slots__ = ("name",)

    def __init__(self, name: str):
        self.name = str(name)

    def __eq__(self, other) -> bool:
        return isinstance(other, ElementwiseImpl) and other.name == self.name

    def __hash__(self) -> int:
        return hash(("EW", self.name))

    def __repr__(self) -> str:
        return f"ElementwiseImpl({self.name!r})"


class DataType:
    """``DataType(name='f32', np=dtype('float32'), nbytes=4)``."""

    __slots__ = ("name", "np", "nbytes")

    def __init__(self, name: str, np=None, nbytes: int | None = None):  # noqa: A002
        self.name = str(name)
        self.np = np
        self.nbytes = nbytes

    def __eq__(self, other) -> bool:
        return isinstance(other, DataType) and other.name == self.name

    def __hash__(self) -> int:
        return hash(("DT", self.name))

    def __str__(self) -> str:
        return self.name

    def __repr__(self) -> str:
        npd = f"dtype({str(self.np)!r})" if self.np is not None else "None"
        return f"DataType(name={self.name!r}, np={npd}, nbytes={self.nbytes!r})"


_NP_NAME = {"f32": "float32", "f64": "float64", "f16": "float16", "bf16": "bfloat16",
            "i32": "int32", "i64": "int64", "u32": "uint32", "u64": "uint64", "bool": "bool"}
_NBYTES = {"f32": 4, "f64": 8, "f16": 2, "bf16": 2, "i32": 4, "i64": 8, "u32": 4, "u64": 8,
           "bool": 1}


def datatype(name: str) -> DataType:
    """Build the DataType the IR writes for an emmy dtype name."""
    npname = _NP_NAME[name]
    try:
        npd = np.dtype(npname)
    except TypeError:  # bfloat16 is not a numpy builtin
        npd = _NpName(npname)
    return DataType(name=name, np=npd, nbytes=_NBYTES[name])


class _NpName:
    """Stand-in for a numpy dtype numpy itself does not know (bfloat16)."""

    def __init__(self, name: str):
        self.name = name

    def __str__(self) -> str:
        return self.name


def _np_dtype_ctor(name: str):
    try:
        return np.dtype(name)
    except TypeError:
        return _NpName(name)


# ---------------------------------------------------------------------------
# node base
# ---------------------------------------------------------------------------


def _fmt(v: Any) -> str:
    if isinstance(v, tuple):
        if len(v) == 1:
            return f"({_fmt(v[0])},)"
        return "(" + ", ".join(_fmt(x) for x in v) + ")"
    if isinstance(v, list):
        return "[" + ", ".join(_fmt(x) for x in v) + "]"
    if isinstance(v, float):
        return repr(v)
    return repr(v)


class Node:
    """Base class: dataclass fields are the IR keyword arguments, in order."""

    def nested(self) -> list:
        return []

    def __repr__(self) -> str:
        parts = [f"{f.name}={_fmt(getattr(self, f.name))}" for f in fields(self)]
        return f"{type(self).__name__}({', '.join(parts)})"


# ---------------------------------------------------------------------------
# expressions
# ---------------------------------------------------------------------------


class Expr(Node):
    @property
    def free_vars(self) -> frozenset:
        out: set[str] = set()
        _collect_vars(self, out)
        return frozenset(out)


def _collect_vars(e, out: set) -> None:
    if isinstance(e, Var):
        out.add(e.name)
    elif isinstance(e, BinaryExpr):
        _collect_vars(e.left, out)
        _collect_vars(e.right, out)
    elif isinstance(e, TernaryExpr):
        _collect_vars(e.cond, out)
        _collect_vars(e.if_true, out)
        _collect_vars(e.if_false, out)
    elif isinstance(e, FuncCallExpr):
        for a in e.args:
            _collect_vars(a, out)
    elif isinstance(e, CastExpr):
        _collect_vars(e.expr, out)
    elif isinstance(e, FlatIndex):
        for a in e.index:
            _collect_vars(a, out)


@dataclass(repr=False, eq=True, frozen=True)
class Var(Expr):
    name: str


@dataclass(repr=False, eq=True, frozen=True)
class Literal(Expr):
    value: Any
    dtype: Any = None


@dataclass(repr=False, eq=True, frozen=True)
class BinaryExpr(Expr):
    op: str
    left: Any
    right: Any


@dataclass(repr=False, eq=True, frozen=True)
class TernaryExpr(Expr):
    cond: Any
    if_true: Any
    if_false: Any


@dataclass(repr=False, eq=True, frozen=True)
class Builtin(Expr):
    name: str


@dataclass(repr=False, eq=True, frozen=True)
class FuncCallExpr(Expr):
    name: str
    args: tuple = ()


@dataclass(repr=False, eq=True, frozen=True)
class CastExpr(Expr):
    dtype: Any
    expr: Any


@dataclass(repr=False, eq=True, frozen=True)
class FlatIndex(Expr):
    buffer: str
    index: tuple = ()


# ---------------------------------------------------------------------------
# axes
# ---------------------------------------------------------------------------


@dataclass(repr=False, eq=True, frozen=True)
class Window(Node):
    parent: Any = None
    base: Any = None
    bound: Any = None
    partition: bool = False


@dataclass(repr=False, eq=True, frozen=True)
class Axis(Node):
    name: str
    extent: Any
    window: Any = None


# ---------------------------------------------------------------------------
# statements
# ---------------------------------------------------------------------------


@dataclass(repr=False, eq=True)
class Tile(Node):
    axes: tuple
    body: tuple
    block_threads: Any = None
    aux_threads: int = 0
    raster_axes: Any = None
    raster_group: Any = None
    raster_orient: str = "m"

    def nested(self) -> list:
        return [self.body]


@dataclass(repr=False, eq=True)
class Load(Node):
    names: tuple
    input: str
    index: tuple
    dtype: Any = None


@dataclass(repr=False, eq=True)
class Assign(Node):
    name: str
    op: Any
    args: tuple
    dtype: Any = None


@dataclass(repr=False, eq=True)
class Accum(Node):
    name: str
    value: str
    op: Any
    dtype: Any = None
    axes: Any = ()
    base: Any = None


@dataclass(repr=False, eq=True)
class Let(Node):
    name: str
    value: Any
    dtype: Any = None


@dataclass(repr=False, eq=True)
class Pre(Node):
    name: str
    carrier: str
    index: Any = ()


@dataclass(repr=False, eq=True)
class Carry(Node):
    name: str
    value: str
    index: Any = ()
    seed: Any = 0.0
    dtype: Any = None


@dataclass(repr=False, eq=True)
class Init(Node):
    name: str
    identity: Any
    dtype: Any = None


@dataclass(repr=False, eq=True)
class Write(Node):
    output: str
    index: tuple
    values: tuple
    value_dtype: Any = None
    atomic: bool = False
    swizzle: str = "NONE"


@dataclass(repr=False, eq=True)
class Loop(Node):
    axis: Any
    body: tuple
    unroll: bool = False
    seed: bool = True

    def nested(self) -> list:
        return [self.body]


@dataclass(repr=False, eq=True)
class StridedLoop(Node):
    axis: Any
    start: Any
    step: Any
    body: tuple
    unroll: bool = False
    end: Any = None
    seed: bool = True

    def nested(self) -> list:
        return [self.body]


@dataclass(repr=False, eq=True)
class Cond(Node):
    cond: Any
    body: tuple
    else_body: tuple = ()

    def nested(self) -> list:
        return [self.body, self.else_body or ()]


@dataclass(repr=False, eq=True)
class Smem(Node):
    name: str
    extents: tuple
    dtype: Any = "float"
    align: int = 0


@dataclass(repr=False, eq=True)
class Sync(Node):
    barrier_id: Any = None
    count: Any = None
    warp: bool = False


@dataclass(repr=False, eq=True)
class WarpShuffle(Node):
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int = 32
    dtype: Any = None


@dataclass(repr=False, eq=True)
class TreeHalve(Node):
    bufs: tuple
    state: tuple
    state_b: tuple
    combine_states: tuple
    length: int
    tid_var: str = "warp"
    dtype: Any = None
    barrier_id: Any = 0
    barrier_count: Any = None
    inner: Any = None


@dataclass(repr=False, eq=True)
class CpAsyncCopy(Node):
    smem: str
    smem_index: tuple
    src: str
    src_index: tuple
    nbytes: int = 16
    swizzle: str = "NONE"
    lane_index: Any = None
    lane_rows: Any = None


@dataclass(repr=False, eq=True)
class CpAsyncCommit(Node):
    pass


@dataclass(repr=False, eq=True)
class CpAsyncWait(Node):
    group: int = 0


@dataclass(repr=False, eq=True)
class SelectBranch(Node):
    value: str
    select: Any = None


@dataclass(repr=False, eq=True)
class Select(Node):
    name: str
    branches: tuple


@dataclass(repr=False, eq=True)
class ZeroPrologue(Node):
    dst: str
    words: int


# -- bulk-async transport and mbarriers (starred in the reference's IR table,
#    ``TASK.md:121-127``; neither its interpreter nor its emitter has them, so
#    their meaning here is this repository's, stated in ``oracle/interp.py``)


@dataclass(repr=False, eq=True)
class TmaDescriptor(Node):
    name: str
    src_buf: str
    src_shape: tuple
    box_extents: tuple
    swizzle: str = "NONE"
    dtype: Any = None


@dataclass(repr=False, eq=True)
class TmaLoad(Node):
    smem: str
    smem_index: Any
    desc: str
    coords: tuple
    mbar: str
    mbar_slot: Any = None


@dataclass(repr=False, eq=True)
class MbarrierInit(Node):
    mbar: str
    count: Any = 1
    slot: Any = None


@dataclass(repr=False, eq=True)
class MbarrierArriveExpectTx(Node):
    mbar: str
    bytes_: Any = 0
    slot: Any = None


@dataclass(repr=False, eq=True)
class MbarrierArrive(Node):
    mbar: str
    slot: Any = None


@dataclass(repr=False, eq=True)
class MbarrierWait(Node):
    mbar: str
    phase: Any = 0
    slot: Any = None


@dataclass(repr=False, eq=True)
class SetMaxNReg(Node):
    count: int = 0
    direction: str = "inc"


# -- warp-level tensor-core fragments (``mma.sync``), starred in the same
#    table (``TASK.md:146-158``)


@dataclass(repr=False, eq=True)
class RegFragment(Node):
    name: str
    role: str = "c"
    shape: Any = "m16n8k16"
    dtype: Any = "bf16"
    count: int = 1
    nregs: Any = None


@dataclass(repr=False, eq=True)
class LdmatrixLoad(Node):
    frag: str
    src_buffer: str
    src_index: tuple
    role: str = "a"
    ldm: Any = None
    swizzle: str = "NONE"
    staged: Any = None
    gmem_guard: Any = None
    k_zero: Any = None
    b_trans: bool = False
    pair_frag: Any = None
    byte_slab: Any = None
    scale_buffer: Any = None
    scale_index: Any = None
    scale_ldm: Any = None
    fragment_layout: Any = None
    fragment_index: Any = None


@dataclass(repr=False, eq=True)
class MmaSyncPtx(Node):
    c_frag: str
    a_frag: str
    b_frag: str
    shape: Any = "m16n8k16"
    ab_dtype: Any = "bf16"
    c_dtype: Any = "f32"
    b_row_major: bool = False
    sfa_frag: Any = None
    sfb_frag: Any = None


@dataclass(repr=False, eq=True)
class RegStore(Node):
    dst_buffer: str
    dst_index: tuple
    frag: str
    shape: Any = "m16n8k16"
    ldm: Any = None
    epilogue: Any = None
    extra_frags: Any = None
    m_guard: Any = None
    n_guard: Any = None
    atomic: bool = False
    fragment_layout: Any = None
    volta_interleaved: Any = None
    fragment_index: Any = None
    swizzle: str = "NONE"
    row_dim: Any = None
    col_dim: Any = None


@dataclass(repr=False, eq=True)
class FragmentPromote(Node):
    dst: str
    src: str


@dataclass(repr=False, eq=True)
class FragmentApply(Node):
    out: str
    op: Any
    args: tuple = ()
    kinds: tuple = ()
    in_place: bool = True
    layout: Any = None
    post: Any = None
    row_base: Any = None
    col_base: Any = None


@dataclass(repr=False, eq=True)
class FragmentRowReduce(Node):
    top: str
    bot: str
    frags: Any = ()
    op: Any = "add"
    layout: Any = None
    dtype: Any = "f32"


@dataclass(repr=False, eq=True)
class FragmentRepack(Node):
    frag: str
    srcs: tuple = ()
    ab_dtype: Any = "bf16"
    fragment_layout: Any = None
    part: Any = None


# -- warpgroup tensor-core products (``wgmma``), starred in the same table
#    (``TASK.md:162-172``)


@dataclass(repr=False, eq=True)
class WgmmaDescriptor(Node):
    name: str
    smem: str
    smem_index: Any = None
    swizzle: str = "B128"
    lbo_bytes: Any = 16
    sbo_bytes: Any = 1024


@dataclass(repr=False, eq=True)
class WgmmaMma(Node):
    c_frags: str
    b_desc: str
    shape: Any = "m64n64k16"
    ab_dtype: Any = "bf16"
    a_desc: Any = None
    a_frag: Any = None
    scale_d: Any = 1
    trans_a: Any = 0
    trans_b: Any = 0


@dataclass(repr=False, eq=True)
class WgmmaFence(Node):
    pass


@dataclass(repr=False, eq=True)
class WgmmaCommit(Node):
    pass


@dataclass(repr=False, eq=True)
class WgmmaWait(Node):
    group: int = 0


# ---------------------------------------------------------------------------
# graph level
# ---------------------------------------------------------------------------


@dataclass
class Tensor:
    name: str
    shape: tuple
    dtype: DataType


@dataclass
class KernelOp:
    name: str
    body: tuple
    zero_delegated: tuple = ()
    serial: tuple = ()
    inputs: tuple = ()
    outputs: tuple = ()


@dataclass
class InputOp:
    pass


@dataclass
class ConstantOp:
    name: str = ""
    value: Any = None


@dataclass
class OtherOp:
    kind: str
    fields: dict = field(default_factory=dict)


@dataclass
class GraphNode:
    name: str
    op: Any
    inputs: tuple
    outputs: tuple  # of Tensor


@dataclass
class Graph:
    inputs: tuple
    outputs: tuple
    nodes: dict

    @classmethod
    def from_dict(cls, data: dict) -> "Graph":
        nodes: dict[str, GraphNode] = {}
        for name, nd in data.get("nodes", {}).items():
            outs = tuple(
                Tensor(name=o["name"], shape=tuple(Dim(int(x)) for x in o.get("shape", ())),
                       dtype=datatype(o.get("dtype", "f32")))
                for o in nd.get("outputs", ())
            )
            kind = nd.get("op")
            f = nd.get("op_fields", {}) or {}
            if kind == "KernelOp":
                body = tuple(parse_stmt(s) for s in f.get("body", ()))
                op = KernelOp(name=f.get("name") or "", body=body,
                              zero_delegated=tuple(f.get("zero_delegated") or ()),
                              serial=tuple(f.get("serial") or ()),
                              inputs=tuple(nd.get("inputs", ())),
                              outputs=tuple(t.name for t in outs))
            elif kind == "InputOp":
                op = InputOp()
            elif kind == "ConstantOp":
                op = ConstantOp(name=f.get("name", name), value=f.get("value"))
            else:
                op = OtherOp(kind=str(kind), fields=dict(f))
            nodes[name] = GraphNode(name=name, op=op, inputs=tuple(nd.get("inputs", ())),
                                    outputs=outs)
        return cls(inputs=tuple(data.get("inputs", ())), outputs=tuple(data.get("outputs", ())),
                   nodes=nodes)


# ---------------------------------------------------------------------------
# repr-grammar parser
# ---------------------------------------------------------------------------

_CTORS: dict[str, Any] = {
    c.__name__: c
    for c in (
        Dim, ElementwiseImpl, DataType, Var, Literal, BinaryExpr, TernaryExpr, Builtin,
        FuncCallExpr, CastExpr, FlatIndex, Window, Axis, Tile, Load, Assign, Accum, Let, Init,
        Write, Loop, StridedLoop, Cond, Smem, Sync, WarpShuffle, TreeHalve, CpAsyncCopy,
        CpAsyncCommit, CpAsyncWait, Select, SelectBranch, ZeroPrologue, TmaDescriptor,
        TmaLoad, MbarrierInit, MbarrierArriveExpectTx, MbarrierArrive, MbarrierWait, SetMaxNReg,
        RegFragment, LdmatrixLoad, MmaSyncPtx, RegStore, WgmmaDescriptor, WgmmaMma, WgmmaFence,
        WgmmaCommit, WgmmaWait, FragmentApply, FragmentRowReduce, FragmentRepack, Pre, Carry,
        FragmentPromote,
    )
}
_CTORS["dtype"] = _np_dtype_ctor
_CONSTS = {"None": None, "True": True, "False": False}


class IRParseError(ValueError):
    pass


def _build(node: ast.AST):
    if isinstance(node, ast.Constant):
        return node.value
    if isinstance(node, ast.Tuple):
        return tuple(_build(e) for e in node.elts)
    if isinstance(node, ast.List):
        return [_build(e) for e in node.elts]
    if isinstance(node, ast.Name):
        if node.id in _CONSTS:
            return _CONSTS[node.id]
        raise IRParseError(f"bare name {node.id!r} in IR body")
    if isinstance(node, ast.UnaryOp) and isinstance(node.op, ast.USub):
        v = _build(node.operand)
        if isinstance(v, (int, float)):
            return -v
    if isinstance(node, ast.Call):
        if not isinstance(node.func, ast.Name):
            raise IRParseError("constructor must be a plain name")
        name = node.func.id
        ctor = _CTORS.get(name)
        if ctor is None:
            raise IRParseError(f"unknown IR constructor {name!r}")
        args = [_build(a) for a in node.args]
        kwargs = {k.arg: _build(k.value) for k in node.keywords}
        try:
            return ctor(*args, **kwargs)
        except TypeError as exc:
            raise IRParseError(f"bad arguments for {name}: {exc}") from exc
    raise IRParseError(f"unsupported syntax {type(node).__name__} in IR body")


def parse_stmt(text: str):
    """Parse one repr-grammar statement string into IR objects."""
    try:
        tree = ast.parse(text, mode="eval")
    except SyntaxError as exc:
        raise IRParseError(f"IR body is not valid repr grammar: {exc}") from exc
    return _build(tree.body)


def load_graph(path: str | Path) -> Graph:
    return Graph.from_dict(json.loads(Path(path).read_text()))


# ---------------------------------------------------------------------------
# walking helpers
# ---------------------------------------------------------------------------


def walk(body):
    """Yield every statement in ``body`` depth-first, in program order."""
    for st in body:
        yield st
        for child in st.nested():
            yield from walk(child)


def is_int_literal(e: Literal) -> bool:
    """Integer-ness of a literal: its dtype decides, the value is the fallback."""
    name = getattr(e.dtype, "name", e.dtype)
    if name in ("int", "i32", "u32", "i64", "u64"):
        return True
    if name in ("float", "f32", "f64", "f16", "bf16"):
        return False
    return isinstance(e.value, int) and not isinstance(e.value, bool)
