"""Structural analysis of Kernel IR used to pick and specialise templates.

Index expressions are reduced to affine forms ``{var: coeff, 1: const}``
over the Tile/loop axes where possible; the templates only accept loads
and writes whose addresses they can prove (for example "element ``U*g+k`` of a
buffer with exactly the Tile's element count" for pointwise), which is the
B200 analogue of the reference's alignment-divisibility proof
(``ptxgen/emit.py:109-135``, ``ptxgen/emit.py:952-969``).
"""

from __future__ import annotations

from . import ir


class NoMatch(Exception):
    """The IR does not have the structure a template needs."""


def affine(e):
    """Affine form of an integer index expression, or None."""
    if isinstance(e, ir.Var):
        return {e.name: 1}
    if isinstance(e, ir.Literal):
        if not ir.is_int_literal(e):
            return None
        return {1: int(e.value)} if int(e.value) else {}
    if isinstance(e, ir.BinaryExpr):
        a, b = affine(e.left), affine(e.right)
        if a is None or b is None:
            return None
        if e.op in ("+", "-"):
            s = 1 if e.op == "+" else -1
            out = dict(a)
            for k, v in b.items():
                out[k] = out.get(k, 0) + s * v
            return {k: v for k, v in out.items() if v}
        if e.op == "*":
            if set(a) <= {1}:
                c = a.get(1, 0)
                return {k: v * c for k, v in b.items() if v * c}
            if set(b) <= {1}:
                c = b.get(1, 0)
                return {k: v * c for k, v in a.items() if v * c}
        return None
    return None


def flat_affine(index, shape):
    """Affine form of the row-major flat offset of ``index`` into ``shape``
    (a short index addresses the trailing dims, ``interp.py:559-576``)."""
    n = len(index)
    if n == 0:
        return {}
    dims = [1] * max(0, n - len(shape)) + [int(d) for d in shape]
    dims = dims[len(dims) - n:]
    out: dict = {}
    stride = 1
    for idx, d in zip(reversed(index), reversed(dims)):
        a = affine(idx)
        if a is None:
            return None
        for k, v in a.items():
            out[k] = out.get(k, 0) + v * stride
        stride *= d
    return {k: v for k, v in out.items() if v}


def numel(shape) -> int:
    n = 1
    for s in shape:
        n *= int(s)
    return n


def is_var(e, name: str) -> bool:
    return isinstance(e, ir.Var) and e.name == name


def int_literal(e):
    if isinstance(e, ir.Literal) and ir.is_int_literal(e):
        return int(e.value)
    return None


def is_lane0(e) -> bool:
    return (isinstance(e, ir.BinaryExpr) and e.op == "==" and is_var(e.left, "lane")
            and int_literal(e.right) == 0)


def split_block_combine(body, start: int):
    """Recognise ``WarpShuffle, Smem*, Cond(lane==0){smem writes}, Sync,
    TreeHalve`` at ``body[start:]``; return (shuffle, treehalve, next index)."""
    i = start
    if i >= len(body) or not isinstance(body[i], ir.WarpShuffle):
        raise NoMatch("expected WarpShuffle")
    ws = body[i]
    if int(ws.length) != 32:
        raise NoMatch("warp shuffle over a partial warp")
    i += 1
    while i < len(body) and isinstance(body[i], ir.Smem):
        i += 1
    if i < len(body) and isinstance(body[i], ir.Cond) and is_lane0(body[i].cond):
        for st in body[i].body:
            if not isinstance(st, ir.Write):
                raise NoMatch("lane-0 block holds more than smem writes")
        i += 1
    else:
        raise NoMatch("expected lane-0 smem writes")
    if i < len(body) and isinstance(body[i], ir.Sync):
        i += 1
    else:
        raise NoMatch("expected Sync")
    if i >= len(body) or not isinstance(body[i], ir.TreeHalve):
        raise NoMatch("expected TreeHalve")
    th = body[i]
    if tuple(th.state) != tuple(ws.state) or th.inner is not None:
        raise NoMatch("TreeHalve states differ from the shuffle's")
    if th.tid_var != "warp":
        raise NoMatch("TreeHalve over something other than warps")
    return ws, th, i + 1


def scalar_stmt(st) -> bool:
    return isinstance(st, (ir.Assign, ir.Let, ir.Init, ir.Load, ir.Accum))


def loads_in(body):
    return [st for st in ir.walk(body) if isinstance(st, ir.Load)]
