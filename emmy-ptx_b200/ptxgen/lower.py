"""Lowering of IR values, expressions and scalar statements to PTX.

Every kernel template drives the per-element arithmetic of the IR through
this module, so the arithmetic of a compiled kernel is the IR's own, op by
op.  The semantics follow the reference golden model (``ptxgen/interp.py``):

* kinds ``s32``, ``s64``, ``f32``, ``f64``, ``pred``; f16/bf16 values live in
  f32 registers already rounded to their storage precision;
* binary promotion: f64 > f32 > s32 (``interp.py:107-112``);
* coercions are PTX ``cvt`` (``interp.py:115-141``): float->int truncates,
  pred->number is 0/1;
* f32 add/sub/mul/div use the ``.rn`` forms, so ptxas never contracts a
  multiply-add into an FMA and every op rounds once, bit for bit like numpy
  (``interp.py:180-217``); max/min return the non-NaN operand;
* sqrt and reciprocal are IEEE (``sqrt.rn``, ``rcp.rn``); the f64-evaluated
  reference value rounded to f32 is the same number;
* exp is ``2^(x*log2 e)`` with the rounding error of the product carried as
  a first-order correction (a Cody-Waite style split of log2 e), about 2 ulp
  -- the reference rounds an f64 exp (``interp.py:256-257``), so exp-based
  ops are checked with a tolerance;
* every IR name owns one register per kind, so accumulators and loop-carried
  values are updated in place across PTX loop back-edges.
"""

from __future__ import annotations

import math

from . import ir, ops
from .model import dtype_info
from .ptx import Kernel, Reg, f32_hex, f64_hex

LOG2E = 1.4426950408889634
LN2 = 0.6931471805599453
# log2(e) split into an f32 head and the f32 tail of the remainder
L2E_HI = float(__import__("numpy").float32(LOG2E))
L2E_LO = float(__import__("numpy").float32(LOG2E - L2E_HI))


def _round_storage(v: float, store: str | None) -> float:
    """``v`` rounded to f32, then to ``store`` when that is f16 or bf16
    (round to nearest even; bf16 keeps the top 16 bits of the f32)."""
    import numpy as np
    f = np.float32(v)
    if store == "f16":
        return float(np.float16(f))
    if store == "bf16" and np.isfinite(f):
        b = int(f.view(np.uint32))
        b = (b + 0x7FFF + ((b >> 16) & 1)) & 0xFFFF0000
        return float(np.uint32(b).view(np.float32))
    return float(f)


class LowerError(NotImplementedError):
    """The IR uses something this lowering does not handle."""


class Val:
    __slots__ = ("reg", "kind")

    def __init__(self, reg: str, kind: str):
        self.reg = reg
        self.kind = kind

    def __repr__(self) -> str:
        return f"Val({self.reg}:{self.kind})"


def value_kind(dtype) -> str:
    k = dtype_info(dtype)[0]
    return "f32" if k in ("bf16", "f16") else k


def storage_kind(dtype) -> str:
    return dtype_info(dtype)[0]


def _promote(a: str, b: str) -> str:
    if "f64" in (a, b):
        return "f64"
    if a in ("f32", "f16") or b in ("f32", "f16"):
        return "f32"
    return "s32"


class Lowerer:
    """Per-kernel lowering state: the kernel builder and the name->register map."""

    def __init__(self, k: Kernel):
        self.k = k
        self.env: dict[str, Val] = {}
        self.home: dict[tuple[str, str], Reg] = {}
        # hooks a template installs
        self.load_hook = None     # (stmt) -> None, binds names
        self.write_hook = None    # (stmt) -> None
        self.extra = {}           # stmt type -> handler
        self.mask = None          # predicate register: lanes whose register writes land

    # -- registers ---------------------------------------------------------

    def home_reg(self, name: str, kind: str) -> Reg:
        key = (name, kind)
        r = self.home.get(key)
        if r is None:
            r = self.k.reg(kind)
            self.home[key] = r
        return r

    def bind(self, name: str, v: Val) -> Val:
        """Write ``v`` into ``name``'s register (one register per name+kind).
        Under a mask only the active lanes take the value; a name first
        bound under a mask starts at 0 in the other lanes (interp.py:458-468)."""
        fresh = (name, v.kind) not in self.home
        r = self.home_reg(name, v.kind)
        if fresh and self.mask is not None and v.kind != "pred":
            zero = {"f32": "0f00000000", "f64": "0d0000000000000000"}.get(v.kind, "0")
            self.k(f"mov.{self._mov_t(v.kind)} {r}, {zero}")
        if r != v.reg:
            guard = f"@{self.mask} " if self.mask is not None else ""
            self.k(f"{guard}mov.{self._mov_t(v.kind)} {r}, {v.reg}")
        out = Val(r, v.kind)
        self.env[name] = out
        return out

    @staticmethod
    def _mov_t(kind: str) -> str:
        return {"f32": "f32", "f64": "f64", "s32": "b32", "s64": "b64", "pred": "pred",
                "u32": "b32", "u64": "b64"}[kind]

    def const(self, value, kind: str) -> Val:
        k = self.k
        r = k.reg(kind)
        if kind == "f32":
            k(f"mov.f32 {r}, {f32_hex(value)}")
        elif kind == "f64":
            k(f"mov.f64 {r}, {f64_hex(value)}")
        elif kind == "s32":
            k(f"mov.b32 {r}, {int(value) & 0xFFFFFFFF}")
        elif kind == "s64":
            k(f"mov.b64 {r}, {int(value) & 0xFFFFFFFFFFFFFFFF}")
        elif kind == "pred":
            k(f"setp.ne.s32 {r}, {1 if value else 0}, 0")
        else:
            raise LowerError(f"constant of kind {kind}")
        return Val(r, kind)

    # -- coercion ----------------------------------------------------------

    def coerce(self, v: Val, kind: str) -> Val:
        if v.kind == kind:
            return v
        k = self.k
        if kind in ("f16", "bf16"):
            f = self.coerce(v, "f32")
            h = k.reg("b16")
            r = k.reg("f32")
            t = "f16" if kind == "f16" else "bf16"
            k(f"cvt.rn.{t}.f32 {h}, {f.reg}")
            k(f"cvt.f32.{t} {r}, {h}")
            return Val(r, "f32")
        r = k.reg(kind)
        if v.kind == "pred":
            one = {"s32": "1", "s64": "1", "f32": "0f3F800000", "f64": "0d3FF0000000000000"}[kind]
            zero = {"s32": "0", "s64": "0", "f32": "0f00000000", "f64": "0d0000000000000000"}[kind]
            t = {"s32": "s32", "s64": "s64", "f32": "f32", "f64": "f64"}[kind]
            k(f"selp.{t} {r}, {one}, {zero}, {v.reg}")
            return Val(r, kind)
        if kind == "pred":
            return self.truthy(v)
        pair = (v.kind, kind)
        table = {
            ("f32", "f64"): "cvt.f64.f32", ("f64", "f32"): "cvt.rn.f32.f64",
            ("s32", "f32"): "cvt.rn.f32.s32", ("s32", "f64"): "cvt.rn.f64.s32",
            ("s64", "f32"): "cvt.rn.f32.s64", ("s64", "f64"): "cvt.rn.f64.s64",
            ("f32", "s32"): "cvt.rzi.s32.f32", ("f64", "s32"): "cvt.rzi.s32.f64",
            ("f32", "s64"): "cvt.rzi.s64.f32", ("f64", "s64"): "cvt.rzi.s64.f64",
            ("s32", "s64"): "cvt.s64.s32", ("s64", "s32"): "cvt.u32.u64",
        }
        if pair not in table:
            raise LowerError(f"coerce {v.kind} -> {kind}")
        k(f"{table[pair]} {r}, {v.reg}")
        return Val(r, kind)

    def truthy(self, v: Val) -> Val:
        if v.kind == "pred":
            return v
        r = self.k.reg("pred")
        t = {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64"}[v.kind]
        zero = {"f32": "0f00000000", "f64": "0d0000000000000000"}.get(v.kind, "0")
        self.k(f"setp.ne.{t} {r}, {v.reg}, {zero}")
        return Val(r, "pred")

    # -- expressions -------------------------------------------------------

    def ev(self, e) -> Val:
        if isinstance(e, ir.Var):
            if e.name not in self.env:
                raise LowerError(f"undefined name {e.name!r}")
            return self.env[e.name]
        if isinstance(e, ir.Literal):
            if ir.is_int_literal(e):
                return self.const(int(e.value), "s32")
            return self.const(float(e.value), "f32")
        if isinstance(e, ir.BinaryExpr):
            if e.op in ops.COMPARE:
                return self.compare(e.op, self.ev(e.left), self.ev(e.right))
            if e.op in ops.LOGICAL:
                a, b = self.truthy(self.ev(e.left)), self.truthy(self.ev(e.right))
                r = self.k.reg("pred")
                self.k(f"{'and' if e.op == '&&' else 'or'}.pred {r}, {a.reg}, {b.reg}")
                return Val(r, "pred")
            return self.apply(e.op, [self.ev(e.left), self.ev(e.right)])
        if isinstance(e, ir.TernaryExpr):
            c = self.truthy(self.ev(e.cond))
            a, b = self.ev(e.if_true), self.ev(e.if_false)
            kind = _promote(a.kind, b.kind)
            return self.select(c, self.coerce(a, kind), self.coerce(b, kind))
        if isinstance(e, ir.FuncCallExpr):
            return self.apply(e.name, [self.ev(a) for a in e.args])
        if isinstance(e, ir.CastExpr):
            return self.coerce(self.ev(e.expr), value_kind(e.dtype))
        if isinstance(e, ir.Builtin):
            return self.builtin(e.name)
        raise LowerError(f"expression {type(e).__name__}")

    def builtin(self, name: str) -> Val:
        key = (name.replace("threadIdx", "thread_idx").replace("blockIdx", "block_idx")
               .replace("blockDim", "block_dim").replace("gridDim", "grid_dim"))
        sreg = {"thread_idx.x": "%tid.x", "tid": "%tid.x", "block_idx.x": "%ctaid.x",
                "block_idx": "%ctaid.x", "cta": "%ctaid.x", "block_dim.x": "%ntid.x",
                "ntid": "%ntid.x", "lane": "%laneid", "lane_id": "%laneid",
                "grid_dim.x": "%nctaid.x", "thread_idx.y": "%tid.y", "thread_idx.z": "%tid.z",
                "block_dim.y": "%ntid.y", "block_dim.z": "%ntid.z", "grid_dim.y": "%nctaid.y",
                "grid_dim.z": "%nctaid.z", "block_idx.y": "%ctaid.y",
                "block_idx.z": "%ctaid.z"}.get(key)
        if key in ("warp", "warp_id"):
            t = self.k.sreg("%tid.x")
            r = self.k.reg("s32")
            self.k(f"shr.u32 {r}, {t}, 5")
            return Val(r, "s32")
        if key in ("warp_size", "warpSize"):
            return self.const(32, "s32")
        if sreg is None:
            raise LowerError(f"builtin {name!r}")
        r = self.k.reg("s32")
        self.k(f"mov.u32 {r}, {sreg}")
        return Val(r, "s32")

    def compare(self, op: str, a: Val, b: Val) -> Val:
        kind = _promote(a.kind, b.kind) if "pred" not in (a.kind, b.kind) else "s32"
        a, b = self.coerce(a, kind), self.coerce(b, kind)
        cmp = {"==": "eq", "!=": "ne", "<": "lt", "<=": "le", ">": "gt", ">=": "ge"}[op]
        if kind in ("f32", "f64") and op == "!=":
            cmp = "neu"  # NaN != x is true, as numpy says
        t = {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64"}[kind]
        r = self.k.reg("pred")
        self.k(f"setp.{cmp}.{t} {r}, {a.reg}, {b.reg}")
        return Val(r, "pred")

    def select(self, c: Val, a: Val, b: Val) -> Val:
        t = {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64"}.get(a.kind)
        r = self.k.reg(a.kind)
        if a.kind == "pred":
            k = self.k
            t1, t2 = k.reg("pred"), k.reg("pred")
            k(f"and.pred {t1}, {c.reg}, {a.reg}")
            k(f"not.pred {t2}, {c.reg}")
            k(f"and.pred {t2}, {t2}, {b.reg}")
            k(f"or.pred {r}, {t1}, {t2}")
            return Val(r, "pred")
        self.k(f"selp.{t} {r}, {a.reg}, {b.reg}, {c.reg}")
        return Val(r, a.kind)

    # -- elementwise ops -----------------------------------------------------

    def apply(self, name: str, args: list[Val]) -> Val:
        name = ops.canon(name)
        if name in ("add", "subtract", "multiply", "divide", "maximum", "minimum"):
            return self.arith(name, args[0], args[1])
        if name == "fma":
            a, b, c = args
            kind = "f64" if "f64" in (a.kind, b.kind, c.kind) else "f32"
            return self.arith("add", self.arith("multiply", self.coerce(a, kind),
                                                self.coerce(b, kind)), self.coerce(c, kind))
        if name == "where":
            c, a, b = args
            kind = _promote(a.kind, b.kind)
            return self.select(self.truthy(c), self.coerce(a, kind), self.coerce(b, kind))
        if name == "clip":
            a, lo, hi = args
            return self.arith("minimum", self.arith("maximum", a, lo), hi)
        if name == "floor_divide":
            a, b = args
            if a.kind in ("f32", "f64") or b.kind in ("f32", "f64"):
                return self.unary("floor", self.arith("divide", a, b))
            return self.arith("divide", a, b)
        if name in ("logical_and", "logical_or"):
            p, q = self.truthy(args[0]), self.truthy(args[1])
            r = self.k.reg("pred")
            self.k(f"{'and' if name == 'logical_and' else 'or'}.pred {r}, {p.reg}, {q.reg}")
            return Val(r, "pred")
        if name in ("remainder", "bitand", "bitor", "bitxor", "shl", "shr"):
            a, b = self.coerce(args[0], "s32"), self.coerce(args[1], "s32")
            r = self.k.reg("s32")
            k = self.k
            if name == "remainder":
                z = k.reg("pred")
                t = k.reg("s32")
                k(f"setp.eq.s32 {z}, {b.reg}, 0")
                k(f"selp.s32 {t}, 1, {b.reg}, {z}")
                k(f"rem.s32 {r}, {a.reg}, {t}")
                k(f"selp.s32 {r}, 0, {r}, {z}")
            elif name in ("bitand", "bitor", "bitxor"):
                k(f"{ {'bitand': 'and', 'bitor': 'or', 'bitxor': 'xor'}[name]}.b32 {r}, {a.reg}, {b.reg}")
            else:
                sh = k.reg("s32")
                k(f"and.b32 {sh}, {b.reg}, 31")
                k(f"{'shl.b32' if name == 'shl' else 'shr.s32'} {r}, {a.reg}, {sh}")
            return Val(r, "s32")
        if name == "power":
            a, b = self.coerce(args[0], "f32"), self.coerce(args[1], "f32")
            lg = self.k.reg("f32")
            self.k(f"lg2.approx.f32 {lg}, {a.reg}")
            t = self.k.reg("f32")
            self.k(f"mul.rn.f32 {t}, {b.reg}, {lg}")
            r = self.k.reg("f32")
            self.k(f"ex2.approx.f32 {r}, {t}")
            return Val(r, "f32")
        if name == "fmod":
            raise LowerError("fmod")
        if len(args) != 1:
            raise LowerError(f"op {name!r} with {len(args)} args")
        return self.unary(name, args[0])

    def arith(self, name: str, a: Val, b: Val) -> Val:
        kind = _promote(a.kind, b.kind)
        a, b = self.coerce(a, kind), self.coerce(b, kind)
        k = self.k
        r = k.reg(kind)
        if kind == "s32":
            if name == "divide":
                z = k.reg("pred")
                t = k.reg("s32")
                k(f"setp.eq.s32 {z}, {b.reg}, 0")
                k(f"selp.s32 {t}, 1, {b.reg}, {z}")
                k(f"div.s32 {r}, {a.reg}, {t}")
                k(f"selp.s32 {r}, 0, {r}, {z}")
            else:
                opc = {"add": "add.s32", "subtract": "sub.s32", "multiply": "mul.lo.s32",
                       "maximum": "max.s32", "minimum": "min.s32"}[name]
                k(f"{opc} {r}, {a.reg}, {b.reg}")
            return Val(r, kind)
        t = kind
        opc = {"add": f"add.rn.{t}", "subtract": f"sub.rn.{t}", "multiply": f"mul.rn.{t}",
               "divide": f"div.rn.{t}", "maximum": f"max.{t}", "minimum": f"min.{t}"}[name]
        k(f"{opc} {r}, {a.reg}, {b.reg}")
        return Val(r, kind)

    exp_mode = "fast"

    def exp_f32(self, x: str) -> str:
        """exp(x) for an f32 register; returns the result register.

        ``fast``: ex2.approx(x * log2 e): relative error about 2^-22 from
        ex2 plus |x| * 2^-24 * ln 2 from rounding the product (6e-7 at
        |x| = 10).  ``accurate``: the product's rounding error, and the tail
        of log2 e, are carried as a first-order correction (about 2 ulp)."""
        k = self.k
        if self.exp_mode == "fast":
            t, y = k.reg("f32"), k.reg("f32")
            k(f"mul.rn.f32 {t}, {x}, {f32_hex(L2E_HI)}")
            k(f"ex2.approx.ftz.f32 {y}, {t}")
            return y
        t, e, p, q, y = (k.reg("f32") for _ in range(5))
        k(f"mul.rn.f32 {t}, {x}, {f32_hex(L2E_HI)}")
        k(f"neg.f32 {e}, {t}")
        k(f"fma.rn.f32 {e}, {x}, {f32_hex(L2E_HI)}, {e}")
        k(f"fma.rn.f32 {e}, {x}, {f32_hex(L2E_LO)}, {e}")
        k(f"ex2.approx.ftz.f32 {p}, {t}")
        k(f"mul.rn.f32 {q}, {e}, {f32_hex(LN2)}")
        k(f"fma.rn.f32 {y}, {p}, {q}, {p}")
        return y

    def unary(self, name: str, v: Val) -> Val:
        k = self.k
        if name == "copy":
            return v
        if name == "logical_not":
            p = self.truthy(v)
            r = k.reg("pred")
            k(f"not.pred {r}, {p.reg}")
            return Val(r, "pred")
        if v.kind == "s32" and name in ("negative", "absolute"):
            r = k.reg("s32")
            k(f"{'neg' if name == 'negative' else 'abs'}.s32 {r}, {v.reg}")
            return Val(r, "s32")
        if name == "bitcast":
            swap = {"f32": "s32", "s32": "f32", "f64": "s64", "s64": "f64"}
            if v.kind not in swap:
                return v
            r = k.reg(swap[v.kind])
            k(f"mov.b{64 if v.kind in ('f64', 's64') else 32} {r}, {v.reg}")
            return Val(r, swap[v.kind])
        x = self.coerce(v, "f32").reg
        r = k.reg("f32")
        one = "0f3F800000"
        if name == "negative":
            k(f"neg.f32 {r}, {x}")
        elif name == "absolute":
            k(f"abs.f32 {r}, {x}")
        elif name == "square":
            k(f"mul.rn.f32 {r}, {x}, {x}")
        elif name in ("exp", "exp_fast"):
            return Val(self.exp_f32(x), "f32")
        elif name == "sqrt":
            k(f"sqrt.rn.f32 {r}, {x}")
        elif name == "reciprocal":
            k(f"rcp.rn.f32 {r}, {x}")
        elif name == "rsqrt":
            s = k.reg("f32")
            k(f"sqrt.rn.f32 {s}, {x}")
            k(f"rcp.rn.f32 {r}, {s}")
        elif name in ("log", "log2", "log10"):
            l2 = k.reg("f32")
            k(f"lg2.approx.f32 {l2}, {x}")
            if name == "log2":
                return Val(l2, "f32")
            c = LN2 if name == "log" else math.log10(2.0)
            k(f"mul.rn.f32 {r}, {l2}, {f32_hex(c)}")
        elif name == "relu":
            p = k.reg("pred")
            k(f"setp.gt.f32 {p}, {x}, 0f00000000")
            k(f"selp.f32 {r}, {x}, 0f00000000, {p}")
        elif name == "sigmoid":
            n = k.reg("f32")
            k(f"neg.f32 {n}, {x}")
            e = self.exp_f32(n)
            d = k.reg("f32")
            k(f"add.rn.f32 {d}, {e}, {one}")
            k(f"rcp.rn.f32 {r}, {d}")
        elif name == "silu":
            n = k.reg("f32")
            k(f"neg.f32 {n}, {x}")
            e = self.exp_f32(n)
            d = k.reg("f32")
            k(f"add.rn.f32 {d}, {e}, {one}")
            k(f"div.rn.f32 {r}, {x}, {d}")
        elif name == "tanh":
            # tanh(x) = sign(x) * (1 - 2 / (exp(2|x|) + 1))
            a, t2, d, q, s = (k.reg("f32") for _ in range(5))
            k(f"abs.f32 {a}, {x}")
            k(f"add.rn.f32 {t2}, {a}, {a}")
            e = self.exp_f32(t2)
            k(f"add.rn.f32 {d}, {e}, {one}")
            k(f"div.rn.f32 {q}, 0f40000000, {d}")
            k(f"sub.rn.f32 {s}, {one}, {q}")
            k(f"copysign.f32 {r}, {x}, {s}")
        elif name == "softplus":
            e = self.exp_f32(x)
            d = k.reg("f32")
            k(f"add.rn.f32 {d}, {e}, {one}")
            l2 = k.reg("f32")
            k(f"lg2.approx.f32 {l2}, {d}")
            k(f"mul.rn.f32 {r}, {l2}, {f32_hex(LN2)}")
        elif name in ("floor", "ceil", "trunc", "round"):
            mode = {"floor": "rmi", "ceil": "rpi", "trunc": "rzi", "round": "rni"}[name]
            k(f"cvt.{mode}.f32.f32 {r}, {x}")
        elif name == "sign":
            pg, pl = k.reg("pred"), k.reg("pred")
            k(f"setp.gt.f32 {pg}, {x}, 0f00000000")
            k(f"setp.lt.f32 {pl}, {x}, 0f00000000")
            k(f"selp.f32 {r}, 0fBF800000, 0f00000000, {pl}")
            k(f"selp.f32 {r}, {one}, {r}, {pg}")
        elif name in ("sin", "cos"):
            k(f"{name}.approx.f32 {r}, {x}")
        elif name == "isnan":
            p = k.reg("pred")
            k(f"testp.notanumber.f32 {p}, {x}")
            return Val(p, "pred")
        elif name == "isinf":
            p = k.reg("pred")
            k(f"testp.infinite.f32 {p}, {x}")
            return Val(p, "pred")
        else:
            raise LowerError(f"unary op {name!r}")
        return Val(r, "f32")

    # -- scalar statements -------------------------------------------------

    def identity(self, op_or_value, kind: str, store: str | None = None) -> Val:
        """An accumulator's start value: the op's identity or a literal,
        made an f32 first and then stored in ``kind`` -- and rounded to f16
        or bf16 when that is the accumulator's storage type
        (``interp.py:732-739``)."""
        if kind in ("s32", "s64"):
            v = int(ops.identity(op_or_value)) if isinstance(op_or_value, str) else int(op_or_value)
            return self.const(v, kind)
        v = ops.identity(op_or_value) if isinstance(op_or_value, str) else float(op_or_value)
        v = _round_storage(v, store)
        return self.const(v, kind)

    def _round(self, v: Val, dtype) -> Val:
        """Coerce to the value kind of ``dtype`` and, for f16/bf16, round to
        the storage precision (``interp.py:128-131``, one ``cvt.rn``)."""
        v = self.coerce(v, value_kind(dtype))
        if storage_kind(dtype) in ("f16", "bf16"):
            v = self.coerce(v, storage_kind(dtype))
        return v

    def do_assign(self, st: ir.Assign) -> None:
        for a in st.args:
            if a not in self.env:
                raise LowerError(f"undefined name {a!r}")
        r = self.apply(st.op.name, [self.env[a] for a in st.args])
        if st.dtype is not None:
            r = self._round(r, st.dtype)
        self.bind(st.name, r)

    def do_let(self, st: ir.Let) -> None:
        v = self.ev(st.value)
        if st.dtype is not None:
            v = self._round(v, st.dtype)
        self.bind(st.name, v)

    def do_init(self, st: ir.Init) -> None:
        self.bind(st.name, self.identity(st.identity, value_kind(st.dtype),
                                         storage_kind(st.dtype)))

    def do_accum(self, st: ir.Accum) -> None:
        kind = value_kind(st.dtype) if st.dtype is not None else "f32"
        store = storage_kind(st.dtype) if st.dtype is not None else None
        acc = self.env.get(st.name)
        if acc is None or acc.kind != kind:
            acc = self.bind(st.name, self.identity(st.op.name, kind, store))
        left = self.env[st.base] if st.base is not None else acc
        if st.value not in self.env:
            raise LowerError(f"undefined name {st.value!r}")
        r = self.apply(st.op.name, [left, self.env[st.value]])
        if st.dtype is not None:
            r = self._round(r, st.dtype)
        self.bind(st.name, r)

    def seed_accums(self, body, enabled: bool) -> None:
        """Loop-entry seeding of the loop's own accumulators
        (``interp.py:782-801``).  The reference seeds them on every lane, not
        only the active ones (``interp.py:794`` assigns the identity without
        the mask), so a loop inside a ``Cond`` resets its accumulator to the
        identity on lanes that do not take the branch too: the seed is an
        unpredicated move."""
        seen: set[str] = set()

        def visit(stmts):
            for st in stmts:
                if isinstance(st, ir.Accum):
                    if st.name in seen:
                        continue
                    seen.add(st.name)
                    if enabled:
                        kind = value_kind(st.dtype) if st.dtype is not None else "f32"
                        store = storage_kind(st.dtype) if st.dtype is not None else None
                        saved, self.mask = self.mask, None
                        self.bind(st.name, self.identity(st.op.name, kind, store))
                        self.mask = saved
                elif isinstance(st, (ir.Loop, ir.StridedLoop)):
                    continue
                else:
                    for child in st.nested():
                        visit(child)

        visit(body)

    def run(self, body) -> None:
        for st in body:
            self.stmt(st)

    def stmt(self, st) -> None:
        t = type(st)
        if t in self.extra:
            self.extra[t](st)
        elif t is ir.Assign:
            self.do_assign(st)
        elif t is ir.Let:
            self.do_let(st)
        elif t is ir.Init:
            self.do_init(st)
        elif t is ir.Accum:
            self.do_accum(st)
        elif t is ir.Load:
            if self.load_hook is None:
                raise LowerError("Load outside a template context")
            self.load_hook(st)
        elif t is ir.Write:
            if self.write_hook is None:
                raise LowerError("Write outside a template context")
            self.write_hook(st)
        elif t is ir.Cond:
            self.do_cond(st)
        elif t in (ir.Smem, ir.Sync):
            pass
        else:
            raise LowerError(f"statement {t.__name__} in this context")

    def do_cond(self, st: ir.Cond) -> None:
        k = self.k
        c = self.truthy(self.ev(st.cond))
        skip = k.label("cond_else")
        done = k.label("cond_end")
        k(f"@!{c.reg} bra {skip}")
        self.run(st.body)
        if st.else_body:
            k(f"bra.uni {done}")
        k.place(skip)
        if st.else_body:
            self.run(st.else_body)
            k.place(done)

    def shuffle_combine(self, states, states_b, combine, length: int = 32) -> None:
        """XOR butterfly over a full warp (every lane active) with the IR's
        own combine statements (``interp.py:868-888``)."""
        k = self.k
        off = length // 2
        while off > 0:
            for s, sb in zip(states, states_b):
                cur = self.env[s]
                if cur.kind not in ("f32", "s32"):
                    raise LowerError("shuffle of a non-32-bit state")
                r = k.reg(cur.kind)
                k(f"shfl.sync.bfly.b32 {r}, {cur.reg}, {off}, 31, -1")
                self.bind(sb, Val(r, cur.kind))
            self.run(combine)
            off //= 2
