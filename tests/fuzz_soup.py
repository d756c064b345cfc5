"""Random statement mixes for the generic lowering (test infrastructure).

``case(seed)`` draws one kernel that is not shaped like any shipped family:
a ``Tile`` over N cells whose body is a random mix of

* ``Load`` of the cell's element of ``x0``/``x1`` or of a gathered element of
  a small table ``t`` (index ``(a0 * p + q) % K``, or ``(a0 + j * s) % K``
  inside a loop over ``j``);
* ``Let`` of a float literal and ``Assign`` of exactly rounded ops;
* ``Cond`` with and without an else body, nested up to depth 2, its
  predicate an integer test of the cell index or a float test of an earlier
  value -- names first defined inside a branch stay visible after it and
  hold 0 on the lanes that did not run it (``ptxgen/interp.py:458-468``);
* ``Select`` chains of two or three branches (``ptxgen/interp.py:960-972``);
* ``Loop`` over a short axis folding an ``Accum`` (add, max or min) that the
  loop seeds (``ptxgen/interp.py:803-821``), and ``StridedLoop``s whose
  start depends on the cell (``a0 % m``), so each lane runs its own trip
  count -- none at all when the start is past the extent, which leaves the
  accumulator at its identity (``ptxgen/interp.py:828-856``);
* integer values: ``Let`` of an int literal or of an index expression of
  the cell, ``Assign`` of s32 add, subtract, multiply, max, min, divide (by
  zero gives 0), remainder, bit and/or/xor and shifts (count masked to 5
  bits) -- ``ptxgen/interp.py:180-200``, ``:359-373`` -- integer
  predicates, and integers mixed into float ops (promoted to f32);
* shared memory (a seeded 40 % of the cases, every lane active): rounds of
  ``Write`` of a value to the lane's slot ``a0 % B`` of an ``Smem`` array,
  ``Sync``, ``Load`` of another lane's slot ``(a0 + s) % B`` -- a barrier
  also precedes each rewrite, and every slot is written before it is read;
  and in the same cases ``WarpShuffle`` butterflies folding a copy of a
  value over 2 to 32 lanes with add, max or min (``ptxgen/interp.py:868-885``);
* unconditional and conditional ``Write``s of ``out[a0]`` (the last write a
  lane performs wins).

Every op is exactly rounded (add, subtract, multiply, max, min, negative,
absolute, relu, divide by ``|b| + 1``, and the integer ops), so the GPU
result must equal the oracle's bit for bit.  Float magnitudes stay below
1e30 and integer ones below 2^30 by construction (each value carries a
bound; an op that could exceed it is not drawn), so nothing overflows.
"""

from __future__ import annotations

import dataclasses
import math

import numpy as np

from ptxgen import irgen
from ptxgen.ir import (Accum, Assign, BinaryExpr, Cond, ElementwiseImpl, Let, Literal, Load,
                       Loop, Select, SelectBranch, Smem, Sync, Var, WarpShuffle, Write,
                       datatype)
from ptxgen.loader import load_kernel_data

F32 = datatype("f32")
BINARY = ("add", "subtract", "multiply", "maximum", "minimum", "divide")
UNARY = ("negative", "absolute", "relu")
INT_BINARY = ("add", "subtract", "multiply", "maximum", "minimum", "divide", "remainder",
              "bitand", "bitor", "bitxor", "shl", "shr")
INT_LIMIT = float(1 << 30)


@dataclasses.dataclass
class Soup:
    name: str
    spec: object
    inputs: dict
    graph: dict
    meta: dict


def _lit_i(v):
    return Literal(value=int(v), dtype="int")


def _lit_f(v):
    return Literal(value=float(v), dtype="float")


def _b(op, a, b):
    return BinaryExpr(op=op, left=a, right=b)


class _Gen:
    def __init__(self, rng, n, k):
        self.rng, self.n, self.k = rng, n, k
        self.count = 0
        self.bound: dict[str, float] = {}      # name -> magnitude bound
        self.ints: set[str] = set()            # names of s32 values
        self.block_threads = 0                 # > 0: shared-memory rounds on
        self.smem_written = False
        self.nonneg: set[str] = set()          # s32 names known to be >= 0

    def fresh(self, prefix="v"):
        self.count += 1
        return f"{prefix}{self.count}"

    def int_pred(self):
        r = self.rng.random()
        a0 = Var(name="a0")
        if r < 0.4:
            m = int(self.rng.integers(2, 9))
            return _b("==", _b("%", a0, _lit_i(m)), _lit_i(int(self.rng.integers(0, m))))
        if r < 0.7:
            return _b("<", a0, _lit_i(int(self.rng.integers(0, self.n + 1))))
        m = int(self.rng.integers(2, 9))
        return _b("<", _b("%", a0, _lit_i(m)), _lit_i(int(self.rng.integers(1, m))))

    def pred(self, scope):
        ints = [v for v in scope if v in self.ints]
        r = self.rng.random()
        if ints and r < 0.2:
            v = str(self.rng.choice(ints))
            c = int(self.rng.integers(-20, 21))
            return _b(str(self.rng.choice(["<", "=="])), Var(name=v), _lit_i(c))
        if scope and r < 0.5:
            v = str(self.rng.choice(scope))
            return _b("<", Var(name=v), _lit_f(float(np.float32(self.rng.uniform(-1, 1)))))
        return self.int_pred()

    def int_let(self, scope, out):
        name = self.fresh("i")
        if self.rng.random() < 0.5:
            v = int(self.rng.integers(-40, 41))
            out.append(Let(name=name, value=_lit_i(v), dtype=None))
            self.bound[name] = float(abs(v))
            nonneg = v >= 0
        else:
            p, q = int(self.rng.integers(1, 5)), int(self.rng.integers(-9, 10))
            m = int(self.rng.integers(2, 17))
            if self.rng.random() < 0.5:
                e = _b("+", _b("*", Var(name="a0"), _lit_i(p)), _lit_i(q))
                self.bound[name] = float(4 * self.n + 10)
                nonneg = q >= 0
            else:
                e = _b("%", Var(name="a0"), _lit_i(m))
                self.bound[name] = float(m)
                nonneg = True
            out.append(Let(name=name, value=e, dtype=None))
        self.ints.add(name)
        if nonneg:
            self.nonneg.add(name)
        scope.append(name)

    def int_assign(self, scope, out):
        ints = [v for v in scope if v in self.ints]
        for _ in range(20):
            op = str(self.rng.choice(INT_BINARY))
            a, b = str(self.rng.choice(ints)), str(self.rng.choice(ints))
            ba, bb = self.bound[a], self.bound[b]
            na, nb = a in self.nonneg, b in self.nonneg
            if op in ("shl", "shr"):
                # the count is masked to 5 bits: only a count known to lie
                # in [0, 31) keeps the bound
                if not nb or bb >= 31:
                    continue
                bnd = ba * 2.0 ** bb if op == "shl" else ba
            else:
                bnd = {"add": ba + bb, "subtract": ba + bb, "multiply": ba * bb,
                       "maximum": max(ba, bb), "minimum": max(ba, bb), "divide": ba,
                       "remainder": min(ba, bb) if nb else ba, "bitand": max(ba, bb),
                       "bitor": 2 * max(ba, bb), "bitxor": 2 * max(ba, bb)}[op]
            if bnd >= INT_LIMIT:
                continue
            name = self.fresh("i")
            out.append(Assign(name=name, op=ElementwiseImpl(op), args=(a, b), dtype=None))
            self.bound[name] = bnd
            self.ints.add(name)
            nonneg = {"add": na and nb, "multiply": na and nb, "maximum": na or nb,
                      "minimum": na and nb, "divide": na and nb, "remainder": na,
                      "bitand": na or nb, "bitor": na and nb, "bitxor": na and nb,
                      "shl": na, "shr": na}.get(op, False)
            if nonneg:
                self.nonneg.add(name)
            scope.append(name)
            return
        self.int_let(scope, out)

    def pick(self, scope):
        return str(self.rng.choice(scope))

    def assign(self, scope, out):
        for _ in range(20):
            if self.rng.random() < 0.7 and len(scope) >= 1:
                op = str(self.rng.choice(BINARY))
                a, b = self.pick(scope), self.pick(scope)
                ba, bb = self.bound[a], self.bound[b]
                if op == "divide":
                    bnd = ba                          # a / (|b| + 1)
                elif op == "multiply":
                    bnd = ba * bb
                elif op in ("add", "subtract"):
                    bnd = ba + bb
                else:
                    bnd = max(ba, bb)
                if bnd >= 1e30:
                    continue
                if op == "divide":
                    d, e = self.fresh("d"), self.fresh("e")
                    one = self.fresh("one")
                    out.append(Assign(name=d, op=ElementwiseImpl("absolute"), args=(b,), dtype=F32))
                    out.append(Let(name=one, value=_lit_f(1.0), dtype=F32))
                    out.append(Assign(name=e, op=ElementwiseImpl("add"), args=(d, one), dtype=F32))
                    b = e
                name = self.fresh()
                out.append(Assign(name=name, op=ElementwiseImpl(op), args=(a, b), dtype=F32))
            else:
                op = str(self.rng.choice(UNARY))
                a = self.pick(scope)
                bnd = self.bound[a]
                name = self.fresh()
                out.append(Assign(name=name, op=ElementwiseImpl(op), args=(a,), dtype=F32))
            self.bound[name] = bnd
            scope.append(name)
            return
        # nothing fitted: a plain negation keeps the mix going
        a = self.pick(scope)
        name = self.fresh()
        out.append(Assign(name=name, op=ElementwiseImpl("negative"), args=(a,), dtype=F32))
        self.bound[name] = self.bound[a]
        scope.append(name)

    def load(self, scope, out, index=None):
        name = self.fresh("in")
        if index is not None:
            out.append(Load(names=(name,), input="t", index=(index,), dtype=F32))
        elif self.rng.random() < 0.7:
            buf = str(self.rng.choice(["x0", "x1"]))
            out.append(Load(names=(name,), input=buf, index=(Var(name="a0"),), dtype=F32))
        else:
            p, q = int(self.rng.integers(1, 7)), int(self.rng.integers(0, 7))
            idx = _b("%", _b("+", _b("*", Var(name="a0"), _lit_i(p)), _lit_i(q)), _lit_i(self.k))
            out.append(Load(names=(name,), input="t", index=(idx,), dtype=F32))
        self.bound[name] = 6.0
        scope.append(name)

    def strided(self, scope, out):
        """A per-lane loop: j = a0 % m, a0 % m + step, ... while j < ext."""
        ext = int(self.rng.integers(1, 12))
        m = int(self.rng.integers(1, 5))
        step = int(self.rng.integers(1, 4))
        ax = self.fresh("j")
        idx = _b("%", _b("+", Var(name="a0"), Var(name=ax)), _lit_i(self.k))
        body, inner = [], list(scope)
        self.load(inner, body, index=idx)
        loaded = inner[-1]
        other = self.pick(scope)
        bo = self.bound[other]
        op = "add" if bo + 6.0 < 1e29 else "maximum"
        t = self.fresh("t")
        body.append(Assign(name=t, op=ElementwiseImpl(op), args=(loaded, other), dtype=F32))
        aop = str(self.rng.choice(["add", "maximum", "minimum"]))
        acc = self.fresh("acc")
        body.append(Accum(name=acc, value=t, op=ElementwiseImpl(aop), dtype=F32,
                          axes=(ax,), base=None))
        out.append(irgen.strided(ax, ext, _b("%", Var(name="a0"), _lit_i(m)), _lit_i(step),
                                 body))
        bt = 6.0 + bo
        # a lane whose start is past ext keeps the identity (+-1e30 for max/min)
        self.bound[acc] = bt * ext if aop == "add" else max(bt, 1e30)
        scope.append(acc)

    def smem_round(self, scope, out):
        """Each lane writes its slot, a barrier, each lane reads another's."""
        b = self.block_threads
        v = self.pick(scope)
        if self.smem_written:
            out.append(Sync(barrier_id=0, count=None, warp=False))   # reads done before rewrite
        out.append(Write(output="sm", index=(_b("%", Var(name="a0"), _lit_i(b)),), values=(v,),
                         value_dtype=F32, atomic=False, swizzle="NONE"))
        out.append(Sync(barrier_id=0, count=None, warp=False))
        s_ = int(self.rng.integers(1, b + 1))
        name = self.fresh("sh")
        out.append(Load(names=(name,), input="sm",
                        index=(_b("%", _b("+", Var(name="a0"), _lit_i(s_)), _lit_i(b)),),
                        dtype=F32))
        self.smem_written = True
        self.bound[name] = self.bound[v]
        scope.append(name)

    def shuffle_round(self, scope, out):
        """A copy of a loaded value folded over ``length`` lanes by a
        butterfly (a loaded value differs per lane; the reference shuffles
        per-lane values only)."""
        loaded = [n for n in scope if n.startswith(("in", "sh"))]
        if not loaded:
            self.smem_round(scope, out)
            return
        v = str(self.rng.choice(loaded))
        length = int(self.rng.choice([2, 4, 8, 16, 32]))
        op = str(self.rng.choice(["add", "maximum", "minimum"]))
        if op == "add" and self.bound[v] * length >= 1e30:
            op = "maximum"
        w = self.fresh("w")
        out.append(Assign(name=w, op=ElementwiseImpl("copy"), args=(v,), dtype=F32))
        wb = f"{w}__o"
        out.append(WarpShuffle(state=(w,), state_b=(wb,),
                               combine_states=(Assign(name=w, op=ElementwiseImpl(op),
                                                      args=(w, wb), dtype=None),),
                               length=length, dtype=F32))
        self.bound[w] = self.bound[v] * (length if op == "add" else 1)
        scope.append(w)

    def block(self, scope, depth, nstmts):
        out = []
        for _ in range(nstmts):
            if depth == 0 and self.block_threads and scope and self.rng.random() < 0.15:
                if self.rng.random() < 0.5:
                    self.smem_round(scope, out)
                else:
                    self.shuffle_round(scope, out)
                continue
            r = self.rng.random()
            if r < 0.16 or not scope:
                self.load(scope, out)
            elif r < 0.36:
                self.assign(scope, out)
            elif r < 0.46:
                if not any(v in self.ints for v in scope) or self.rng.random() < 0.3:
                    self.int_let(scope, out)
                else:
                    self.int_assign(scope, out)
            elif r < 0.50:
                name = self.fresh("c")
                v = float(np.float32(self.rng.uniform(-2, 2)))
                out.append(Let(name=name, value=_lit_f(v), dtype=F32))
                self.bound[name] = abs(v)
                scope.append(name)
            elif r < 0.64 and depth < 2:
                pred = self.pred(scope)
                inner = list(scope)
                body = self.block(inner, depth + 1, int(self.rng.integers(1, 4)))
                else_body = ()
                inner2 = list(scope)
                if self.rng.random() < 0.5:
                    else_body = tuple(self.block(inner2, depth + 1, int(self.rng.integers(1, 4))))
                out.append(Cond(cond=pred, body=tuple(body), else_body=else_body))
                # names defined in a branch stay visible (0 where it did not run)
                for nm in inner + inner2:
                    if nm not in scope:
                        scope.append(nm)
            elif r < 0.74 and len(scope) >= 2:
                nb = int(self.rng.integers(2, 4))
                vals = [self.pick(scope) for _ in range(nb)]
                branches = [SelectBranch(value=v, select=self.pred(scope)) for v in vals[:-1]]
                branches.append(SelectBranch(value=vals[-1], select=None))
                name = self.fresh("s")
                out.append(Select(name=name, branches=tuple(branches)))
                self.bound[name] = max(self.bound[v] for v in vals)
                scope.append(name)
            elif r < 0.84 and depth < 2 and scope:
                ext = int(self.rng.integers(1, 7))
                ax = self.fresh("j")
                s_ = int(self.rng.integers(1, 5))
                idx = _b("%", _b("+", Var(name="a0"), _b("*", Var(name=ax), _lit_i(s_))),
                         _lit_i(self.k))
                body, inner = [], list(scope)
                self.load(inner, body, index=idx)
                loaded = inner[-1]
                other = self.pick(scope)
                op = str(self.rng.choice(["add", "multiply", "maximum"]))
                t = self.fresh("t")
                bt = (self.bound[loaded] * self.bound[other] if op == "multiply"
                      else self.bound[loaded] + self.bound[other])
                if bt * ext >= 1e30:
                    op, bt = "maximum", max(self.bound[loaded], self.bound[other])
                body.append(Assign(name=t, op=ElementwiseImpl(op), args=(loaded, other), dtype=F32))
                aop = str(self.rng.choice(["add", "maximum", "minimum"]))
                acc = self.fresh("acc")
                body.append(Accum(name=acc, value=t, op=ElementwiseImpl(aop), dtype=F32,
                                  axes=(ax,), base=None))
                out.append(Loop(axis=irgen.ax(ax, ext), body=tuple(body), unroll=False, seed=True))
                # the loop runs 1..6 times: a max/min fold is one of its
                # values, a sum at most ext of them (lanes that skip the loop
                # under a Cond hold 0)
                self.bound[acc] = bt * ext if aop == "add" else bt
                scope.append(acc)
            elif r < 0.90 and depth < 2 and scope:
                self.strided(scope, out)
            else:
                if scope:
                    v = self.pick(scope)
                    if depth == 0 or self.rng.random() < 0.5:
                        out.append(Write(output="out", index=(Var(name="a0"),), values=(v,),
                                         value_dtype=F32, atomic=False, swizzle="NONE"))
                    else:
                        out.append(Cond(cond=self.pred(scope), body=(
                            Write(output="out", index=(Var(name="a0"),), values=(v,),
                                  value_dtype=F32, atomic=False, swizzle="NONE"),), else_body=()))
        return out


def case(seed: int) -> Soup:
    rng = np.random.default_rng(77_000 + seed)
    n = int(rng.integers(1, 5000))
    k = int(rng.integers(1, 65))
    block = int(rng.choice([32, 64, 128, 256]))
    srng = np.random.default_rng(88_000 + seed)       # shared-memory draws only
    shared = srng.random() < 0.4
    if shared:
        n = block * int(srng.integers(1, 21))         # every lane of every CTA active
    g = _Gen(rng, n, k)
    if shared:
        g.block_threads = block
    scope: list[str] = []
    body = g.block(scope, 0, int(rng.integers(4, 14)))
    if shared and not g.smem_written:
        g.smem_round(scope, body)
    if g.smem_written:
        body.insert(0, Smem(name="sm", extents=(block,), dtype="float", align=0))
    # every lane writes at least once, at the end
    body.append(Write(output="out", index=(Var(name="a0"),), values=(scope[-1],),
                      value_dtype=F32, atomic=False, swizzle="NONE"))
    t = irgen.tile([irgen.ax("a0", n)], body)
    inputs = [("t", (k,), "f32", 2), ("x0", (n,), "f32", 0), ("x1", (n,), "f32", 1)]
    graph, meta = irgen.package("k_soup", "out", [t], inputs, [], ("out", (n,), "f32"),
                                ["x0", "x1", "t", "out"], (math.ceil(n / block), 1, 1),
                                (block, 1, 1), rtol=0.0, atol=0.0, pid=f"soup{seed}")
    spec = load_kernel_data(graph, meta, f"soup{seed}")
    ins = {"x0": rng.standard_normal(n).astype(np.float32),
           "x1": rng.standard_normal(n).astype(np.float32),
           "t": rng.standard_normal(k).astype(np.float32)}
    return Soup(f"soup{seed}", spec, ins, graph, meta)
