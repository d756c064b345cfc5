"""Differential fuzzing of the IR -> sm_100a path (test infrastructure).

``case(seed)`` draws one kernel from the IR families the reference ships --
pointwise op DAGs, full reductions, row reductions and fused rows, tiled and
split-K matmul, online-softmax attention (f32 and bf16) -- with random
shapes, thread counts and element-wise programs, builds its IR with
``ptxgen.irgen`` (the shipped problems' repr grammar and meta.json schema)
and seeded inputs.  ``compare(case, got, want)`` applies the family's bound:
bit-exact for DAGs of exactly rounded ops, otherwise the tolerance the
reference's own tests use for that family.

Random pointwise DAGs stay finite by construction: every value carries an
upper bound on its magnitude and an op whose result could pass 1e30 is not
drawn, divisors are |b| + 1, and the ex2-based ops only see loaded inputs.

A second generator, seeded apart from the one that draws the program, picks
the element type of pointwise cases (f32, f64, or f16 when the program is
exactly rounded and its bound stays below f16's range) and of full and row
sums (f32 or f16 input): the reference's f16/f64 value kinds
(``ptxgen/interp.py:115-141``) under the same families.
"""

from __future__ import annotations

import dataclasses

import numpy as np

from ptxgen import irgen
from ptxgen.loader import load_kernel_data

EXACT_UNARY = ("negative", "absolute", "relu", "square")
EXACT_BINARY = ("add", "subtract", "multiply", "maximum", "minimum", "divide")
APPROX_UNARY = ("exp", "tanh", "sigmoid")
FAMILIES = ("pointwise", "reduce_full", "rows", "matmul", "splitk", "attention")
_NPT = {"f32": np.float32, "f64": np.float64, "f16": np.float16}


@dataclasses.dataclass
class Case:
    name: str
    family: str
    spec: object
    inputs: dict
    exact: bool
    tol: float
    extra: dict = dataclasses.field(default_factory=dict)


def _pointwise_program(rng):
    n_vec = int(rng.integers(1, 4))
    consts = [(f"c{i}", float(np.float32(rng.uniform(-2, 2))))
              for i in range(int(rng.integers(0, 3)))]
    steps, bound, loaded = [], {}, []
    for i in range(n_vec):
        steps.append(("load", f"in{i}", f"x{i}", "vec"))
        bound[f"in{i}"] = 6.0
        loaded.append(f"in{i}")
    for i, (c, v) in enumerate(consts):
        steps.append(("load", f"k{i}", c, "const"))
        bound[f"k{i}"] = abs(v)
    need_one = False
    exact = True
    for j in range(int(rng.integers(1, 7))):
        avail = list(bound)
        for _ in range(20):
            r = rng.random()
            if r < 0.55:
                op = str(rng.choice(EXACT_BINARY))
                a, b = (str(x) for x in rng.choice(avail, 2))
                if op == "divide":
                    bb = bound[a]
                elif op == "multiply":
                    bb = bound[a] * bound[b]
                elif op in ("add", "subtract"):
                    bb = bound[a] + bound[b]
                else:
                    bb = max(bound[a], bound[b])
                args = (a, b)
            elif r < 0.85:
                op = str(rng.choice(EXACT_UNARY))
                a = str(rng.choice(avail))
                bb = bound[a] ** 2 if op == "square" else bound[a]
                args = (a,)
            else:
                op = str(rng.choice(APPROX_UNARY))
                a = str(rng.choice(loaded))
                bb = float(np.exp(bound[a])) if op == "exp" else 1.0
                args = (a,)
            if bb < 1e30:
                break
        else:
            continue
        if op == "divide":
            # denominator |b| + 1 >= 1
            steps.append(("op", f"d{j}", "absolute", args[1]))
            steps.append(("op", f"e{j}", "add", f"d{j}", "one"))
            args = (args[0], f"e{j}")
            need_one = True
        if op in APPROX_UNARY:
            exact = False
        steps.append(("op", f"v{j}", op, *args))
        bound[f"v{j}"] = bb
    if not any(s[0] == "op" for s in steps):
        steps.append(("op", "v0", "negative", "in0"))
    if need_one:
        steps.insert(0, ("load", "one", "c_one", "const"))
        consts.append(("c_one", 1.0))
    return steps, consts, exact, max(bound.values())


def _draw(rng, family, seed):
    f32 = np.float32
    drng = np.random.default_rng(50_000 + seed)      # element-type draws only
    if family == "pointwise":
        steps, consts, exact, top = _pointwise_program(rng)
        unroll = int(rng.choice([1, 2, 4]))
        n = unroll * int(rng.integers(1, 1 << 15))
        vec = sorted({s[2] for s in steps if s[0] == "load" and s[3] == "vec"})
        r = drng.random()
        dt = "f64" if r < 0.2 else ("f16" if r < 0.4 and exact and top < 3e4 else "f32")
        g, m = irgen.pointwise(n, unroll, steps, out="out", constants=consts,
                               block=int(rng.choice([64, 128, 256, 512])),
                               entry="k_fuzz_pointwise", pid=f"fuzz{seed}", dtype=dt)
        ins = {b: rng.standard_normal(n).astype(f32).astype(_NPT[dt]) for b in vec}
        return g, m, ins, exact, 1e-5, {"n": n, "program": steps, "dtype": dt}
    if family == "reduce_full":
        n = int(rng.integers(1, 1 << 18))
        threads = int(rng.choice([32, 64, 128, 256, 512, 1024]))
        mean = bool(rng.random() < 0.3)
        dt = "f16" if drng.random() < 0.25 else "f32"
        g, m = irgen.reduce_full(n, threads=threads, mean=mean, pid=f"fuzz{seed}", dtype=dt)
        x = rng.uniform(-1, 1, n).astype(f32).astype(_NPT[dt])
        return g, m, {"x": x}, False, 1e-5, {"n": n, "dtype": dt}
    if family == "rows":
        kind = str(rng.choice(["rowsum", "rmsnorm", "softmax", "l2norm"]))
        rows = int(rng.integers(1, 200))
        cols = int(rng.integers(1, 3000))
        threads = int(rng.choice([32, 64, 128, 256]))
        if kind == "rowsum":
            dt = "f16" if drng.random() < 0.25 else "f32"
            g, m = irgen.reduce_rows(rows, cols, threads=threads, pid=f"fuzz{seed}", dtype=dt)
            x = rng.standard_normal((rows, cols)).astype(f32).astype(_NPT[dt])
            return g, m, {"x": x}, False, 1e-5, {"kind": kind, "rows": rows, "cols": cols,
                                                  "dtype": dt}
        elif kind == "rmsnorm":
            g, m = irgen.rmsnorm(rows, cols, threads=threads, pid=f"fuzz{seed}")
        elif kind == "softmax":
            g, m = irgen.softmax(rows, cols, threads=threads, pid=f"fuzz{seed}")
        else:
            g, m = irgen.l2norm(rows, cols, threads=threads, pid=f"fuzz{seed}")
        spec = load_kernel_data(g, m, "x")
        ins = {}
        for name in spec.arg_order:
            a = spec.args[name]
            if not a.output and a.data is None:
                ins[name] = rng.standard_normal(a.shape).astype(f32)
        return g, m, ins, False, 1e-5, {"kind": kind, "rows": rows, "cols": cols}
    if family == "matmul":
        mm, nn, kk = (32 * int(rng.integers(1, 9)), 64 * int(rng.integers(1, 5)),
                      64 * int(rng.integers(2, 5)))
        g, m = irgen.matmul(mm, nn, kk, pid=f"fuzz{seed}")
        ins = {"x0": rng.uniform(-1, 1, (mm, kk)).astype(f32),
               "x1": rng.uniform(-1, 1, (kk, nn)).astype(f32)}
        return g, m, ins, False, 1e-4, {"mnk": (mm, nn, kk)}
    if family == "splitk":
        sk = 8 * int(rng.integers(1, 5))
        mm, nn, kk = (16 * int(rng.integers(1, 9)), 32 * int(rng.integers(1, 5)),
                      sk * int(rng.integers(1, 9)))
        g, m = irgen.matmul_splitk(mm, nn, kk, slice_k=sk, pid=f"fuzz{seed}")
        ins = {"x0": rng.uniform(-1, 1, (mm, kk)).astype(f32),
               "x1": rng.uniform(-1, 1, (kk, nn)).astype(f32)}
        return g, m, ins, False, 1e-4, {"mnk": (mm, nn, kk), "slice_k": sk}
    if family == "attention":
        dt = str(rng.choice(["f32", "bf16"]))
        b, h = int(rng.integers(1, 3)), 1
        s = int(rng.choice([32, 64, 96, 128]))
        d = int(rng.choice([32, 64]))
        g, m = irgen.attention_bhsd(b, h, s, d, dt, pid=f"fuzz{seed}")
        if dt == "bf16":
            from ml_dtypes import bfloat16
            mk = lambda: rng.standard_normal((b, h, s, d)).astype(bfloat16)  # noqa: E731
        else:
            mk = lambda: rng.standard_normal((b, h, s, d)).astype(f32)  # noqa: E731
        ins = {"q": mk(), "k": mk(), "v": mk()}
        return g, m, ins, False, (1e-4 if dt == "f32" else 2e-2), {"shape": (b, h, s, d),
                                                                      "dtype": dt}
    raise ValueError(family)


def case(seed: int) -> Case:
    rng = np.random.default_rng(10_000 + seed)
    family = FAMILIES[seed % len(FAMILIES)]
    g, m, ins, exact, tol, extra = _draw(rng, family, seed)
    spec = load_kernel_data(g, m, f"fuzz{seed}")
    # ``data`` arguments (ConstantOps) travel with the inputs, as the runner
    # passes them (the GPU launcher uploads them itself; the oracle needs them)
    from ptxgen.runtime import _np_dtype
    for name in spec.arg_order:
        a = spec.args[name]
        if a.data is not None and not a.output and name not in ins:
            ins[name] = np.asarray(a.data, dtype=np.float64).astype(
                _np_dtype(a.dtype)).reshape(a.shape)
    return Case(f"fuzz{seed}_{family}", family, spec, ins, exact, tol, extra)


def compare(c: Case, got: dict, want: dict) -> None:
    """Raise AssertionError when ``got`` is outside the family's bound."""
    for name, ref in want.items():
        g = np.asarray(got[name]).astype(np.float64)
        r = np.asarray(ref).astype(np.float64)
        if c.exact:
            assert np.array_equal(g, r, equal_nan=True), (c.name, name)
            continue
        if c.family in ("matmul", "splitk"):
            a = np.abs(c.inputs["x0"].astype(np.float64))
            b = np.abs(c.inputs["x1"].astype(np.float64))
            bound = c.tol * (a @ b) + 1e-6
        elif c.family == "attention":
            bound = c.tol * max(np.abs(r).max(), 1e-6)
        elif c.family == "reduce_full" or c.extra.get("kind") == "rowsum":
            x = np.abs(next(iter(c.inputs.values())).astype(np.float64))
            total = x.sum() if c.family == "reduce_full" else x.sum(axis=-1).reshape(r.shape)
            if name == "mean":
                total = total / c.extra["n"]
            bound = c.tol * np.maximum(total, 1e-3)
            if c.extra.get("dtype") == "f16":   # the sum order may move the f16 rounding
                bound = bound + np.spacing(np.abs(np.asarray(ref))).astype(np.float64)
        else:
            bound = c.tol * np.maximum(np.abs(r), 1.0)
        err = np.abs(g - r)
        assert np.all(err <= bound), (c.name, name, float(err.max()), c.extra)
