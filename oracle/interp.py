"""CPU oracle for Emmy Kernel IR: a numpy restatement of the reference's
golden model ``ptxgen/interp.py`` (ColonelToad/emmy-ptx).

TEST INFRASTRUCTURE ONLY.  Only ``tests/``, ``__graft_entry__.smoke()`` and
``bench.py``'s CPU-baseline / reference legs may import this module, and only
as the checker (or the timed CPU baseline).  The product path never calls it.

Parity status: pinned.  ``tests/test_oracle.py`` checks this module against
every ``expected.npz`` golden vector shipped with the reference's 15 problems
and, bit for bit, against outputs of the reference interpreter itself that
``tests/golden/make_golden.py`` recorded on extra inputs.

Execution model (same as the reference, ``ptxgen/interp.py:12-17``): one
chunk of CTAs at a time, every thread of the chunk is one lane of a numpy
array, divergence is a boolean lane mask, ``Sync`` is a no-op because all
lanes move in lockstep.

Arithmetic follows the reference rule by rule:

* value kinds and PTX ``cvt`` coercions        -- ``interp.py:115-141``
* type promotion of binary ops                  -- ``interp.py:107-112``
* f32 arithmetic rounds after every op; integer
  division truncates; max/min ignore NaN        -- ``interp.py:172-217``
* transcendentals evaluated in f64, rounded
  once to f32                                   -- ``interp.py:230-319``
* fma is ``a*b+c`` with two roundings; shifts
  mask the count to 5 bits                      -- ``interp.py:322-374``

One deliberate difference: the reference's ``WarpShuffle`` gathers partner
lanes with the *global* CTA index (``interp.py:874-878``), which selects the
wrong lanes once a grid spans more than one chunk (more than 2**20 lanes).
This restatement uses the lane's position inside the chunk, which is what the
``shfl.sync`` the IR stands for does.  Both agree on every single-chunk run,
which covers all golden vectors.

bf16 (absent from the reference) is handled as a storage type: loads widen to
f32 exactly, stores round to nearest even.
"""

from __future__ import annotations

import math
import os
import sys
from contextlib import contextmanager

import numpy as np

_PKG = os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "emmy-ptx_b200")
if _PKG not in sys.path:
    sys.path.insert(0, _PKG)

from ptxgen import ir  # noqa: E402
from ptxgen import ops  # noqa: E402
from ptxgen.model import KernelSpec, dtype_info  # noqa: E402

try:  # bf16 storage; ml_dtypes ships with the image
    from ml_dtypes import bfloat16 as _BF16
except Exception:  # pragma: no cover
    _BF16 = None

_NP = {"f32": np.float32, "f64": np.float64, "f16": np.float16, "s32": np.int32,
       "s64": np.int64, "pred": np.bool_}
_FLOAT = ("f32", "f64", "f16")


def storage_dtype(dtype) -> np.dtype:
    kind = dtype_info(dtype)[0]
    if kind == "bf16":
        if _BF16 is None:
            raise NotImplementedError("bf16 needs ml_dtypes")
        return np.dtype(_BF16)
    return np.dtype(_NP[kind])


# ---------------------------------------------------------------------------
# typed lane values
# ---------------------------------------------------------------------------


class Val:
    """A per-lane value of one kind (f32, f64, f16, s32, s64, pred)."""

    __slots__ = ("kind", "a")

    def __init__(self, kind: str, a):
        self.kind = kind
        self.a = np.asarray(a, dtype=_NP[kind])


def coerce(x: Val, kind: str) -> Val:
    """PTX cvt semantics, as ``interp.py:115-141`` states them."""
    if x.kind == kind:
        return x
    a = x.a
    if x.kind == "pred":
        if kind in ("s32", "s64"):
            return Val(kind, np.where(a, 1, 0))
        return Val(kind, np.where(a, 1.0, 0.0))
    if kind == "f16":
        return Val("f16", a.astype(np.float32).astype(np.float16))
    if kind in ("f32", "f64"):
        return Val(kind, a.astype(_NP[kind]))
    if kind in ("s32", "s64"):
        if x.kind in _FLOAT:  # cvt.rzi: toward zero
            return Val(kind, np.trunc(a.astype(np.float64)).astype(_NP[kind]))
        return Val(kind, a.astype(_NP[kind]))
    raise NotImplementedError(f"coerce {x.kind} -> {kind}")


def truthy(x: Val) -> np.ndarray:
    if x.kind == "pred":
        return x.a
    if x.kind == "f16":
        return x.a.astype(np.float32) != 0
    return x.a != 0


def promote(a: Val, b: Val) -> str:
    """``interp.py:107-112``: f64 wins, any float gives f32, else s32."""
    if a.kind == "f64" or b.kind == "f64":
        return "f64"
    if a.kind in ("f32", "f16") or b.kind in ("f32", "f16"):
        return "f32"
    return "s32"


def as_int64(x: Val) -> np.ndarray:
    if x.kind in ("s32", "s64", "pred"):
        return x.a.astype(np.int64)
    return np.trunc(x.a.astype(np.float64)).astype(np.int64)


def _nan_max(a, b):
    return np.where(np.isnan(a), b, np.where(np.isnan(b), a, np.maximum(a, b)))


def _nan_min(a, b):
    return np.where(np.isnan(a), b, np.where(np.isnan(b), a, np.minimum(a, b)))


def binary_arith(name: str, x: Val, y: Val) -> Val:
    """add/subtract/multiply/divide/maximum/minimum (``interp.py:180-217``)."""
    kind = promote(x, y)
    a, b = coerce(x, kind).a, coerce(y, kind).a
    if kind == "s32":
        if name == "divide":
            af, bf = a.astype(np.float64), b.astype(np.float64)
            with np.errstate(divide="ignore", invalid="ignore"):
                q = np.trunc(af / bf)
            r = np.where(bf != 0, q, 0.0)
        else:
            r = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply,
                 "maximum": np.maximum, "minimum": np.minimum}[name](a, b)
        return Val("s32", np.asarray(r).astype(np.int32))
    with np.errstate(all="ignore"):
        if name == "maximum":
            r = _nan_max(a, b)
        elif name == "minimum":
            r = _nan_min(a, b)
        else:
            r = {"add": np.add, "subtract": np.subtract, "multiply": np.multiply,
                 "divide": np.divide}[name](a, b)
    return Val(kind, r)


def _erf64(x: np.ndarray) -> np.ndarray:
    flat = np.asarray(x, dtype=np.float64).ravel()
    out = np.array([math.erf(t) for t in flat], dtype=np.float64)
    return out.reshape(np.shape(x))


def _f64_then_f32(fn, x):
    with np.errstate(all="ignore"):
        return Val("f32", np.asarray(fn(x.astype(np.float64))).astype(np.float32))


_F64_UNARY = {
    "exp": np.exp, "exp_fast": np.exp, "expm1": np.expm1, "log": np.log, "log1p": np.log1p,
    "log2": np.log2, "log10": np.log10, "sqrt": np.sqrt,
    "rsqrt": lambda t: 1.0 / np.sqrt(t), "reciprocal": lambda t: 1.0 / t,
    "tanh": np.tanh, "sin": np.sin, "cos": np.cos, "sinh": np.sinh, "cosh": np.cosh,
    "sigmoid": lambda t: 1.0 / (1.0 + np.exp(-t)),
    "silu": lambda t: t / (1.0 + np.exp(-t)),
    "softplus": lambda t: np.log1p(np.exp(t)),
    "floor": np.floor, "ceil": np.ceil, "trunc": np.trunc, "round": np.rint,
}


def unary_op(name: str, x: Val) -> Val:
    """Unary ops (``interp.py:230-319``)."""
    if name == "copy":
        return x
    if x.kind == "s32" and name in ("negative", "absolute"):
        return Val("s32", (-x.a if name == "negative" else np.abs(x.a)).astype(np.int32))
    if name == "bitcast":
        a = np.ascontiguousarray(x.a)
        swap = {"f32": ("s32", np.int32), "s32": ("f32", np.float32),
                "f64": ("s64", np.int64), "s64": ("f64", np.float64)}
        if x.kind in swap:
            k, t = swap[x.kind]
            return Val(k, a.view(t))
        return x
    if name == "logical_not":
        return Val("pred", ~truthy(x))
    f = coerce(x, "f32").a
    if name == "negative":
        return Val("f32", -f)
    if name == "absolute":
        return Val("f32", np.abs(f))
    if name == "square":
        return binary_arith("multiply", Val("f32", f), Val("f32", f))
    if name in _F64_UNARY:
        return _f64_then_f32(_F64_UNARY[name], f)
    if name == "erf":
        return Val("f32", _erf64(f).astype(np.float32))
    if name in ("gelu", "gelu_tanh"):
        d = f.astype(np.float64)
        if name == "gelu_tanh":
            t = np.tanh(math.sqrt(2.0 / math.pi) * (d + 0.044715 * d ** 3))
        else:
            t = _erf64((d / math.sqrt(2.0)).astype(np.float32)).astype(np.float32)
            t = t.astype(np.float64)
        return Val("f32", (0.5 * d * (1.0 + t)).astype(np.float32))
    if name == "relu":
        return Val("f32", np.where(f > 0, f, np.float32(0.0)))
    if name == "sign":
        return Val("f32", np.where(f > 0, 1.0, np.where(f < 0, -1.0, 0.0)))
    if name == "isnan":
        return Val("pred", np.isnan(f))
    if name == "isinf":
        return Val("pred", np.isinf(f))
    raise NotImplementedError(f"unsupported unary op {name!r}")


def apply_op(name: str, args: list[Val]) -> Val:
    """Dispatch one elementwise op (``interp.py:322-374``)."""
    name = ops.canon(name)
    if name in ("add", "subtract", "multiply", "divide", "maximum", "minimum"):
        return binary_arith(name, args[0], args[1])
    if name == "fma":
        a, b, c = args
        kind = "f64" if "f64" in (a.kind, b.kind, c.kind) else "f32"
        a, b, c = coerce(a, kind).a, coerce(b, kind).a, coerce(c, kind).a
        return Val(kind, a * b + c)
    if name == "where":
        c, a, b = args
        kind = promote(a, b)
        return Val(kind, np.where(truthy(c), coerce(a, kind).a, coerce(b, kind).a))
    if name == "clip":
        a, lo, hi = args
        return binary_arith("minimum", binary_arith("maximum", a, lo), hi)
    if name == "floor_divide":
        a, b = args
        if a.kind in _FLOAT or b.kind in _FLOAT:
            return unary_op("floor", binary_arith("divide", a, b))
        return binary_arith("divide", a, b)
    if name == "fmod":
        a, b = args
        if a.kind in _FLOAT or b.kind in _FLOAT:
            af, bf = coerce(a, "f32").a, coerce(b, "f32").a
            with np.errstate(all="ignore"):
                return Val("f32", np.fmod(af.astype(np.float64), bf.astype(np.float64))
                           .astype(np.float32))
        with np.errstate(divide="ignore"):     # integer fmod by 0 gives 0
            return Val("s32", np.fmod(coerce(a, "s32").a, coerce(b, "s32").a).astype(np.int32))
    if name in ("logical_and", "logical_or"):
        p, q = truthy(args[0]), truthy(args[1])
        return Val("pred", (p & q) if name == "logical_and" else (p | q))
    if name == "power":
        a, b = coerce(args[0], "f32").a, coerce(args[1], "f32").a
        with np.errstate(all="ignore"):
            r = np.exp(b.astype(np.float64) * np.log(a.astype(np.float64)))
        return Val("f32", r.astype(np.float32))
    if name in ("remainder", "bitand", "bitor", "bitxor", "shl", "shr"):
        a, b = coerce(args[0], "s32").a, coerce(args[1], "s32").a
        if name == "remainder":
            with np.errstate(divide="ignore"):  # integer fmod by 0 gives 0
                return Val("s32", np.fmod(a, b).astype(np.int32))
        if name == "bitand":
            return Val("s32", a & b)
        if name == "bitor":
            return Val("s32", a | b)
        if name == "bitxor":
            return Val("s32", a ^ b)
        sh = b & 31
        return Val("s32", np.left_shift(a, sh) if name == "shl" else np.right_shift(a, sh))
    return unary_op(name, args[0])


# ---------------------------------------------------------------------------
# the machine
# ---------------------------------------------------------------------------

_SWIZZLE = {"B128": (6, 0x7), "B64": (6, 0x3), "B32": (6, 0x1)}
_STEP_LIMIT = 1_000_000


def swizzle_index(flat: np.ndarray, mode) -> np.ndarray:
    """XOR swizzle of a shared-memory element index (``interp.py:578-586``)."""
    base, _, shift_txt = str(mode or "NONE").partition("@")
    if base not in _SWIZZLE:
        return flat
    shift, mask = _SWIZZLE[base]
    if shift_txt:
        shift = int(shift_txt)
    return flat ^ (((flat >> shift) & mask) << 3)


def plan_carries(body):
    """(carrier -> (seed, dtype), id(loop body) -> carriers it carries,
    id(loop body) -> carriers with a Carry inside it, carriers set outside
    every loop).  A carrier's carrying loop is the innermost loop that holds
    all its Carry statements."""
    stacks: dict[str, list] = {}
    info: dict[str, tuple] = {}

    def walk(stmts, stack):
        for st in stmts:
            if isinstance(st, ir.Carry):
                stacks.setdefault(st.name, []).append(stack)
                got = (float(st.seed) if not isinstance(st.seed, ir.Literal) else
                       float(st.seed.value), st.dtype if st.dtype is not None else "f32")
                if info.setdefault(st.name, got) != got:
                    raise ValueError(f"carrier {st.name!r}: Carry seeds or dtypes differ")
            if isinstance(st, (ir.Loop, ir.StridedLoop)):
                walk(st.body, stack + (id(st.body),))
            else:
                for child in st.nested():
                    walk(child, stack)

    walk(body, ())
    home: dict[int, list] = {}
    inside: dict[int, set] = {}
    top = set()
    for c, sts in stacks.items():
        common = sts[0]
        for s_ in sts[1:]:
            n = 0
            while n < min(len(common), len(s_)) and common[n] == s_[n]:
                n += 1
            common = common[:n]
        if common:
            home.setdefault(common[-1], []).append(c)
        else:
            top.add(c)
        for s_ in sts:
            for b in s_:
                inside.setdefault(b, set()).add(c)
    return info, home, inside, top


_TMA_SWIZZLE = {"NONE": 0, "B32": 32, "B64": 64, "B128": 128}


def tma_check_descriptor(d, buf_numel: int, eb: int) -> None:
    """The limits a TmaDescriptor must meet (the TMA unit's, plus a view
    that stays inside its buffer)."""
    shape = tuple(int(e) for e in d.src_shape)
    box = tuple(int(e) for e in d.box_extents)
    span = _TMA_SWIZZLE.get(str(d.swizzle or "NONE"))
    if span is None:
        raise ValueError(f"TMA swizzle {d.swizzle!r}")
    if not 1 <= len(shape) <= 5 or len(box) != len(shape):
        raise ValueError("TMA descriptor rank must be 1..5 with a box of the same rank")
    if int(np.prod(shape)) > buf_numel or min(shape) < 1:
        raise ValueError(f"TMA view {shape} exceeds buffer {d.src_buf!r}")
    if any(not 1 <= b <= 256 for b in box):
        raise ValueError("TMA box extents must be 1..256")
    if (shape[-1] * eb) % 16 or (box[-1] * eb) % 16:
        raise ValueError("TMA row and box row must be multiples of 16 bytes")
    if span and box[-1] * eb != span:
        raise ValueError(f"TMA swizzle {d.swizzle} needs a {span}-byte box row")


def mma_layout(role: str):
    """Row and column of every register-fragment element of each of the 32
    lanes of an ``mma.m16n8k16`` (16-bit A and B, f32 C), as [32, E] arrays
    -- A: (m, k), 8 elements; B: (k, n), 4; C: (m, n), 4 -- the layouts the
    PTX ISA gives for that shape: g = lane >> 2, t = lane & 3."""
    lane = np.arange(32)
    g, t = (lane >> 2)[:, None], (lane & 3)[:, None]
    if role == "a":
        i = np.arange(8)[None]
        return g + 8 * ((i // 2) % 2), 2 * t + (i % 2) + 8 * (i // 4)
    if role == "b":
        i = np.arange(4)[None]
        return 2 * t + (i % 2) + 8 * (i // 2), np.broadcast_to(g, (32, 4))
    i = np.arange(4)[None]
    return g + 8 * (i // 2), 2 * t + (i % 2)


def wgmma_n(shape) -> int:
    """N of an ``m64nNk16`` shape string (0 for any other)."""
    s = str(shape)
    if s.startswith("m64n") and s.endswith("k16"):
        n = int(s[4:-3])
        if n % 8 == 0 and 8 <= n <= 256:
            return n
    return 0


def wgmma_c_layout(n: int):
    """Row and column of the N/2 accumulator elements of each of the 128
    threads of a warpgroup for an m64nNk16 product: warp w holds rows
    16w..16w+15 as N/8 blocks of the m16n8 accumulator layout."""
    tid = np.arange(128)
    w, lane = (tid >> 5)[:, None], tid & 31
    g, t = (lane >> 2)[:, None], (lane & 3)[:, None]
    e = np.arange(n // 2)[None]
    j, i = e // 4, e % 4
    return 16 * w + g + 8 * (i // 2), 8 * j + 2 * t + (i % 2)


def _kind_np(dt: np.dtype) -> str:
    if _BF16 is not None and dt == np.dtype(_BF16):
        return "f32"
    return {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64",
            np.dtype(np.float16): "f16"}[np.dtype(dt)]


def tma_swizzle_perm(box, eb: int, swizzle):
    """Element position of each box element in shared memory under a TMA
    swizzle (None without one): byte o goes to o ^ (((o >> 7) & m) << 4)."""
    span = _TMA_SWIZZLE[str(swizzle or "NONE")]
    if not span:
        return None
    m = span // 16 - 1
    o = np.arange(int(np.prod(box)), dtype=np.int64) * eb
    return (o ^ (((o >> 7) & m) << 4)) // eb


def _kind(dtype) -> str:
    k = dtype_info(dtype)[0]
    return "f32" if k == "bf16" else k


class Machine:
    """Runs one KernelSpec over numpy buffers (``interp.py:382-1017``)."""

    def __init__(self, spec: KernelSpec, inputs: dict[str, np.ndarray]):
        bx, by, bz = (int(v) for v in spec.block)
        if by != 1 or bz != 1:
            raise NotImplementedError("1-D blocks only")
        self.spec = spec
        self.T = bx
        self.nctas = int(np.prod(spec.grid))
        self.mem: dict[str, np.ndarray] = {}
        for name, arg in spec.args.items():
            if arg.scalar:
                continue
            dt = storage_dtype(arg.dtype)
            data = inputs.get(name)
            if data is None:
                data = np.zeros(arg.shape, dtype=dt)
            self.mem[name] = np.ascontiguousarray(np.asarray(data, dtype=dt))
        self.smem_decl: dict[str, tuple[tuple[int, ...], np.dtype]] = {}
        for st in ir.walk(spec.op.body):
            if isinstance(st, ir.Smem):
                self.smem_decl[st.name] = (tuple(int(e) for e in st.extents),
                                           storage_dtype(st.dtype))
        self.handlers = {
            ir.Tile: self.do_tile, ir.Load: self.do_load, ir.Assign: self.do_assign,
            ir.Accum: self.do_accum, ir.Let: self.do_let, ir.Write: self.do_write,
            ir.Loop: self.do_loop, ir.StridedLoop: self.do_strided, ir.Cond: self.do_cond,
            ir.Init: self.do_init, ir.Smem: self.do_nothing, ir.Sync: self.do_nothing,
            ir.WarpShuffle: self.do_shuffle, ir.TreeHalve: self.do_tree,
            ir.CpAsyncCopy: self.do_cp_async, ir.CpAsyncCommit: self.do_nothing,
            ir.CpAsyncWait: self.do_nothing, ir.Select: self.do_select,
            ir.ZeroPrologue: self.do_zero_prologue,
            ir.TmaDescriptor: self.do_nothing, ir.TmaLoad: self.do_tma_load,
            ir.MbarrierInit: self.do_mbarrier, ir.MbarrierArriveExpectTx: self.do_mbarrier,
            ir.MbarrierArrive: self.do_mbarrier, ir.MbarrierWait: self.do_mbarrier,
            ir.SetMaxNReg: self.do_nothing, ir.RegFragment: self.do_reg_fragment,
            ir.LdmatrixLoad: self.do_ldmatrix, ir.MmaSyncPtx: self.do_mma_sync,
            ir.RegStore: self.do_reg_store, ir.WgmmaDescriptor: self.do_wgmma_desc,
            ir.WgmmaMma: self.do_wgmma, ir.WgmmaFence: self.do_nothing,
            ir.WgmmaCommit: self.do_nothing, ir.WgmmaWait: self.do_wgmma_wait,
            ir.FragmentApply: self.do_frag_apply, ir.FragmentRowReduce: self.do_frag_rowreduce,
            ir.FragmentRepack: self.do_frag_repack, ir.Pre: self.do_pre, ir.Carry: self.do_carry,
            ir.FragmentPromote: self.do_frag_promote,
        }
        (self.carriers, self.carry_home, self.carry_inside,
         self.carry_top) = plan_carries(spec.op.body)
        self.wg_desc: dict[str, tuple] = {}
        self.frags: dict[str, np.ndarray] = {}
        self.frag_role: dict[str, tuple[str, str]] = {}
        self.frag_shape: dict[str, str] = {}
        self.tma_descs = {st.name: st for st in ir.walk(spec.op.body)
                          if isinstance(st, ir.TmaDescriptor)}

    # -- lane state -------------------------------------------------------

    # -- carried state (Pre / Carry) ---------------------------------------
    # Starred in the reference's table (``TASK.md:105-106``), absent from its
    # interpreter.  A carrier is a set of cells (literal indices) of one
    # dtype, seeded with one literal.  Its carrying loop is the innermost
    # loop that holds all its Carry statements: the cells are seeded when
    # that loop starts, a step's Pre reads see the state the previous step
    # left (the seed on the first step), a Carry sets a cell's next value
    # (active lanes only; cells not set keep theirs), and the next state
    # becomes the state at the end of each step.  Pre after the loop reads
    # the final state.  A carrier set outside every loop is updated at once.

    def _cell(self, index) -> tuple:
        idx = index if isinstance(index, tuple) else (() if index is None else (index,))
        out = []
        for e in idx:
            v = e.value if isinstance(e, ir.Literal) else e
            if not isinstance(v, int) or isinstance(v, bool):
                raise NotImplementedError("carried-state cells take literal indices")
            out.append(int(v))
        return tuple(out)

    def _carry_seed(self, c: str) -> Val:
        seed, dt = self.carriers[c]
        return coerce(Val("f32", np.float32(seed)) if _kind(dt) in ("f32", "f64", "f16") else
                      Val("s32", int(seed)), _kind(dt))

    def _carry_reset(self, c: str) -> None:
        seed = self._carry_seed(c)
        for state in (self.carry_cur, self.carry_nxt):
            cells = state.setdefault(c, {})
            for key in list(cells):
                cells[key] = Val(seed.kind, np.where(self.live(), seed.a, cells[key].a))

    def _carry_get(self, state, c: str, key: tuple) -> Val:
        cells = state.setdefault(c, {})
        if key not in cells:
            seed = self._carry_seed(c)
            cells[key] = Val(seed.kind, np.broadcast_to(seed.a, (self.n,)).copy())
        return cells[key]

    def do_pre(self, st: ir.Pre) -> None:
        if st.carrier not in self.carriers:
            raise KeyError(f"carrier {st.carrier!r} has no Carry")
        self.bind(st.name, self._carry_get(self.carry_cur, st.carrier, self._cell(st.index)))

    def do_carry(self, st: ir.Carry) -> None:
        key = self._cell(st.index)
        kind = _kind(self.carriers[st.name][1])
        v = coerce(self.env[st.value], kind)
        old = self._carry_get(self.carry_nxt, st.name, key)
        new = Val(kind, np.where(self.live(), np.broadcast_to(v.a, (self.n,)), old.a))
        self.carry_nxt[st.name][key] = new
        if st.name in self.carry_top:
            self._carry_get(self.carry_cur, st.name, key)
            self.carry_cur[st.name][key] = new

    def _start_chunk(self, first: int, count: int) -> None:
        self.first = first
        self.count = count
        self.n = count * self.T
        lane = np.arange(self.n, dtype=np.int64)
        self.tid = lane % self.T
        self.cta = first + lane // self.T
        self.local = self.cta - first          # CTA index inside the chunk
        self.mask: np.ndarray | None = None
        self.env: dict[str, Val] = {"lane": Val("s32", self.tid & 31),
                                    "warp": Val("s32", self.tid >> 5)}
        self.smem = {nm: np.zeros((count,) + shp, dtype=dt)
                     for nm, (shp, dt) in self.smem_decl.items()}
        self.carry_cur: dict[str, dict] = {}
        self.carry_nxt: dict[str, dict] = {}
        for name in self.spec.arg_order:
            arg = self.spec.args[name]
            if arg.scalar:
                v = arg.value if arg.value is not None else 0.0
                self.env[name] = Val(_kind(arg.dtype), v)

    def live(self) -> np.ndarray:
        return np.ones(self.n, dtype=bool) if self.mask is None else self.mask

    @contextmanager
    def under(self, cond):
        saved = self.mask
        if cond is not None:
            c = np.broadcast_to(cond, (self.n,)).astype(bool)
            self.mask = c if saved is None else (saved & c)
        try:
            yield
        finally:
            self.mask = saved

    def bind(self, name: str, v: Val) -> None:
        """Register write; lanes outside the mask keep their old value."""
        m = self.mask
        if m is not None and not m.all():
            old = self.env.get(name)
            base = 0 if old is None else coerce(old, v.kind).a
            v = Val(v.kind, np.where(m, v.a, base))
        self.env[name] = v

    # -- expressions ------------------------------------------------------

    def ev(self, e) -> Val:
        if isinstance(e, ir.Var):
            try:
                return self.env[e.name]
            except KeyError:
                raise KeyError(f"undefined name {e.name!r}") from None
        if isinstance(e, ir.Literal):
            if ir.is_int_literal(e):
                return Val("s32", int(e.value))
            return Val("f32", np.float32(e.value))
        if isinstance(e, ir.BinaryExpr):
            if e.op in ops.COMPARE:
                a, b = self.ev(e.left), self.ev(e.right)
                k = promote(a, b)
                fn = {"==": np.equal, "!=": np.not_equal, "<": np.less, "<=": np.less_equal,
                      ">": np.greater, ">=": np.greater_equal}[e.op]
                with np.errstate(invalid="ignore"):
                    return Val("pred", fn(coerce(a, k).a, coerce(b, k).a))
            if e.op in ops.LOGICAL:
                p, q = truthy(self.ev(e.left)), truthy(self.ev(e.right))
                return Val("pred", (p & q) if e.op == "&&" else (p | q))
            return apply_op(e.op, [self.ev(e.left), self.ev(e.right)])
        if isinstance(e, ir.TernaryExpr):
            c = truthy(self.ev(e.cond))
            a, b = self.ev(e.if_true), self.ev(e.if_false)
            k = promote(a, b)
            return Val(k, np.where(c, coerce(a, k).a, coerce(b, k).a))
        if isinstance(e, ir.FuncCallExpr):
            return apply_op(e.name, [self.ev(a) for a in e.args])
        if isinstance(e, ir.CastExpr):
            return coerce(self.ev(e.expr), _kind(e.dtype))
        if isinstance(e, ir.FlatIndex):
            return Val("s32", self.flat(e.index, self.shape_of(e.buffer)).astype(np.int32))
        if isinstance(e, ir.Builtin):
            return self.builtin(e.name)
        raise NotImplementedError(f"unsupported expression {type(e).__name__}")

    def builtin(self, name: str) -> Val:
        """GPU built-ins (``interp.py:520-552``)."""
        key = (name.replace("threadIdx", "thread_idx").replace("blockIdx", "block_idx")
               .replace("blockDim", "block_dim").replace("gridDim", "grid_dim"))
        g = self.spec.grid
        table = {
            "thread_idx.x": lambda: self.tid, "tid": lambda: self.tid,
            "block_idx.x": lambda: self.cta, "block_idx": lambda: self.cta,
            "cta": lambda: self.cta,
            "block_dim.x": lambda: self.T, "ntid": lambda: self.T,
            "lane": lambda: self.tid & 31, "lane_id": lambda: self.tid & 31,
            "warp": lambda: self.tid >> 5, "warp_id": lambda: self.tid >> 5,
            "warp_size": lambda: 32, "warpSize": lambda: 32,
            "thread_idx.y": lambda: 0, "thread_idx.z": lambda: 0,
            "block_idx.y": lambda: (self.cta // int(g[0])) % int(g[1]),
            "block_idx.z": lambda: self.cta // (int(g[0]) * int(g[1])),
            "block_dim.y": lambda: int(self.spec.block[1]),
            "block_dim.z": lambda: int(self.spec.block[2]),
            "grid_dim.x": lambda: int(g[0]), "grid_dim.y": lambda: int(g[1]),
            "grid_dim.z": lambda: int(g[2]),
        }
        if key not in table:
            raise NotImplementedError(f"unknown builtin {name!r}")
        return Val("s32", table[key]())

    def shape_of(self, name: str) -> tuple[int, ...]:
        if name in self.smem_decl:
            return self.smem_decl[name][0]
        if name in self.spec.args:
            return self.spec.args[name].shape
        raise KeyError(f"unknown buffer {name!r}")

    def flat(self, index, shape) -> np.ndarray:
        """Row-major offset; a short index addresses the trailing dims
        (``interp.py:559-576``)."""
        n = len(index)
        if n == 0:
            return np.zeros((), dtype=np.int64)
        dims = [1] * max(0, n - len(shape)) + [int(d) for d in shape]
        dims = dims[len(dims) - n:]
        total = np.zeros((), dtype=np.int64)
        stride = 1
        for idx, d in zip(reversed(index), reversed(dims)):
            total = total + as_int64(self.ev(idx)) * stride
            stride *= d
        return total

    def lane_flat(self, index, shape) -> np.ndarray:
        return np.broadcast_to(self.flat(index, shape), (self.n,))

    # -- statements -------------------------------------------------------

    def run_body(self, body) -> None:
        for st in body:
            h = self.handlers.get(type(st))
            if h is None:
                raise NotImplementedError(f"unsupported statement {type(st).__name__}")
            h(st)

    def do_nothing(self, st) -> None:
        return None

    def do_tile(self, st: ir.Tile) -> None:
        """``interp.py:634-663``: gid guard, clamped row-major axis decode."""
        ext = [int(a.extent.as_static()) for a in st.axes]
        total = int(np.prod(ext)) if ext else 1
        gid = self.cta * self.T + self.tid
        ok = gid < total
        safe = np.minimum(gid, total - 1) if total else gid
        saved = {a.name: self.env.get(a.name) for a in st.axes}
        stride = 1
        for axis, e in reversed(list(zip(st.axes, ext))):
            if e == 1:
                self.env[axis.name] = Val("s32", 0)
            elif stride == 1:
                self.env[axis.name] = Val("s32", safe % e)
            else:
                self.env[axis.name] = Val("s32", (safe // stride) % e)
            stride *= e
        with self.under(ok):
            self.run_body(st.body)
        for name, old in saved.items():
            if old is None:
                self.env.pop(name, None)
            else:
                self.env[name] = old

    def _read(self, buf: str, flat: np.ndarray, kind: str, swz="NONE") -> Val:
        """One element per lane from global or shared memory
        (``interp.py:665-689``); out-of-range active addresses raise."""
        m = self.live()
        if not m.all():
            flat = np.where(m, flat, 0)
        if buf in self.smem_decl:
            view = self.smem[buf].reshape(self.count, -1)
            flat = swizzle_index(flat, swz)
            if np.any((flat < 0) | (flat >= view.shape[1])):
                raise IndexError(f"shared load out of bounds in {buf!r}")
            raw = view[self.local, flat]
        else:
            arr = self.mem[buf].reshape(-1)
            if np.any((flat < 0) | (flat >= arr.size)):
                raise IndexError(f"global load out of bounds in {buf!r}")
            raw = arr[flat]
        if _BF16 is not None and raw.dtype == np.dtype(_BF16):
            raw = raw.astype(np.float32)
        skind = {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64",
                 np.dtype(np.float16): "f16", np.dtype(np.int32): "s32",
                 np.dtype(np.int64): "s64", np.dtype(np.bool_): "pred"}[raw.dtype]
        return coerce(Val(skind, raw), kind)

    def do_load(self, st: ir.Load) -> None:
        """``interp.py:691-704``: consecutive names read consecutive cells."""
        if st.dtype is not None:
            dt = st.dtype
        elif st.input in self.smem_decl:
            dt = self.smem_decl[st.input][1].name
        else:
            dt = self.spec.args[st.input].dtype
        kind = _kind(dt)
        flat = self.lane_flat(st.index, self.shape_of(st.input))
        m = self.live()
        if not m.all():
            flat = np.where(m, flat, 0)
        swz = getattr(st, "swizzle", "NONE")
        for k, name in enumerate(st.names):
            self.bind(name, self._read(st.input, flat + k, kind, swz))

    def do_assign(self, st: ir.Assign) -> None:
        r = apply_op(st.op.name, [self.env[a] for a in st.args])
        if st.dtype is not None:
            r = coerce(r, _kind(st.dtype))
        self.bind(st.name, r)

    def identity(self, op_or_value, kind: str) -> Val:
        """Accumulator seed (``interp.py:732-739``)."""
        if kind in ("s32", "s64"):
            v = int(ops.identity(op_or_value)) if isinstance(op_or_value, str) else int(op_or_value)
        elif isinstance(op_or_value, str):
            v = np.float32(ops.identity(op_or_value))
        else:
            v = np.float32(op_or_value)
        return Val(kind, v)

    def do_accum(self, st: ir.Accum) -> None:
        """``interp.py:712-721``: ``name = op(base or name, value)``; a missing
        or retyped accumulator restarts from the identity."""
        kind = _kind(st.dtype) if st.dtype is not None else "f32"
        acc = self.env.get(st.name)
        if acc is None or acc.kind != kind:
            acc = self.identity(st.op.name, kind)
        left = self.env[st.base] if st.base is not None else acc
        r = apply_op(st.op.name, [left, self.env[st.value]])
        if st.dtype is not None:
            r = coerce(r, kind)
        self.bind(st.name, r)

    def do_let(self, st: ir.Let) -> None:
        v = self.ev(st.value)
        if st.dtype is not None:
            v = coerce(v, _kind(st.dtype))
        self.bind(st.name, v)

    def do_init(self, st: ir.Init) -> None:
        self.bind(st.name, self.identity(st.identity, _kind(st.dtype)))

    def do_write(self, st: ir.Write) -> None:
        """``interp.py:741-778``: masked stores; ``atomic`` accumulates."""
        shared = st.output in self.smem_decl
        if shared:
            arr = self.smem[st.output]
        elif st.output in self.mem:
            arr = self.mem[st.output]
        else:
            raise KeyError(f"write to unknown buffer {st.output!r}")
        dt = arr.dtype
        is_bf16 = _BF16 is not None and dt == np.dtype(_BF16)
        kind = "f32" if is_bf16 else {np.dtype(np.float32): "f32", np.dtype(np.float64): "f64",
                                      np.dtype(np.float16): "f16", np.dtype(np.int32): "s32",
                                      np.dtype(np.int64): "s64",
                                      np.dtype(np.bool_): "pred"}[dt]
        base = self.lane_flat(st.index, self.shape_of(st.output))
        m = self.live()
        for k, name in enumerate(st.values):
            idx = base + k
            data = np.broadcast_to(coerce(self.env[name], kind).a, (self.n,))
            if shared:
                idx = swizzle_index(idx, getattr(st, "swizzle", "NONE"))
            ci = self.local
            if not m.all():
                idx, data, ci = idx[m], data[m], ci[m]
            if shared:
                view = arr.reshape(self.count, -1)
                if np.any((idx < 0) | (idx >= view.shape[1])):
                    raise IndexError(f"shared store out of bounds in {st.output!r}")
                view[ci, idx] = np.asarray(data).astype(dt)
            else:
                flat = arr.reshape(-1)
                if np.any((idx < 0) | (idx >= flat.size)):
                    raise IndexError(f"store out of bounds in {st.output!r}")
                if st.atomic:
                    np.add.at(flat, idx, np.asarray(data).astype(dt))
                else:
                    flat[idx] = np.asarray(data).astype(dt)

    def seed_accums(self, body, enabled: bool) -> None:
        """Reset the accumulators a loop owns (``interp.py:782-801``): every
        Accum in the body except those inside nested loops, which seed
        themselves."""
        seen: set[str] = set()

        def visit(stmts):
            for st in stmts:
                if isinstance(st, ir.Accum):
                    if st.name in seen:
                        continue
                    seen.add(st.name)
                    if enabled:
                        k = _kind(st.dtype) if st.dtype is not None else "f32"
                        self.env[st.name] = self.identity(st.op.name, k)
                elif isinstance(st, (ir.Loop, ir.StridedLoop)):
                    continue
                else:
                    for child in st.nested():
                        visit(child)

        visit(body)

    def _counted(self, axis: str, var: np.ndarray, bound: np.ndarray, step, body) -> None:
        saved = self.env.get(axis)
        steps = 0
        while True:
            alive = var < bound
            if self.mask is not None:
                alive = alive & self.mask
            if not np.any(alive):
                break
            self.env[axis] = Val("s32", var)
            with self.under(alive):
                self.run_body(body)
            for c in self.carry_inside.get(id(body), ()):
                self.carry_cur[c] = {key: v for key, v in self.carry_nxt.get(c, {}).items()}
            var = var + step
            steps += 1
            if steps > _STEP_LIMIT:
                raise RuntimeError(f"loop over {axis!r} did not terminate")
        if saved is None:
            self.env.pop(axis, None)
        else:
            self.env[axis] = saved

    def do_loop(self, st: ir.Loop) -> None:
        """``interp.py:803-826``: 0 .. extent-1."""
        self.seed_accums(st.body, bool(st.seed))
        for c in self.carry_home.get(id(st.body), ()):
            self._carry_reset(c)
        ext = int(st.axis.extent.as_static())
        self._counted(st.axis.name, np.zeros((), dtype=np.int64), np.int64(ext), 1, st.body)

    def do_strided(self, st: ir.StridedLoop) -> None:
        """``interp.py:828-856``: start, start+step, ... while < end (or extent)."""
        self.seed_accums(st.body, bool(st.seed))
        for c in self.carry_home.get(id(st.body), ()):
            self._carry_reset(c)
        ext = int(st.axis.extent.as_static())
        start = as_int64(self.ev(st.start))
        step = as_int64(self.ev(st.step)) if hasattr(st.step, "free_vars") else np.int64(int(st.step))
        bound = as_int64(self.ev(st.end)) if st.end is not None else np.int64(ext)
        self._counted(st.axis.name, start, bound, step, st.body)

    def do_cond(self, st: ir.Cond) -> None:
        c = truthy(self.ev(st.cond))
        with self.under(c):
            self.run_body(st.body)
        if st.else_body:
            with self.under(~c):
                self.run_body(st.else_body)

    def do_shuffle(self, st: ir.WarpShuffle) -> None:
        """XOR butterfly over ``length`` lanes (``interp.py:868-888``).  A
        partner that is inactive, or beyond the block, yields the caller's
        own value, as ``shfl.sync`` does."""
        m = self.live()
        off = int(st.length) // 2
        while off > 0:
            partner = self.tid ^ off
            src = np.clip(self.local * self.T + partner, 0, self.n - 1)
            ok = m[src] & (partner < self.T)
            for s, sb in zip(st.state, st.state_b):
                cur = self.env[s]
                got = np.broadcast_to(cur.a, (self.n,))[src]
                self.bind(sb, Val(cur.kind, np.where(ok, got, cur.a)))
            self.run_body(st.combine_states)
            off //= 2

    def do_tree(self, st: ir.TreeHalve) -> None:
        """Shared-memory halving tree, then broadcast of slot 0
        (``interp.py:890-926``)."""
        if st.inner is not None:
            raise NotImplementedError("TreeHalve(inner=...) is not supported")
        t = as_int64(self.env[st.tid_var])
        t = np.broadcast_to(t, (self.n,))
        m = self.live()
        kinds = {s: self.env[s].kind for s in st.state}
        bkind = {b: _kind(self.smem_decl[b][1].name) for b in st.bufs}
        views = {b: self.smem[b].reshape(self.count, -1) for b in st.bufs}
        half = int(st.length) // 2
        while half > 0:
            act = (t < half) & m
            for b, s, sb in zip(st.bufs, st.state, st.state_b):
                v = views[b]
                hi = v.shape[1] - 1
                self.bind(s, Val(bkind[b], v[self.local, np.clip(t, 0, hi)]))
                self.bind(sb, Val(bkind[b], v[self.local, np.clip(t + half, 0, hi)]))
            with self.under(act):
                self.run_body(st.combine_states)
            for b, s in zip(st.bufs, st.state):
                v = views[b]
                data = np.broadcast_to(coerce(self.env[s], bkind[b]).a, (self.n,))
                idx = np.clip(t, 0, v.shape[1] - 1)
                if act.any():
                    v[self.local[act], idx[act]] = data[act]
            half //= 2
        for b, s in zip(st.bufs, st.state):
            self.bind(s, coerce(Val(bkind[b], views[b][self.local, 0]), kinds[s]))

    def do_cp_async(self, st: ir.CpAsyncCopy) -> None:
        """Copies land immediately (``interp.py:930-958``)."""
        if st.smem not in self.smem:
            raise KeyError(f"cp.async destination {st.smem!r} is not a Smem buffer")
        view = self.smem[st.smem].reshape(self.count, -1)
        numel = view.shape[1]
        src = self.mem[st.src].reshape(-1)
        dshape = self.smem_decl[st.smem][0]
        dst = self.lane_flat(st.smem_index, dshape)
        if st.lane_index is not None:
            cols = int(dshape[-1]) if dshape else 1
            dst = dst + as_int64(self.ev(st.lane_index[0])) * cols + as_int64(
                self.ev(st.lane_index[1]))
        dst = swizzle_index(dst, st.swizzle)
        sidx = self.lane_flat(st.src_index, self.shape_of(st.src))
        m = self.live()
        ci = self.local
        if not m.all():
            dst, sidx, ci = dst[m], sidx[m], ci[m]
        count = int(st.nbytes) // src.dtype.itemsize
        offs = np.arange(count, dtype=np.int64)
        d = dst[:, None] + offs
        s = sidx[:, None] + offs
        if np.any(d >= numel) or np.any(s >= src.size):
            raise IndexError("cp.async out of bounds")
        view.reshape(-1)[ci[:, None] * numel + d] = src[s]

    def do_select(self, st: ir.Select) -> None:
        """``interp.py:960-972``: last branch is the default."""
        br = list(st.branches)
        kind = self.env[br[-1].value].kind
        for b in br[:-1]:
            k = self.env[b.value].kind
            if k in ("f32", "f64") or kind in ("f32", "f64"):
                kind = "f64" if "f64" in (k, kind) else "f32"
            else:
                kind = "s32"
        res = self.env[br[-1].value]
        for b in reversed(br[:-1]):
            c = truthy(self.ev(b.select))
            res = Val(kind, np.where(c, coerce(self.env[b.value], kind).a, coerce(res, kind).a))
        self.bind(st.name, res)

    # -- bulk-async transport and mbarriers --------------------------------
    # Starred in the reference's IR table (``TASK.md:121-127``) and absent
    # from its interpreter and emitter, so the meaning is defined here; the
    # CUDA lowering (``ptxgen/generic.py``) follows it.

    def do_mbarrier(self, st) -> None:
        """MbarrierInit / ArriveExpectTx / Arrive / Wait order copies and
        threads on the GPU; in the lockstep model every copy has landed when
        it is issued, so they change no value.  ``mbar`` must name a Smem
        array of 8-byte elements and ``slot`` (default 0) index into it."""
        decl = self.smem_decl.get(st.mbar)
        if decl is None or decl[1].itemsize != 8:
            raise KeyError(f"mbarrier {st.mbar!r} is not a Smem array of 8-byte elements")
        if st.slot is not None:
            slot = as_int64(self.ev(st.slot))
            m = self.live()
            if np.any(m & ((slot < 0) | (slot >= int(np.prod(decl[0])))))[()]:
                raise IndexError(f"mbarrier slot out of range in {st.mbar!r}")

    def do_tma_load(self, st: ir.TmaLoad) -> None:
        """One box of a buffer into shared memory, landing at once.

        The descriptor views its buffer row-major with ``src_shape`` (at most
        the buffer's element count); the box is ``box_extents`` elements
        from origin ``coords`` (both outermost first; the origin may be
        negative), and box elements outside ``src_shape`` read as zero.  The
        box lands row-major at element ``smem_index`` of the Smem buffer
        (a flat offset, or an index into its shape).  With swizzle B32, B64
        or B128 the box's inner extent is exactly 32, 64 or 128 bytes and
        byte ``o`` of the box lands at ``o ^ (((o >> 7) & m) << 4)``, m = 1,
        3 or 7 -- the TMA unit's pattern -- and the destination must sit on a
        1024-byte boundary (16 bytes without swizzle).  Each active lane
        issues the copy (IRs issue it from one thread).  Errors, raised here
        and reported as ``emmy_err`` 0x305 by the CUDA lowering: an inner
        coordinate not on a 16-byte boundary, a misaligned destination, a
        box that does not fit the Smem buffer."""
        d = self.tma_descs.get(st.desc)
        if d is None:
            raise KeyError(f"unknown TMA descriptor {st.desc!r}")
        shape = tuple(int(e) for e in d.src_shape)
        box = tuple(int(e) for e in d.box_extents)
        src = self.mem[d.src_buf].reshape(-1)
        eb = src.dtype.itemsize
        tma_check_descriptor(d, src.size, eb)
        if st.smem not in self.smem:
            raise KeyError(f"TMA destination {st.smem!r} is not a Smem buffer")
        view = self.smem[st.smem].reshape(self.count, -1)
        if view.dtype.itemsize != eb:
            raise ValueError("TMA source and destination element sizes differ")
        idx = st.smem_index if isinstance(st.smem_index, tuple) else (st.smem_index,)
        dshape = self.smem_decl[st.smem][0] if isinstance(st.smem_index, tuple) else (
            view.shape[1],)
        dst = self.lane_flat(idx, dshape)
        coords = [np.broadcast_to(as_int64(self.ev(c)), (self.n,)) for c in st.coords]
        if len(coords) != len(shape):
            raise ValueError("TMA coords and descriptor rank differ")
        whole = src[:int(np.prod(shape))].reshape(shape)
        perm = tma_swizzle_perm(box, eb, d.swizzle)
        align = 1024 if perm is not None else 16
        for ln in np.nonzero(self.live())[0]:
            c = [int(x[ln]) for x in coords]
            if (c[-1] * eb) % 16:
                raise ValueError("TMA inner coordinate not on a 16-byte boundary")
            d0 = int(dst[ln])
            if (d0 * eb) % align or d0 < 0 or d0 + int(np.prod(box)) > view.shape[1]:
                raise IndexError(f"TMA box does not fit {st.smem!r} at element {d0}")
            data = np.zeros(box, dtype=src.dtype)
            bsl, ssl = [], []
            for o, b, n in zip(c, box, shape):
                lo, hi = max(o, 0), min(o + b, n)
                if hi <= lo:
                    break
                bsl.append(slice(lo - o, hi - o))
                ssl.append(slice(lo, hi))
            else:
                data[tuple(bsl)] = whole[tuple(ssl)]
            flat = data.reshape(-1)
            pos = d0 + (perm if perm is not None else np.arange(flat.size))
            view[self.local[ln], pos] = flat

    # -- warp-level tensor-core fragments (mma.sync) ------------------------
    # Starred in the reference's IR table (``TASK.md:146-158``) with no
    # behaviour in its interpreter; defined here for the m16n8k16 atom with
    # 16-bit A/B (bf16 or f16) and an f32 C.  A fragment is a per-lane array
    # (``count`` cells of 8 A, 4 B or 4 C elements per lane) laid out as the
    # PTX ISA lays out the registers of ``mma.m16n8k16`` (``mma_layout``).
    # Loads and the product are warp-collective: they update every lane of
    # the warp whatever the lane mask; stores honour it.

    def _frag_ref(self, ref, index=None):
        name, _, rest = str(ref).partition("[")
        cell = int(rest.rstrip("]")) if rest else 0
        if index is not None:
            if rest:
                raise ValueError(f"fragment {ref!r} indexed twice")
            cell = int(as_int64(self.ev(index)).reshape(-1)[0]) if hasattr(
                index, "free_vars") else int(index)
        f = self.frags.get(name)
        if f is None:
            raise KeyError(f"undeclared fragment {name!r}")
        if not 0 <= cell < f.shape[0]:
            raise IndexError(f"fragment cell {cell} of {name!r}")
        return name, cell

    def _warps(self) -> int:
        if self.T % 32:
            raise ValueError("fragment operations need whole warps")
        return self.n // 32

    def do_reg_fragment(self, st: ir.RegFragment) -> None:
        role = str(st.role).lower()
        wg_n = wgmma_n(st.shape)
        if str(st.shape) != "m16n8k16" and not (role == "c" and wg_n):
            raise NotImplementedError(f"{role} fragment shape {st.shape!r}")
        dt = dtype_info(st.dtype)[0]
        if role in ("a", "b") and dt not in ("bf16", "f16"):
            raise NotImplementedError(f"{role} fragment of {st.dtype!r}")
        if role == "c" and dt != "f32" and not (dt == "f16" and not wg_n):
            raise NotImplementedError(f"c fragment of {st.dtype!r}")
        elems = {"a": 8, "b": 4, "c": wg_n // 2 if wg_n else 4}[role]
        self.frags[st.name] = np.zeros((int(st.count or 1), self.n, elems), np.float32)
        self.frag_role[st.name] = (role, dt)
        self.frag_shape[st.name] = str(st.shape)

    def do_ldmatrix(self, st: ir.LdmatrixLoad) -> None:
        """Fill one A or B cell from a 16-bit Smem buffer.  ``src_index`` =
        (row, col) of the cell's origin, the same on every lane of a warp;
        element (r, c) of the buffer is at r * ldm + c (``ldm`` defaults to
        the buffer's last extent), then the IR's shared-memory swizzle.  A
        (16 x 16, m by k) reads rows r0 + m, columns c0 + k; B (16 x 8, k by
        n) reads rows r0 + n, columns c0 + k, or with ``b_trans`` rows r0 + k,
        columns c0 + n."""
        for opt in ("staged", "gmem_guard", "k_zero", "pair_frag", "byte_slab",
                    "scale_buffer", "scale_index", "scale_ldm", "fragment_layout"):
            if getattr(st, opt) not in (None, False, "NONE"):
                raise NotImplementedError(f"LdmatrixLoad option {opt}")
        name, cell = self._frag_ref(st.frag, st.fragment_index)
        role, _ = self.frag_role[name]
        if role != str(st.role).lower() or role not in ("a", "b"):
            raise ValueError(f"LdmatrixLoad role {st.role!r} into {role} fragment {name!r}")
        if st.src_buffer not in self.smem or self.smem[st.src_buffer].dtype.itemsize != 2:
            raise ValueError("LdmatrixLoad reads a 16-bit Smem buffer")
        view = self.smem[st.src_buffer].reshape(self.count, -1)
        shape = self.smem_decl[st.src_buffer][0]
        ldm = int(st.ldm) if st.ldm is not None else int(shape[-1])
        w = self._warps()
        r0 = np.broadcast_to(as_int64(self.ev(st.src_index[0])), (self.n,)).reshape(w, 32)
        c0 = np.broadcast_to(as_int64(self.ev(st.src_index[1])), (self.n,)).reshape(w, 32)
        if np.any(r0 != r0[:, :1]) or np.any(c0 != c0[:, :1]):
            raise ValueError("LdmatrixLoad origin differs within a warp")
        rows, cols = mma_layout(role)               # [32, E]: (m, k) or (k, n)
        if role == "a":
            rr, cc = rows, cols
        elif st.b_trans:
            rr, cc = rows, cols                     # buffer [K][N]
        else:
            rr, cc = cols, rows                     # buffer [N][K]
        flat = (r0[:, :1, None] + rr[None]) * ldm + (c0[:, :1, None] + cc[None])
        flat = swizzle_index(flat, st.swizzle)
        if np.any((flat < 0) | (flat >= view.shape[1])):
            raise IndexError(f"LdmatrixLoad outside {st.src_buffer!r}")
        ci = self.local.reshape(w, 32)[:, :, None]
        vals = view[np.broadcast_to(ci, flat.shape), flat].astype(np.float32)
        self.frags[name][cell] = vals.reshape(self.n, -1)

    def do_mma_sync(self, st: ir.MmaSyncPtx) -> None:
        """c = a . b + c per warp on one m16n8k16 cell: the exact products
        summed with the accumulator and rounded once to f32 (the tensor core
        adds in an order and width of its own; the CUDA path is held to a
        bound, not to bits)."""
        if str(st.shape) != "m16n8k16" or st.b_row_major or st.sfa_frag or st.sfb_frag:
            raise NotImplementedError("MmaSyncPtx: m16n8k16, B column-major, no scales")
        w = self._warps()
        (an, ac), (bn, bc), (cn, cc) = (self._frag_ref(x) for x in
                                        (st.a_frag, st.b_frag, st.c_frag))
        ar, acl = mma_layout("a")
        br_, bcl = mma_layout("b")
        cr, ccl = mma_layout("c")
        A = np.zeros((w, 16, 16))
        B = np.zeros((w, 16, 8))
        Cm = np.zeros((w, 16, 8))
        af = self.frags[an][ac].reshape(w, 32, -1)
        bf = self.frags[bn][bc].reshape(w, 32, -1)
        cf = self.frags[cn][cc].reshape(w, 32, -1)
        A[:, ar, acl] = af
        B[:, br_, bcl] = bf
        Cm[:, cr, ccl] = cf
        D = (np.einsum("wmk,wkn->wmn", A, B) + Cm).astype(np.float32)
        if self.frag_role[cn][1] == "f16":
            # an f16 accumulator: A and B are f16 and each product's sum is
            # rounded once to f16
            if self.frag_role[an][1] != "f16" or self.frag_role[bn][1] != "f16":
                raise ValueError("an f16 accumulator takes f16 A and B")
            D = (np.einsum("wmk,wkn->wmn", A, B) + Cm).astype(np.float16).astype(np.float32)
        self.frags[cn][cc] = D[:, cr, ccl].reshape(self.n, -1)

    def _c_cell(self, ref, dtype="f32"):
        name, cell = self._frag_ref(ref)
        if (self.frag_role[name] != ("c", dtype) or self.frag_shape[name] != "m16n8k16"):
            raise ValueError(f"{ref!r} is not an m16n8 {dtype} c fragment")
        return name, cell

    def do_frag_promote(self, st: ir.FragmentPromote) -> None:
        """dst (f32) += src (f16), element by element with one f32 rounding,
        then src = 0; lanes outside the mask keep both."""
        dn, dc = self._c_cell(st.dst)
        sn, sc = self._c_cell(st.src, "f16")
        m = self.live()[:, None]
        d, s_ = self.frags[dn][dc], self.frags[sn][sc]
        self.frags[dn][dc] = np.where(m, (d + s_).astype(np.float32), d)
        self.frags[sn][sc] = np.where(m, np.float32(0), s_)

    def do_frag_apply(self, st: ir.FragmentApply) -> None:
        """out = op(out, *args) (``in_place``) or op(*args), element by
        element of an m16n8 c cell, with the IR's op semantics.  Argument
        kinds: "frag" (a c cell), "row" (a (top, bot) pair of per-lane names:
        top for the lane's row g elements, bot for row g + 8), "scalar" (a
        name or literal).  Lanes outside the mask keep their elements."""
        if st.layout is not None or st.post is not None:
            raise NotImplementedError("FragmentApply layout / post")
        name, cell = self._c_cell(st.out)
        args = list(st.args)
        kinds = list(st.kinds)
        if len(args) != len(kinds):
            raise ValueError("FragmentApply args and kinds differ in length")
        cur = self.frags[name][cell]
        cols = []
        if st.in_place:
            cols.append(lambda e: Val("f32", cur[:, e]))
        for a, kd in zip(args, kinds):
            if kd == "frag":
                an, ac = self._c_cell(a)
                src = self.frags[an][ac]
                cols.append(lambda e, src=src: Val("f32", src[:, e]))
            elif kd == "row":
                top, bot = (self.env[x] for x in a)
                cols.append(lambda e, top=top, bot=bot: bot if e >= 2 else top)
            elif kd == "scalar":
                v = self.env[a] if isinstance(a, str) else self.ev(a)
                cols.append(lambda e, v=v: v)
            else:
                raise NotImplementedError(f"FragmentApply argument kind {kd!r}")
        opname = getattr(st.op, "name", st.op)
        out = cur.copy()
        for e in range(4):
            r = coerce(apply_op(opname, [f(e) for f in cols]), "f32")
            out[:, e] = np.broadcast_to(r.a, (self.n,))
        m = self.live()
        self.frags[name][cell] = np.where(m[:, None], out, cur)

    def do_frag_rowreduce(self, st: ir.FragmentRowReduce) -> None:
        """top / bot = op over the lane's row-g / row-(g + 8) elements of the
        cells in ``frags`` (in order, two elements per cell), then over the
        four lanes of the row (exchanges with lane ^ 1, then lane ^ 2): every
        lane of the quad gets the same row value."""
        refs = [st.frags] if isinstance(st.frags, str) else list(st.frags)
        cells = [self.frags[n][c] for n, c in (self._c_cell(r) for r in refs)]
        opname = ops.canon(getattr(st.op, "name", st.op))
        if opname not in ("add", "maximum", "minimum"):
            raise NotImplementedError(f"FragmentRowReduce op {st.op!r}")
        self._warps()
        res = []
        for half in (0, 1):
            v = None
            for c in cells:
                for e in (2 * half, 2 * half + 1):
                    x = Val("f32", c[:, e])
                    v = x if v is None else coerce(apply_op(opname, [v, x]), "f32")
            for x in (1, 2):
                partner = np.arange(self.n) ^ x
                v = coerce(apply_op(opname, [v, Val("f32", v.a[partner])]), "f32")
            res.append(v)
        self.bind(st.top, res[0])
        self.bind(st.bot, res[1])

    def do_frag_repack(self, st: ir.FragmentRepack) -> None:
        """An A cell (m16 x k16) from two c cells (m16 x n8, keys 0-7 and
        8-15), each value rounded to the 16-bit type: in the PTX layouts the
        c cells' elements are exactly the A cell's, in order."""
        if st.fragment_layout is not None or st.part is not None:
            raise NotImplementedError("FragmentRepack layout / part")
        name, cell = self._frag_ref(st.frag)
        role, dt = self.frag_role[name]
        if role != "a" or dtype_info(st.ab_dtype)[0] != dt:
            raise ValueError("FragmentRepack fills an a fragment of its own type")
        if len(st.srcs) != 2:
            raise ValueError("FragmentRepack takes two c cells")
        vals = np.concatenate([self.frags[n][c] for n, c in (self._c_cell(r) for r in st.srcs)],
                              axis=1)
        self.frags[name][cell] = vals.astype(storage_dtype(dt)).astype(np.float32)

    # -- warpgroup products (wgmma) ------------------------------------------
    # Starred (``TASK.md:162-172``), no behaviour in the reference; defined
    # here for m64nNk16 with 16-bit A and B read from shared memory through
    # descriptors, both K-major (A [M][K], B [N][K]), and an f32 C fragment
    # per warpgroup (``wgmma_c_layout``).  A product lands at once; fence,
    # commit and wait order it on the GPU.  Warpgroup-collective: every lane
    # of the group takes part whatever the lane mask.

    def do_wgmma_desc(self, st: ir.WgmmaDescriptor) -> None:
        """Record a descriptor: the Smem buffer, the element where the
        operand starts (the same on every lane of a warpgroup), the layout
        (``swizzle`` NONE, B32, B64 or B128) and its byte strides."""
        if st.smem not in self.smem or self.smem[st.smem].dtype.itemsize != 2:
            raise ValueError("wgmma descriptors address a 16-bit Smem buffer")
        idx = st.smem_index if st.smem_index is not None else ir.Literal(0, None)
        idx = idx if isinstance(idx, tuple) else (idx,)
        shape = self.smem_decl[st.smem][0] if len(idx) > 1 else (self.smem[st.smem][0].size,)
        start = self.lane_flat(idx, shape)
        g = self._warpgroups()
        s2 = start.reshape(g, 128)
        if np.any(s2 != s2[:, :1]):
            raise ValueError("wgmma descriptor start differs within a warpgroup")
        self.wg_desc[st.name] = (st.smem, s2[:, 0].astype(np.int64), str(st.swizzle or "NONE"),
                                 int(st.lbo_bytes or 0), int(st.sbo_bytes or 0))

    def _warpgroups(self) -> int:
        if self.T % 128:
            raise ValueError("wgmma needs whole warpgroups (blocks of 128 threads)")
        return self.n // 128

    def _wgmma_operand(self, name: str, rows: int) -> np.ndarray:
        """[warpgroups, rows, 16] values of a K-major operand."""
        smem, start, swz, lbo, sbo = self.wg_desc[name]
        view = self.smem[smem].reshape(self.count, -1)
        r = np.arange(rows)[:, None]
        kk = np.arange(16)[None]
        b0 = start[:, None, None] * 2
        span = _TMA_SWIZZLE[swz]
        if not span:
            b = b0 + (r // 8) * sbo + (kk // 8) * lbo + (r % 8) * 16 + (kk % 8) * 2
        else:
            if np.any(b0 % span + 32 > span):
                raise ValueError("wgmma K slice crosses a swizzled row")
            b = b0 + (r // 8) * sbo + (r % 8) * span + kk * 2
            b = b ^ (((b >> 7) & (span // 16 - 1)) << 4)
        el = b // 2
        if np.any((el < 0) | (el >= view.shape[1])):
            raise IndexError(f"wgmma operand outside {smem!r}")
        cta = self.local.reshape(-1, 128)[:, 0]
        return view[cta[:, None, None], el].astype(np.float64)

    def do_wgmma(self, st: ir.WgmmaMma) -> None:
        """c = a . b (+ c when ``scale_d``) for each warpgroup: M = 64 rows of
        A and N rows of B (B [N][K]) over K = 16, exact products summed with
        the accumulator and rounded once to f32."""
        n = wgmma_n(st.shape)
        if not n or st.a_frag is not None or st.a_desc is None or st.trans_a or st.trans_b:
            raise NotImplementedError("WgmmaMma: m64nNk16, A and B K-major from descriptors")
        g = self._warpgroups()
        name, cell = self._frag_ref(st.c_frags)
        if wgmma_n(self.frag_shape[name]) != n:
            raise ValueError("WgmmaMma shape and its c fragment differ")
        A = self._wgmma_operand(st.a_desc, 64)
        B = self._wgmma_operand(st.b_desc, n)
        cr, ccl = wgmma_c_layout(n)
        cf = self.frags[name][cell].reshape(g, 128, -1)
        C = np.zeros((g, 64, n))
        C[:, cr, ccl] = cf
        sd = np.broadcast_to(truthy(self.ev(st.scale_d)) if hasattr(st.scale_d, "free_vars")
                             else bool(st.scale_d), (self.n,)).reshape(g, 128)
        if np.any(sd != sd[:, :1]):
            raise ValueError("wgmma scale_d differs within a warpgroup")
        D = np.einsum("gmk,gnk->gmn", A, B) + np.where(sd[:, :1, None], C, 0.0)
        self.frags[name][cell] = D.astype(np.float32)[:, cr, ccl].reshape(self.n, -1)

    def do_wgmma_wait(self, st: ir.WgmmaWait) -> None:
        if int(st.group or 0) != 0:
            raise NotImplementedError("WgmmaWait with groups left in flight")

    def do_reg_store(self, st: ir.RegStore) -> None:
        """Each active lane stores its C elements: element (m, n) of the cell
        to (r0 + m) * ldm + c0 + n of the buffer (``ldm`` defaults to its
        last extent), only where r0 + m < ``m_guard`` and c0 + n < ``n_guard``
        when given; ``atomic`` adds.  (r0, c0) = ``dst_index`` of the lane."""
        for opt in ("epilogue", "extra_frags", "fragment_layout", "volta_interleaved",
                    "row_dim", "col_dim"):
            if getattr(st, opt) not in (None, False, (), []):
                raise NotImplementedError(f"RegStore option {opt}")
        if str(st.swizzle or "NONE") != "NONE":
            raise NotImplementedError("RegStore swizzle")
        name, cell = self._frag_ref(st.frag, st.fragment_index)
        if self.frag_role[name][0] != "c":
            raise ValueError("RegStore stores a c fragment")
        arr = self.mem[st.dst_buffer]
        ldm = int(st.ldm) if st.ldm is not None else int(arr.shape[-1])
        r0 = np.broadcast_to(as_int64(self.ev(st.dst_index[0])), (self.n,))
        c0 = np.broadcast_to(as_int64(self.ev(st.dst_index[1])), (self.n,))
        wg_n = wgmma_n(self.frag_shape[name])
        if wg_n:
            cr, ccl = wgmma_c_layout(wg_n)
            lane = (self.tid & 127).astype(np.int64)
        else:
            cr, ccl = mma_layout("c")
            lane = (self.tid & 31).astype(np.int64)
        rows = r0[:, None] + cr[lane]
        cols = c0[:, None] + ccl[lane]
        ok = np.broadcast_to(self.live()[:, None], rows.shape).copy()
        for guard, idx in ((st.m_guard, rows), (st.n_guard, cols)):
            if guard is not None:
                lim = np.broadcast_to(as_int64(self.ev(guard)), (self.n,))
                ok &= idx < lim[:, None]
        flat = (rows * ldm + cols)[ok]
        vals = self.frags[name][cell][ok]
        out = arr.reshape(-1)
        if np.any((flat < 0) | (flat >= out.size)):
            raise IndexError(f"RegStore outside {st.dst_buffer!r}")
        data = coerce(Val("f32", vals.astype(np.float32)), _kind_np(out.dtype)).a
        if st.atomic:
            for f, v in zip(flat, data):            # lanes in order, one rounding each
                out[f] = (out[f] + v).astype(out.dtype)
        else:
            out[flat] = data

    def do_zero_prologue(self, st: ir.ZeroPrologue) -> None:
        """CTA 0 clears the first ``words`` 32-bit words (``interp.py:974-980``)."""
        if not np.any(self.cta == 0):
            return
        arr = self.mem[st.dst]
        nbytes = min(int(st.words) * 4, arr.nbytes)
        if nbytes > 0:
            arr.reshape(-1).view(np.uint8)[:nbytes] = 0

    # -- entry ------------------------------------------------------------

    def run(self, lane_budget: int = 1 << 20) -> dict[str, np.ndarray]:
        """Whole grid in chunks of CTAs (``interp.py:984-1017``)."""
        sm = 0
        for shp, dt in self.smem_decl.values():
            sm += int(np.prod(shp)) * np.dtype(dt).itemsize
        chunk = max(1, min(self.nctas, (256 << 20) // max(1, sm)))
        chunk = min(chunk, max(1, lane_budget // self.T))
        for first in range(0, self.nctas, chunk):
            self._start_chunk(first, min(chunk, self.nctas - first))
            self.run_body(self.spec.op.body)
        return {n: self.mem[n] for n, a in self.spec.args.items() if a.output}


def interpret(spec: KernelSpec, inputs: dict[str, np.ndarray]) -> dict[str, np.ndarray]:
    """Run ``spec`` on the CPU; returns the output buffers
    (``interp.py:1020-1021``)."""
    return Machine(spec, inputs).run()


def make_inputs(spec: KernelSpec, produced: dict | None = None) -> dict[str, np.ndarray]:
    """The runner's argument forms (``docs/API.md:40-50``,
    ``scripts/verify_semantics.py:33-56``): ``seed`` -> standard normal from
    ``default_rng(seed)``, ``data`` -> exact values, outputs zeroed,
    intermediates from earlier kernels, then ``zero_outputs`` cleared."""
    produced = produced or {}
    rngs: dict[int, np.random.Generator] = {}
    out: dict[str, np.ndarray] = {}
    for name in spec.arg_order:
        a = spec.args[name]
        if a.scalar:
            continue
        dt = storage_dtype(a.dtype)
        if a.intermediate:
            out[name] = np.asarray(produced[name]).astype(dt).reshape(a.shape)
        elif a.output:
            out[name] = np.zeros(a.shape, dtype=dt)
        elif a.data is not None:
            out[name] = np.asarray(a.data, dtype=np.float64).astype(dt).reshape(a.shape)
        else:
            seed = int(a.seed or 0)
            rng = rngs.setdefault(seed, np.random.default_rng(seed))
            out[name] = rng.standard_normal(a.shape).astype(dt)
    for name in spec.zero_outputs:
        if name in out:
            out[name][...] = 0
    return out
