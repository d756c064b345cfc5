"""HBM-bound kernel templates for sm_100a: pointwise, full reduction, rows.

Each template recognises one IR shape (``match_*``), then writes a kernel
whose memory schedule is B200-first while its arithmetic is the IR's own
statements, lowered op by op by ``ptxgen.lower``:

* pointwise: the Tile's per-element expression DAG over a flat grid-stride
  loop of 128-bit loads and stores, two vectors in flight per thread;
* full reduction: 128-bit grid-stride accumulation with the IR's Accum
  statements, the IR's WarpShuffle combine, a cross-warp combine through
  shared memory, then a grid-level pass -- per-CTA partials in a module
  scratch array and a last-CTA ticket (no waiting anywhere);
* rows (row reduce and fused rows): one CTA per row, the row's 128-bit
  chunks held in registers across both IR passes, so x is read from HBM
  once (RMSNorm, softmax and L2-norm are single-pass over HBM).

Every template is correct for any launch geometry (grid-stride loops and a
runtime block size), so the PTX also runs under meta.json's own launch; the
``@emmy-plan`` header gives the B200 launch the local launcher uses.
"""

from __future__ import annotations

import math

from . import ir
from .analysis import (NoMatch, flat_affine, int_literal, is_var, numel, scalar_stmt,
                       split_block_combine)
from .lower import Lowerer, LowerError, Val, storage_kind, value_kind
from .model import KernelSpec, dtype_info
from .ptx import Kernel, Module

MAX_PARTIALS = 4096   # grid-level reduction scratch: CTAs x states
ERR_TOO_MANY_CTAS = 0x101
ERR_PARTIAL_WARP = 0x102


def _require_whole_warps(k: Kernel, ntid: str, mod: "Module") -> None:
    """Full-mask warp shuffles need every lane present: refuse a block size
    that is not a multiple of 32 through the error word, without trapping."""
    mod.add_global(".visible .global .align 4 .u32 emmy_err;")
    p = k.reg("pred")
    r = k.reg("u32")
    k(f"and.b32 {r}, {ntid}, 31")
    k(f"setp.ne.u32 {p}, {r}, 0")
    ok = k.label("whole")
    k(f"@!{p} bra {ok}")
    k(f"st.global.u32 [emmy_err], {ERR_PARTIAL_WARP}")
    k("ret")
    k.place(ok)


def _params(spec: KernelSpec):
    out = []
    for n in spec.arg_order:
        a = spec.args[n]
        if a.scalar:
            raise NoMatch("scalar kernel parameters are not used by these templates")
        out.append((f"p_{n}", ".u64"))
    return out


def _ld_suffix(dtype) -> str:
    return {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64", "f16": "b16", "bf16": "b16",
            "pred": "u8"}[storage_kind(dtype)]


def _load_scalar(lo: Lowerer, addr: str, dtype, kind_out: str, nc: bool = True) -> Val:
    """One element of a global buffer at ``addr`` converted to ``kind_out``."""
    k = lo.k
    sk = storage_kind(dtype)
    pre = "ld.global.nc" if nc else "ld.global"
    if sk in ("f16", "bf16"):
        h = k.reg("b16")
        k(f"{pre}.b16 {h}, [{addr}]")
        r = k.reg("f32")
        k(f"cvt.f32.{sk} {r}, {h}")
        v = Val(r, "f32")
    elif sk == "pred":
        b = k.reg("s32")
        k(f"{pre}.u8 {b}, [{addr}]")
        p = k.reg("pred")
        k(f"setp.ne.s32 {p}, {b}, 0")
        v = Val(p, "pred")
    else:
        r = k.reg(sk)
        k(f"{pre}.{sk} {r}, [{addr}]")
        v = Val(r, sk)
    return lo.coerce(v, kind_out)


def _store_scalar(lo: Lowerer, addr: str, dtype, v: Val) -> None:
    k = lo.k
    sk = storage_kind(dtype)
    if sk in ("f16", "bf16"):
        f = lo.coerce(v, "f32")
        h = k.reg("b16")
        k(f"cvt.rn.{sk}.f32 {h}, {f.reg}")
        k(f"st.global.b16 [{addr}], {h}")
    elif sk == "pred":
        s = lo.coerce(v, "s32")
        k(f"st.global.u8 [{addr}], {s.reg}")
    else:
        s = lo.coerce(v, sk)
        k(f"st.global.{sk} [{addr}], {s.reg}")


def _vec_ok(spec: KernelSpec, bufs, n_elems: int) -> int:
    """Vector width for 128-bit access of ``bufs`` over ``n_elems`` elements."""
    sizes = {dtype_info(spec.args[b].dtype)[2] for b in bufs}
    if sizes != {4}:
        return 1
    return 4 if n_elems % 4 == 0 else 1


def grid_stride(k: Kernel, start: str, stride: str, count: int, process, unroll: int = 4):
    """``for i = start; i < count; i += stride`` with ``unroll`` indices
    handed to ``process`` at once while all are in range (so their loads are
    in flight together), then one at a time."""
    i = k.reg("u32")
    last = k.reg("u32")
    p = k.reg("pred")
    k(f"mov.u32 {i}, {start}")
    lu, l1, done = k.label("gsu"), k.label("gs1"), k.label("gsdone")
    if unroll > 1:
        k.place(lu)
        k(f"mad.lo.u32 {last}, {stride}, {unroll - 1}, {i}")
        k(f"setp.ge.u32 {p}, {last}, {count}")
        k(f"@{p} bra {l1}")
        idx = [i]
        for u in range(1, unroll):
            r = k.reg("u32")
            k(f"mad.lo.u32 {r}, {stride}, {u}, {i}")
            idx.append(r)
        process(idx)
        k(f"mad.lo.u32 {i}, {stride}, {unroll}, {i}")
        k(f"bra.uni {lu}")
    k.place(l1)
    k(f"setp.ge.u32 {p}, {i}, {count}")
    k(f"@{p} bra {done}")
    process([i])
    k(f"add.u32 {i}, {i}, {stride}")
    k(f"bra.uni {l1}")
    k.place(done)


def grid_blocked(k: Kernel, tid: str, ntid: str, cta: str, ncta: str, count: int, process,
                 unroll: int = 4):
    """Indices ``0 .. count-1`` in blocks of ``ntid * unroll`` contiguous
    indices, block b handled by CTA ``b % nctaid`` (a grid-stride loop over
    blocks): in one trip a thread takes ``b*ntid*unroll + u*ntid + tid`` for
    every u, so a CTA's loads in flight cover one contiguous block and the
    grid's cover consecutive blocks.  The partial last block goes one index
    at a time."""
    blk, bs, base, last, i = (k.reg("u32") for _ in range(5))
    p = k.reg("pred")
    k(f"mul.lo.u32 {bs}, {ntid}, {unroll}")
    k(f"mov.u32 {blk}, {cta}")
    lu, tail, tl, done = k.label("gbu"), k.label("gbt"), k.label("gbtl"), k.label("gbdone")
    k.place(lu)
    k(f"mad.lo.u32 {base}, {blk}, {bs}, {tid}")
    k(f"mad.lo.u32 {last}, {ntid}, {unroll - 1}, {base}")
    k(f"setp.ge.u32 {p}, {last}, {count}")
    k(f"@{p} bra {tail}")
    idx = [base]
    for u in range(1, unroll):
        r = k.reg("u32")
        k(f"mad.lo.u32 {r}, {ntid}, {u}, {base}")
        idx.append(r)
    process(idx)
    k(f"add.u32 {blk}, {blk}, {ncta}")
    k(f"bra.uni {lu}")
    k.place(tail)
    k(f"mov.u32 {i}, {base}")
    k.place(tl)
    k(f"setp.ge.u32 {p}, {i}, {count}")
    k(f"@{p} bra {done}")
    process([i])
    k(f"add.u32 {i}, {i}, {ntid}")
    k(f"bra.uni {tl}")
    k.place(done)


# ---------------------------------------------------------------------------
# pointwise
# ---------------------------------------------------------------------------


class PointwisePlan:
    def __init__(self):
        self.tile: ir.Tile | None = None
        self.unroll = 1
        self.n_elems = 0
        self.out = ""
        self.dag = None          # symbolic value of output element 0
        self.inputs: list[str] = []
        self.consts: list[str] = []


def _sym_exec(spec: KernelSpec, tile: ir.Tile):
    """Symbolically run a straight-line Tile body.  Returns
    (writes: {(buf, flat_offset_affine_const): sym}, stride per element)."""
    axes = [a.name for a in tile.axes]
    ext = [int(a.extent.as_static()) for a in tile.axes]
    tstride = {}
    s = 1
    for name, e in reversed(list(zip(axes, ext))):
        tstride[name] = s
        s *= e
    cells = s
    env: dict = {}
    writes: dict = {}
    unroll = None

    def elem_offset(index, buf):
        nonlocal unroll
        f = flat_affine(index, spec.args[buf].shape)
        if f is None:
            raise NoMatch("non-affine index")
        const = f.pop(1, 0)
        if not f:
            return ("const", const)
        u = None
        for name, c in f.items():
            if name not in tstride or c % tstride[name]:
                raise NoMatch("index not a multiple of the tile stride")
            q = c // tstride[name]
            if u is None:
                u = q
            elif q != u:
                raise NoMatch("index strides disagree")
        if set(f) != {n for n in axes if ext[axes.index(n)] > 1} and not (
                set(f) <= set(axes)):
            raise NoMatch("index misses tile axes")
        for n, e in zip(axes, ext):
            if e > 1 and n not in f:
                raise NoMatch("index ignores a tile axis")
        if unroll is None:
            unroll = u
        elif unroll != u:
            raise NoMatch("mixed unroll factors")
        return ("elem", const)

    for st in tile.body:
        if isinstance(st, ir.Load):
            if st.input not in spec.args:
                raise NoMatch("load from non-argument buffer")
            kind, off = elem_offset(st.index, st.input)
            dk = value_kind(st.dtype) if st.dtype is not None else value_kind(spec.args[st.input].dtype)
            for j, name in enumerate(st.names):
                if kind == "const":
                    if numel(spec.args[st.input].shape) <= off + j:
                        raise NoMatch("constant load out of range")
                    env[name] = ("cst", st.input, off + j, dk)
                else:
                    env[name] = ("ld", st.input, off + j, dk)
        elif isinstance(st, ir.Assign):
            for a in st.args:
                if a not in env:
                    raise NoMatch("undefined name")
            env[st.name] = ("op", st.op.name, st.dtype.name if st.dtype is not None else None,
                            tuple(env[a] for a in st.args))
        elif isinstance(st, ir.Let):
            v = st.value
            if isinstance(v, ir.Literal):
                env[st.name] = ("lit", v.value, ir.is_int_literal(v),
                                st.dtype.name if st.dtype is not None else None)
            elif isinstance(v, ir.Var) and v.name in env:
                env[st.name] = env[v.name]
            else:
                raise NoMatch("Let of a non-literal")
        elif isinstance(st, ir.Write):
            if st.atomic or st.output not in spec.args or not spec.args[st.output].output:
                raise NoMatch("write not a plain output store")
            kind, off = elem_offset(st.index, st.output)
            if kind != "elem":
                raise NoMatch("write to a fixed element")
            for j, name in enumerate(st.values):
                if name not in env:
                    raise NoMatch("undefined name")
                key = (st.output, off + j)
                if key in writes:
                    raise NoMatch("element written twice")
                writes[key] = env[name]
        else:
            raise NoMatch(f"{type(st).__name__} in a pointwise body")
    return writes, unroll or 1, cells


def _shift(sym, k):
    if sym[0] == "ld":
        return ("ld", sym[1], sym[2] - k, sym[3])
    if sym[0] == "op":
        return ("op", sym[1], sym[2], tuple(_shift(a, k) for a in sym[3]))
    return sym


def match_pointwise(spec: KernelSpec) -> PointwisePlan:
    body = spec.op.body
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        raise NoMatch("pointwise needs one Tile")
    tile = body[0]
    writes, unroll, cells = _sym_exec(spec, tile)
    outs = {b for b, _ in writes}
    if len(outs) != 1:
        raise NoMatch("pointwise writes one buffer")
    out = outs.pop()
    offs = sorted(o for _, o in writes)
    if offs != list(range(unroll)):
        raise NoMatch("writes do not cover the cell")
    n = cells * unroll
    if numel(spec.args[out].shape) != n:
        raise NoMatch("output size differs from the tile's element count")
    base = writes[(out, 0)]
    for kk in range(1, unroll):
        if _shift(writes[(out, kk)], kk) != base:
            raise NoMatch("unrolled slots compute different functions")
    plan = PointwisePlan()
    plan.tile, plan.unroll, plan.n_elems, plan.out, plan.dag = tile, unroll, n, out, base

    def visit(s):
        if s[0] == "ld":
            if s[2] != 0:
                raise NoMatch("element reads a neighbour")
            if numel(spec.args[s[1]].shape) != n:
                raise NoMatch("input size differs from output")
            if s[1] not in plan.inputs:
                plan.inputs.append(s[1])
        elif s[0] == "cst":
            if (s[1], s[2]) not in plan.consts:
                plan.consts.append((s[1], s[2]))
        elif s[0] == "op":
            for a in s[3]:
                visit(a)

    visit(base)
    return plan


def _eval_dag(lo: Lowerer, sym, leaf, memo: dict) -> Val:
    key = id(sym) if sym[0] == "op" else sym
    if key in memo:
        return memo[key]
    if sym[0] in ("ld", "cst"):
        v = leaf(sym)
    elif sym[0] == "lit":
        _, value, is_int, dt = sym
        v = lo.const(int(value), "s32") if is_int else lo.const(float(value), "f32")
        if dt is not None:
            v = lo.coerce(v, value_kind(dt))
    else:
        _, opname, dt, args = sym
        v = lo.apply(opname, [_eval_dag(lo, a, leaf, memo) for a in args])
        if dt is not None:
            v = lo.coerce(v, value_kind(dt))
            if storage_kind(dt) in ("f16", "bf16"):
                v = lo.coerce(v, storage_kind(dt))
    memo[key] = v
    return v


def emit_pointwise(spec: KernelSpec, plan: PointwisePlan) -> Module:
    k = Kernel(spec.entry, _params(spec))
    lo = Lowerer(k)
    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    cvals = {}
    for buf, off in plan.consts:
        a = k.reg("u64")
        k(f"add.u64 {a}, {base[buf]}, {off * dtype_info(spec.args[buf].dtype)[2]}")
        cvals[(buf, off)] = _load_scalar(lo, a, spec.args[buf].dtype,
                                          value_kind(spec.args[buf].dtype))
    n = plan.n_elems
    vec = _vec_ok(spec, plan.inputs + [plan.out], n)
    nvec = n // vec
    out_dt = spec.args[plan.out].dtype
    k.comment(f"pointwise: {n} elements, {vec}-wide, IR unroll {plan.unroll}")

    gid, stride = k.reg("u32"), k.reg("u32")
    tid, ntid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ntid.x", "%ctaid.x", "%nctaid.x"))
    k(f"mad.lo.u32 {gid}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {stride}, {ncta}, {ntid}")

    def process(idx_regs):
        """Load, compute and store the vectors at indices ``idx_regs``."""
        lanes = {}
        for j, idx in enumerate(idx_regs):
            for b in plan.inputs:
                ebytes = dtype_info(spec.args[b].dtype)[2]
                a = k.addr(base[b], idx, ebytes * vec)
                if vec == 4:
                    rs = k.regs("f32" if storage_kind(spec.args[b].dtype) == "f32" else "s32", 4)
                    t = "f32" if storage_kind(spec.args[b].dtype) == "f32" else "b32"
                    k(f"ld.global.nc.L1::no_allocate.v4.{t} {{{', '.join(rs)}}}, [{a}]")
                    for e in range(4):
                        lanes[(j, b, e)] = lo.coerce(Val(rs[e], storage_kind(spec.args[b].dtype)),
                                                     value_kind(spec.args[b].dtype))
                else:
                    lanes[(j, b, 0)] = _load_scalar(lo, a, spec.args[b].dtype,
                                                     value_kind(spec.args[b].dtype))
        for j, idx in enumerate(idx_regs):
            outs = []
            for e in range(vec):
                def leaf(s, j=j, e=e):
                    if s[0] == "cst":
                        return lo.coerce(cvals[(s[1], s[2])], s[3])
                    return lo.coerce(lanes[(j, s[1], e)], s[3])
                outs.append(_eval_dag(lo, plan.dag, leaf, {}))
            ebytes = dtype_info(out_dt)[2]
            a = k.addr(base[plan.out], idx, ebytes * vec)
            if vec == 4:
                sk = storage_kind(out_dt)
                vals = [lo.coerce(v, sk).reg for v in outs]
                t = "f32" if sk == "f32" else "b32"
                k(f"st.global.v4.{t} [{a}], {{{', '.join(vals)}}}")
            else:
                _store_scalar(lo, a, out_dt, outs[0])

    grid_stride(k, gid, stride, nvec, process, unroll=4)
    tail = n - nvec * vec
    if tail:
        raise NoMatch("tail of a vectorised pointwise")  # vec==4 implies n % 4 == 0
    m = Module(comment=f"emmy-b200 pointwise template for {spec.entry}")
    m.kernels.append(k)
    # one-shot grid: every thread takes exactly one batch of 4 vectors (the
    # unrolled body), no grid-stride tail -- measured faster on B200 than a
    # persistent grid (6.8 vs 6.1 TB/s for c=a+b over 2^28)
    m.plan = {"entry": spec.entry, "kind": "pointwise", "block": 256, "grid_per_sm": 0,
              "grid_max": max(1, math.ceil(nvec / (256 * 4))), "smem": 0}
    return m


# ---------------------------------------------------------------------------
# shared pieces of the reduction templates
# ---------------------------------------------------------------------------


class LoopBody:
    """A strided loop over one axis whose loads are classified for vector
    access: ``row`` (buffer [.., C] addressed by (row, axis)), ``elem`` (1-D
    buffer addressed by axis), ``col`` (buffer [C] addressed by axis in a row
    kernel) and ``const`` (1-element buffer)."""

    def __init__(self, loop: ir.StridedLoop):
        self.loop = loop
        self.axis = loop.axis.name
        self.extent = int(loop.axis.extent.as_static())
        self.loads: dict[int, tuple] = {}  # id(Load) -> (class, buffer, const offset)
        self.writes: dict[int, tuple] = {}


def _classify_loop(spec, lb: LoopBody, row_var: str | None, n_cols: int):
    for st in ir.walk(lb.loop.body):
        if isinstance(st, (ir.Loop, ir.StridedLoop, ir.Cond, ir.WarpShuffle, ir.TreeHalve,
                           ir.CpAsyncCopy, ir.Smem, ir.Sync, ir.Select)):
            raise NoMatch(f"{type(st).__name__} inside the reduction loop")
        if isinstance(st, ir.Load):
            if st.input not in spec.args:
                raise NoMatch("shared-memory load in loop")
            if len(st.names) != 1:
                raise NoMatch("grouped load in loop")
            shape = spec.args[st.input].shape
            f = flat_affine(st.index, shape)
            if f is None:
                raise NoMatch("non-affine load index")
            c = f.pop(1, 0)
            if not f and numel(shape) == 1 and c == 0:
                lb.loads[id(st)] = ("const", st.input, 0)
            elif f == {lb.axis: 1} and c == 0 and numel(shape) == n_cols and row_var is None:
                lb.loads[id(st)] = ("elem", st.input, 0)
            elif (row_var is not None and f == {row_var: n_cols, lb.axis: 1} and c == 0
                  and int(shape[-1]) == n_cols):
                lb.loads[id(st)] = ("row", st.input, 0)
            elif row_var is not None and f == {lb.axis: 1} and c == 0 and numel(shape) == n_cols:
                lb.loads[id(st)] = ("col", st.input, 0)
            else:
                raise NoMatch(f"load of {st.input} has an unsupported index")
        if isinstance(st, ir.Write):
            if st.atomic or st.output not in spec.args or len(st.values) != 1:
                raise NoMatch("unsupported write in loop")
            shape = spec.args[st.output].shape
            f = flat_affine(st.index, shape)
            if f is None or f.pop(1, 0) != 0:
                raise NoMatch("unsupported write index")
            if row_var is not None and f == {row_var: n_cols, lb.axis: 1} and int(shape[-1]) == n_cols:
                lb.writes[id(st)] = ("row", st.output)
            else:
                raise NoMatch("unsupported write index")
    if lb.extent != n_cols:
        raise NoMatch("loop extent differs from the row length")
    if lb.loop.end is not None:
        raise NoMatch("strided loop with an explicit end")


def _block_combine(lo: Lowerer, k: Kernel, ws: ir.WarpShuffle, slots: str, parity: str | None,
                   ident: list[Val]):
    """Every thread ends with the CTA-wide combined states.

    Warp butterfly with the IR's combine statements, lane 0 of each warp
    stores its states to shared ``slots`` (double-buffered by ``parity``), one
    barrier, then every warp loads all warps' slots (identity past the last
    warp) and repeats the butterfly, so no second barrier is needed."""
    states = list(ws.state)
    ns = len(states)
    lo.shuffle_combine(states, ws.state_b, ws.combine_states)
    lane, warp, ntid = k.sreg("%laneid"), k.reg("u32"), k.sreg("%ntid.x")
    tid = k.sreg("%tid.x")
    k(f"shr.u32 {warp}, {tid}, 5")
    base = k.reg("u32")
    k(f"mov.u32 {base}, {slots}")
    if parity is not None:
        off = k.reg("u32")
        k(f"mul.lo.u32 {off}, {parity}, {32 * ns * 4}")
        k(f"add.u32 {base}, {base}, {off}")
    p = k.reg("pred")
    a = k.reg("u32")
    k(f"setp.eq.u32 {p}, {lane}, 0")
    k(f"mad.lo.u32 {a}, {warp}, {ns * 4}, {base}")
    for j, s in enumerate(states):
        v = lo.env[s]
        k(f"@{p} st.shared.{'f32' if v.kind == 'f32' else 'b32'} [{a}+{j * 4}], {v.reg}")
    k("bar.sync 0")
    nw = k.reg("u32")
    k(f"add.u32 {nw}, {ntid}, 31")
    k(f"shr.u32 {nw}, {nw}, 5")
    k(f"setp.lt.u32 {p}, {lane}, {nw}")
    k(f"mad.lo.u32 {a}, {lane}, {ns * 4}, {base}")
    for j, s in enumerate(states):
        v = lo.env[s]
        r = k.reg(v.kind)
        k(f"mov.{'f32' if v.kind == 'f32' else 'b32'} {r}, {ident[j].reg}")
        k(f"@{p} ld.shared.{'f32' if v.kind == 'f32' else 'b32'} {r}, [{a}+{j * 4}]")
        lo.bind(s, Val(r, v.kind))
    lo.shuffle_combine(states, ws.state_b, ws.combine_states)


# ---- fused cross-GPU reduction ---------------------------------------------
# Inbox of one rank (``ptxgen.dist.PeerInbox``, one per kernel): partial
# states at (parity * XG_MAX_RANKS + rank) * 16 bytes, flags at XG_FLAGS +
# (parity * XG_MAX_RANKS + rank) * 4.  Parity is the launch epoch's low bit:
# a rank one launch ahead writes the other half, and cannot be two ahead,
# because finishing a launch needs every rank's flag of that launch.
XG_MAX_RANKS = 8
XG_MAX_STATES = 4
XG_FLAGS = 2 * XG_MAX_RANKS * 16
XG_WAIT_NS = 2_000_000_000
ERR_PEER_TIMEOUT = 0x203
# flags: "release" -- one st.release.sys per rank; "fence" -- one
# fence.acq_rel.sys after the partials, then relaxed system-scope flag stores
XG_PUBLISH = "release"
# polling: "acquire" -- ld.acquire.sys per poll; "relaxed" -- ld.relaxed.sys
# per poll and one fence.acq_rel.sys once every flag has been seen
XG_POLL = "acquire"


def _xgpu_globals(mod: Module) -> dict:
    mod.add_global(".visible .global .align 4 .u32 emmy_xworld;")
    mod.add_global(".visible .global .align 4 .u32 emmy_xrank;")
    mod.add_global(".visible .global .align 4 .u32 emmy_xepoch;")
    mod.add_global(f".visible .global .align 8 .u64 emmy_xpeer[{XG_MAX_RANKS}];")
    return {"world": "emmy_xworld", "rank": "emmy_xrank", "epoch": "emmy_xepoch",
            "peers": "emmy_xpeer", "max_ranks": XG_MAX_RANKS}


def _emit_xgpu_exchange(lo: Lowerer, k: Kernel, ws: ir.WarpShuffle, ident: list[Val],
                        slots: str, world: str | None = None) -> None:
    """With ``emmy_xworld`` > 1, warp 0 of the CTA holding this rank's total
    exchanges it with the other ranks, one lane per rank, all in parallel:
    lane i stores the total into rank i's inbox over NVLink and raises its
    flag there (release, system scope) with the launch epoch, then waits --
    bounded by %globaltimer -- for rank i's flag in its own inbox (acquire)
    and loads rank i's partial.  The warp then folds the ranks' partials in
    rank order with the IR's combine, passing them along with shuffles (the
    same result on every rank), and lane 0 shares it with the CTA through
    shared memory.  ``world``: a register that already holds
    ``emmy_xworld`` (loaded at the kernel's start, off the critical path).

    One lane per rank keeps the exchange's latency flat in the number of
    ranks: a single thread publishing and polling rank after rank paid one
    system-scope release per rank in series."""
    states = list(ws.state)
    kinds = [lo.env[s].kind for s in states]
    tt = ["f32" if kd == "f32" else "b32" for kd in kinds]
    tid = k.sreg("%tid.x")
    p, q = k.reg("pred"), k.reg("pred")
    done, bcast, join = k.label("xdone"), k.label("xbcast"), k.label("xjoin")
    if world is None:
        world = k.reg("u32")
        k(f"ld.global.u32 {world}, [emmy_xworld]")
    k(f"setp.le.u32 {p}, {world}, 1")
    k(f"@{p} bra {done}")
    k("bar.sync 0")                           # the CTA's combine reads of the slots are done
    k(f"setp.ge.u32 {q}, {tid}, 32")
    k(f"@{q} bra {bcast}")
    rank, ep, par, slot = (k.reg("u32") for _ in range(4))
    k(f"ld.global.u32 {rank}, [emmy_xrank]")
    k(f"ld.global.u32 {ep}, [emmy_xepoch]")
    k(f"add.u32 {ep}, {ep}, 1")
    k("bar.warp.sync -1")                     # every lane has read the old epoch
    k(f"setp.eq.u32 {p}, {tid}, 0")
    k(f"@{p} st.global.u32 [emmy_xepoch], {ep}")
    k(f"and.b32 {par}, {ep}, 1")
    k(f"mad.lo.u32 {slot}, {par}, {XG_MAX_RANKS}, {rank}")
    peers, own, pa, a = (k.reg("u64") for _ in range(4))
    k(f"mov.u64 {peers}, emmy_xpeer")
    k(f"mad.wide.u32 {own}, {rank}, 8, {peers}")
    k(f"ld.global.u64 {own}, [{own}]")
    vals = [k.reg(kd) for kd in kinds]
    k(f"setp.ge.u32 {p}, {tid}, {world}")
    k(f"@{p} bra {join}")
    # lane i: publish this rank's partial states, then the flag, to rank i
    k(f"mad.wide.u32 {pa}, {tid}, 8, {peers}")
    k(f"ld.global.u64 {pa}, [{pa}]")
    off = k.reg("u64")
    k(f"mul.wide.u32 {off}, {slot}, 16")
    k(f"add.u64 {a}, {pa}, {off}")
    for j, s in enumerate(states):
        k(f"st.global.{tt[j]} [{a}+{4 * j}], {lo.env[s].reg}")
    k(f"mul.wide.u32 {off}, {slot}, 4")
    k(f"add.u64 {a}, {pa}, {off}")
    if XG_PUBLISH == "fence":
        k("fence.acq_rel.sys")
        k(f"st.global.relaxed.sys.u32 [{a}+{XG_FLAGS}], {ep}")
    else:
        k(f"st.global.release.sys.u32 [{a}+{XG_FLAGS}], {ep}")
    # lane i: wait for rank i's flag of this epoch in the own inbox
    row, f = k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {row}, {par}, {XG_MAX_RANKS}, {tid}")
    fa = k.reg("u64")
    k(f"mad.wide.u32 {fa}, {row}, 4, {own}")
    t0, t1 = k.reg("u64"), k.reg("u64")
    k(f"mov.u64 {t0}, %globaltimer")
    spin, got, tout = k.label("xspin"), k.label("xgot"), k.label("xtout")
    k.place(spin)
    k(f"ld.global.{'relaxed' if XG_POLL == 'relaxed' else 'acquire'}.sys.u32 {f}, [{fa}+{XG_FLAGS}]")
    k(f"setp.eq.u32 {p}, {f}, {ep}")
    k(f"@{p} bra {got}")
    k(f"mov.u64 {t1}, %globaltimer")
    k(f"sub.u64 {t1}, {t1}, {t0}")
    k(f"setp.gt.u64 {p}, {t1}, {XG_WAIT_NS}")
    k(f"@{p} bra {tout}")
    k(f"bra.uni {spin}")
    k.place(tout)
    # a rank that timed out contributes whatever its slot holds; the error
    # word reports it
    k(f"st.global.u32 [emmy_err], {ERR_PEER_TIMEOUT}")
    k.place(got)
    if XG_POLL == "relaxed":
        k("fence.acq_rel.sys")               # the flag seen orders the partial's reads
    va = k.reg("u64")
    k(f"mad.wide.u32 {va}, {row}, 16, {own}")
    for j in range(len(states)):
        k(f"ld.global.relaxed.sys.{tt[j]} {vals[j]}, [{va}+{4 * j}]")
    k.place(join)
    k("bar.warp.sync -1")
    # fold the ranks' partials in rank order (every lane, the same bits)
    for j, s in enumerate(states):
        lo.bind(s, ident[j])
    i = k.reg("u32")
    fl, fend = k.label("xfold"), k.label("xfoldend")
    k(f"mov.u32 {i}, 0")
    k.place(fl)
    k(f"setp.ge.u32 {p}, {i}, {world}")
    k(f"@{p} bra {fend}")
    for j, (s, sb) in enumerate(zip(states, ws.state_b)):
        r = k.reg(kinds[j])
        k(f"shfl.sync.idx.b32 {r}, {vals[j]}, {i}, 31, -1")
        lo.bind(sb, Val(r, kinds[j]))
    lo.run(ws.combine_states)
    k(f"add.u32 {i}, {i}, 1")
    k(f"bra.uni {fl}")
    k.place(fend)
    k(f"setp.eq.u32 {p}, {tid}, 0")
    for j, s in enumerate(states):
        k(f"@{p} st.shared.{tt[j]} [{slots}+{4 * j}], {lo.env[s].reg}")
    k.place(bcast)
    k("bar.sync 0")
    for j, s in enumerate(states):
        r = k.reg(kinds[j])
        k(f"ld.shared.{tt[j]} {r}, [{slots}+{4 * j}]")
        lo.bind(s, Val(r, kinds[j]))
    k.place(done)


def _preload_consts(lo: Lowerer, spec, base, lbs) -> dict:
    """Load every 1-element buffer the loops read, once, before any branch,
    so the register holds the value on every path."""
    out = {}
    for lb in lbs:
        for cls, buf, _ in lb.loads.values():
            if cls == "const" and buf not in out:
                out[buf] = _load_scalar(lo, base[buf], spec.args[buf].dtype,
                                        value_kind(spec.args[buf].dtype))
    return out


def _state_identities(lo: Lowerer, loop_body, states) -> list[Val]:
    """Neutral element per combined state: the identity of the Accum that
    defines it in the reduction loop.  An accumulator stored as f16 or bf16
    is rounded after every step, so its per-thread partials depend on which
    elements each thread folds: such IR keeps its own thread mapping (the
    generic lowering) instead of a template's re-partitioned grid."""
    acc = {}
    for st in ir.walk(loop_body):
        if isinstance(st, ir.Accum):
            acc.setdefault(st.name, st)
    out = []
    for s in states:
        if s not in acc:
            raise NoMatch(f"combined state {s} has no Accum in the loop")
        st = acc[s]
        if st.dtype is not None and storage_kind(st.dtype) in ("f16", "bf16"):
            raise NoMatch(f"state {s} accumulates in {storage_kind(st.dtype)}")
        kind = value_kind(st.dtype) if st.dtype is not None else "f32"
        out.append(lo.identity(st.op.name, kind))
    return out


# ---------------------------------------------------------------------------
# full reduction
# ---------------------------------------------------------------------------


class FullReducePlan:
    pass


def match_full_reduce(spec: KernelSpec) -> FullReducePlan:
    body = spec.op.body
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        raise NoMatch("needs one Tile")
    tile = body[0]
    if len(tile.axes) != 1:
        raise NoMatch("full reduction tiles one cooperative axis")
    coop = tile.axes[0].name
    threads = int(tile.axes[0].extent.as_static())
    tb = tile.body
    i = 0
    pre = []
    while i < len(tb) and scalar_stmt(tb[i]) and not isinstance(tb[i], ir.Accum):
        pre.append(tb[i])
        i += 1
    if i >= len(tb) or not isinstance(tb[i], ir.StridedLoop):
        raise NoMatch("expected the strided reduction loop")
    loop = tb[i]
    if not is_var(loop.start, coop) or int_literal(loop.step) != threads:
        raise NoMatch("loop is not strided by the cooperative threads")
    lb = LoopBody(loop)
    n = lb.extent
    _classify_loop(spec, lb, None, n)
    if not any(c[0] == "elem" for c in lb.loads.values()):
        raise NoMatch("loop reads no array")
    ws, th, j = split_block_combine(tb, i + 1)
    post = list(tb[j:])
    for st in ir.walk(post):
        if isinstance(st, (ir.Loop, ir.StridedLoop, ir.WarpShuffle, ir.TreeHalve, ir.CpAsyncCopy,
                           ir.Sync)):
            raise NoMatch("unsupported statement after the reduction")
        if isinstance(st, ir.Load) and numel(spec.args.get(st.input).shape if st.input in spec.args
                                             else (2,)) != 1:
            raise NoMatch("epilogue load of an array")
        if isinstance(st, ir.Write) and (st.output not in spec.args or
                                         numel(spec.args[st.output].shape) != 1):
            raise NoMatch("epilogue write to an array")
    plan = FullReducePlan()
    plan.tile, plan.coop, plan.threads, plan.pre, plan.lb = tile, coop, threads, pre, lb
    plan.ws, plan.post, plan.n = ws, post, n
    return plan


def _const_load_hook(lo: Lowerer, spec, base):
    def hook(st: ir.Load):
        if st.input not in spec.args:
            raise LowerError("load of non-argument")
        f = flat_affine(st.index, spec.args[st.input].shape)
        if f is None:
            raise LowerError("non-affine scalar load")
        c = f.pop(1, 0)
        if f:
            raise LowerError("scalar load depends on an axis")
        dk = value_kind(st.dtype) if st.dtype is not None else value_kind(spec.args[st.input].dtype)
        eb = dtype_info(spec.args[st.input].dtype)[2]
        for j, name in enumerate(st.names):
            a = lo.k.reg("u64")
            lo.k(f"add.u64 {a}, {base[st.input]}, {(c + j) * eb}")
            lo.bind(name, _load_scalar(lo, a, spec.args[st.input].dtype, dk))
    return hook


def _scalar_write_hook(lo: Lowerer, spec, base, row_reg=None, row_stride=None):
    def hook(st: ir.Write):
        if st.atomic:
            raise LowerError("atomic epilogue write")
        shape = spec.args[st.output].shape
        f = flat_affine(st.index, shape)
        if f is None:
            raise LowerError("non-affine write")
        c = f.pop(1, 0)
        eb = dtype_info(spec.args[st.output].dtype)[2]
        a = lo.k.reg("u64")
        if f:
            if row_reg is None or set(f) != {row_reg[0]}:
                raise LowerError("write index depends on an unknown axis")
            lo.k(f"mad.wide.u32 {a}, {row_reg[1]}, {f[row_reg[0]] * eb}, {base[st.output]}")
            if c:
                lo.k(f"add.u64 {a}, {a}, {c * eb}")
        else:
            lo.k(f"add.u64 {a}, {base[st.output]}, {c * eb}")
        for j, name in enumerate(st.values):
            _store_scalar(lo, f"{a}+{j * eb}", spec.args[st.output].dtype, lo.env[name])
    return hook


# The full reduction's main loop: 16-byte loads in flight per thread, the
# layout of a CTA's loads, threads per CTA and CTAs per SM.  Measured on B200
# for 2^26 f32, back-to-back launches (mean of 100, three passes):
#   blocked, 4 loads, 512 x 3 CTAs per SM  41.9-42.4 us  (kept)
#   strided, 4 loads, 512 x 3              42.1-42.6
#   strided, 4 loads, 512 x 2              43.0-43.2
#   blocked, 8 loads, 512 x 2 / 256 x 4    42.8-43.1
#   strided, 4 loads, 512 x 4 / 256 x 8    43.2-44.6
# One contiguous range per CTA measured 45.3-51.4 us.  Dropping the fence
# before the last CTA's fold saved at most 0.1 us; it stays.
FULL_REDUCE_UNROLL = 4
# "strided": the loads in flight of one thread lie a grid width apart;
# "blocked": a CTA's loads in flight cover one contiguous block (grid_blocked)
FULL_REDUCE_LAYOUT = "blocked"
FULL_REDUCE_BLOCK, FULL_REDUCE_PER_SM = 512, 3
FULL_REDUCE_FENCE = True


def emit_full_reduce(spec: KernelSpec, plan: FullReducePlan) -> Module:
    k = Kernel(spec.entry, _params(spec))
    lo = Lowerer(k)
    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    lo.load_hook = _const_load_hook(lo, spec, base)
    lo.write_hook = _scalar_write_hook(lo, spec, base)
    lb, ws = plan.lb, plan.ws
    states = list(ws.state)
    ns = len(states)
    n = plan.n
    arrays = sorted({c[1] for c in lb.loads.values() if c[0] == "elem"})
    vec = _vec_ok(spec, arrays, n)
    nvec = n // vec
    sym = spec.entry
    mod = Module(comment=f"emmy-b200 full-reduction template for {spec.entry}")
    mod.add_global(".visible .global .align 4 .u32 emmy_err;")
    mod.add_global(".visible .global .align 4 .u32 emmy_ticket;")
    mod.add_global(f".visible .global .align 16 .b8 emmy_part[{MAX_PARTIALS * 4}];")
    k.shared(f"\t.shared .align 16 .b8 red_slots[{32 * ns * 4}];")
    k.shared("\t.shared .align 4 .u32 red_last;")
    k.comment(f"full reduction of {n} elements, {vec}-wide, {ns} state(s); scratch: emmy_part")

    tid, ntid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ntid.x", "%ctaid.x", "%nctaid.x"))
    _require_whole_warps(k, ntid, mod)
    # refuse launches whose partials do not fit the scratch array
    p = k.reg("pred")
    tot = k.reg("u32")
    k(f"mul.lo.u32 {tot}, {ncta}, {ns}")
    k(f"setp.gt.u32 {p}, {tot}, {MAX_PARTIALS}")
    ok = k.label("fits")
    k(f"@!{p} bra {ok}")
    k(f"st.global.u32 [emmy_err], {ERR_TOO_MANY_CTAS}")
    k("ret")
    k.place(ok)

    # a launch that overlaps its predecessor (emmy_launch_ex) may be
    # scheduled now: this grid only reads its inputs until the wait below
    k("griddepcontrol.launch_dependents")
    lo.run(plan.pre)
    lo.seed_accums(lb.loop.body, bool(lb.loop.seed))
    ident = _state_identities(lo, lb.loop.body, states)
    xg, xworld = None, None
    if ns <= XG_MAX_STATES:
        xg = _xgpu_globals(mod)
        xworld = k.reg("u32")
        k(f"ld.global.u32 {xworld}, [emmy_xworld]")   # in flight during the stream
    gid, stride = k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {gid}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {stride}, {ncta}, {ntid}")

    consts = _preload_consts(lo, spec, base, [lb])

    def run_elements(idx_regs):
        lanes = {}
        for j, idx in enumerate(idx_regs):
            for b in arrays:
                eb = dtype_info(spec.args[b].dtype)[2]
                a = k.addr(base[b], idx, eb * vec)
                if vec == 4:
                    rs = k.regs("f32" if storage_kind(spec.args[b].dtype) == "f32" else "s32", 4)
                    t = "f32" if storage_kind(spec.args[b].dtype) == "f32" else "b32"
                    k(f"ld.global.nc.L1::no_allocate.v4.{t} {{{', '.join(rs)}}}, [{a}]")
                    for e in range(4):
                        lanes[(j, b, e)] = Val(rs[e], storage_kind(spec.args[b].dtype))
                else:
                    lanes[(j, b, 0)] = _load_scalar(lo, a, spec.args[b].dtype,
                                                     storage_kind(spec.args[b].dtype))
        for j, idx in enumerate(idx_regs):
            for e in range(vec):
                def hook(st, j=j, e=e):
                    cls, buf, _ = lb.loads[id(st)]
                    dk = value_kind(st.dtype) if st.dtype is not None else value_kind(spec.args[buf].dtype)
                    if cls == "const":
                        lo.bind(st.names[0], lo.coerce(consts[buf], dk))
                    else:
                        lo.bind(st.names[0], lo.coerce(lanes[(j, buf, e)], dk))
                saved = lo.load_hook
                lo.load_hook = hook
                ax = k.reg("s32")
                k(f"mad.lo.u32 {ax}, {idx}, {vec}, {e}")
                lo.bind(lb.axis, Val(ax, "s32"))
                lo.run(lb.loop.body)
                lo.load_hook = saved

    if FULL_REDUCE_LAYOUT == "blocked":
        grid_blocked(k, tid, ntid, cta, ncta, nvec, run_elements, unroll=FULL_REDUCE_UNROLL)
    else:
        grid_stride(k, gid, stride, nvec, run_elements, unroll=FULL_REDUCE_UNROLL)

    _block_combine(lo, k, ws, "red_slots", None, ident)
    # before the first global write (partials, ticket, exchange, output):
    # when launched to overlap the previous kernel in the stream, that kernel
    # -- which may be this one, with the same scratch -- has completed and
    # its writes are visible (returns at once otherwise)
    k("griddepcontrol.wait")

    # ---- grid level: partials + last-CTA ticket -------------------------
    single = k.label("single")
    k(f"setp.eq.u32 {p}, {ncta}, 1")
    k(f"@{p} bra {single}")
    is0 = k.reg("pred")
    k(f"setp.eq.u32 {is0}, {tid}, 0")
    pa = k.reg("u64")
    k(f"mov.u64 {pa}, emmy_part")
    a = k.reg("u64")
    k(f"mul.wide.u32 {a}, {cta}, {ns * 4}")
    k(f"add.u64 {a}, {pa}, {a}")
    for j, s in enumerate(states):
        v = lo.env[s]
        k(f"@{is0} st.global.{'f32' if v.kind == 'f32' else 'b32'} [{a}+{j * 4}], {v.reg}")
    old = k.reg("u32")
    last = k.reg("u32")
    skip_t = k.label("noticket")
    k(f"@!{is0} bra {skip_t}")
    # release: thread 0's partial store above is ordered before the ticket
    k(f"atom.acq_rel.gpu.global.add.u32 {old}, [emmy_ticket], 1")
    nm1 = k.reg("u32")
    k(f"sub.u32 {nm1}, {ncta}, 1")
    pl = k.reg("pred")
    k(f"setp.eq.u32 {pl}, {old}, {nm1}")
    k(f"selp.u32 {last}, 1, 0, {pl}")
    k(f"st.shared.u32 [red_last], {last}")
    k(f"@{pl} st.global.u32 [emmy_ticket], 0")
    k.place(skip_t)
    k("bar.sync 0")
    k(f"ld.shared.u32 {last}, [red_last]")
    k(f"setp.eq.u32 {p}, {last}, 0")
    exit_l = k.label("notlast")
    k(f"@{p} bra {exit_l}")
    # thread 0's ticket acquired every CTA's partial; the barrier and this
    # fence carry that to the threads that read them
    if FULL_REDUCE_FENCE:
        k("fence.acq_rel.gpu")
    # the last CTA folds all partials with the IR's combine
    for j, s in enumerate(states):
        lo.bind(s, ident[j])
    jr = k.reg("u32")
    k(f"mov.u32 {jr}, {tid}")
    lp, lpe = k.label("part"), k.label("partend")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {jr}, {ncta}")
    k(f"@{p} bra {lpe}")
    k(f"mul.wide.u32 {a}, {jr}, {ns * 4}")
    k(f"add.u64 {a}, {pa}, {a}")
    for j, (s, sb) in enumerate(zip(states, ws.state_b)):
        v = lo.env[s]
        r = k.reg(v.kind)
        k(f"ld.global.cg.{'f32' if v.kind == 'f32' else 'b32'} {r}, [{a}+{j * 4}]")
        lo.bind(sb, Val(r, v.kind))
    lo.run(ws.combine_states)
    k(f"add.u32 {jr}, {jr}, {ntid}")
    k(f"bra.uni {lp}")
    k.place(lpe)
    k("bar.sync 0")  # red_slots are reused
    _block_combine(lo, k, ws, "red_slots", None, ident)
    k.place(single)
    if xworld is not None:
        _emit_xgpu_exchange(lo, k, ws, ident, "red_slots", world=xworld)
    # epilogue: the IR's statements after the tree, with the cooperative
    # index equal to the thread index (so "coop == 0" is one thread)
    co = k.reg("s32")
    k(f"mov.u32 {co}, {tid}")
    lo.bind(plan.coop, Val(co, "s32"))
    lo.run(plan.post)
    k.place(exit_l)
    mod.kernels.append(k)
    # launch shape: FULL_REDUCE_BLOCK threads x FULL_REDUCE_PER_SM CTAs per SM
    mod.plan = {"entry": spec.entry, "kind": "reduce_full", "block": FULL_REDUCE_BLOCK,
                "grid_per_sm": FULL_REDUCE_PER_SM,
                "grid_max": max(1, min(MAX_PARTIALS // ns, math.ceil(nvec / FULL_REDUCE_BLOCK))),
                "smem": 0,
                "scratch": {"emmy_part": MAX_PARTIALS * 4, "emmy_ticket": 4},
                # the kernel reads only its inputs before griddepcontrol.wait
                "overlap": True}
    if xg is not None:
        mod.plan["xgpu"] = xg
    return mod


# ---------------------------------------------------------------------------
# rows: row reduction and fused row kernels
# ---------------------------------------------------------------------------


class RowsPlan:
    pass


def match_rows(spec: KernelSpec) -> RowsPlan:
    body = spec.op.body
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        raise NoMatch("needs one Tile")
    tile = body[0]
    if len(tile.axes) != 2:
        raise NoMatch("rows tile (row, cooperative) axes")
    row, coop = tile.axes[0].name, tile.axes[1].name
    n_rows = int(tile.axes[0].extent.as_static())
    threads = int(tile.axes[1].extent.as_static())
    tb = tile.body
    i = 0
    pre = []
    while i < len(tb) and scalar_stmt(tb[i]) and not isinstance(tb[i], ir.Accum):
        pre.append(tb[i])
        i += 1
    if i >= len(tb) or not isinstance(tb[i], ir.StridedLoop):
        raise NoMatch("expected the row reduction loop")
    loop1 = tb[i]
    if not is_var(loop1.start, coop) or int_literal(loop1.step) != threads:
        raise NoMatch("loop is not strided by the cooperative threads")
    n_cols = int(loop1.axis.extent.as_static())
    lb1 = LoopBody(loop1)
    _classify_loop(spec, lb1, row, n_cols)
    ws, th, j = split_block_combine(tb, i + 1)
    mid = []
    while j < len(tb) and scalar_stmt(tb[j]) and not isinstance(tb[j], ir.Accum):
        mid.append(tb[j])
        j += 1
    tail = list(tb[j:])
    lb2 = None
    post = []
    if len(tail) == 1 and isinstance(tail[0], ir.StridedLoop):
        loop2 = tail[0]
        if not is_var(loop2.start, coop) or int_literal(loop2.step) != threads:
            raise NoMatch("second pass not strided by the cooperative threads")
        lb2 = LoopBody(loop2)
        _classify_loop(spec, lb2, row, n_cols)
        for st in ir.walk(loop2.body):
            if isinstance(st, ir.Accum):
                raise NoMatch("accumulation in the second pass")
    else:
        for st in ir.walk(tail):
            if isinstance(st, (ir.Loop, ir.StridedLoop, ir.WarpShuffle, ir.TreeHalve, ir.Sync,
                               ir.CpAsyncCopy)):
                raise NoMatch("unsupported row tail")
        post = tail
    for st in ir.walk(pre + mid):
        if isinstance(st, ir.Load) and (st.input not in spec.args or
                                        numel(spec.args[st.input].shape) != 1):
            raise NoMatch("row prologue loads an array")
    for b in {c[1] for c in lb1.loads.values() if c[0] == "row"}:
        if numel(spec.args[b].shape) != n_rows * n_cols:
            raise NoMatch("row buffer size mismatch")
    plan = RowsPlan()
    plan.tile, plan.row, plan.coop, plan.rows, plan.cols = tile, row, coop, n_rows, n_cols
    plan.threads, plan.pre, plan.lb1, plan.ws, plan.mid = threads, pre, lb1, ws, mid
    plan.lb2, plan.post = lb2, post
    return plan


def rows_block(n_cols: int, vec: int) -> int:
    """256 threads per row once a row has 512+ chunks (8 CTAs of 256 per SM
    measured faster than 4 of 512 for 4096-wide rows), fewer for short rows."""
    chunks = max(1, n_cols // vec)
    if chunks >= 512:
        return 256
    return 128 if chunks >= 128 else max(32, 32 * math.ceil(chunks / 32))


def emit_rows(spec: KernelSpec, plan: RowsPlan) -> Module:
    k = Kernel(spec.entry, _params(spec))
    lo = Lowerer(k)
    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    lo.load_hook = _const_load_hook(lo, spec, base)
    lb1, lb2, ws = plan.lb1, plan.lb2, plan.ws
    states = list(ws.state)
    ns = len(states)
    C, R = plan.cols, plan.rows
    row_bufs1 = sorted({c[1] for c in lb1.loads.values() if c[0] == "row"})
    row_bufs2 = sorted({c[1] for c in lb2.loads.values() if c[0] == "row"}) if lb2 else []
    col_bufs = sorted({c[1] for lb in (lb1, lb2) if lb for c in lb.loads.values()
                       if c[0] == "col"})
    out_bufs = sorted({w[1] for w in lb2.writes.values()}) if lb2 else []
    vec = _vec_ok(spec, row_bufs1 + row_bufs2 + col_bufs + out_bufs, C)
    nch = C // vec
    blk = rows_block(C, vec)
    cached = [b for b in row_bufs2 if b in row_bufs1]
    kmax = math.ceil(nch / blk) if (cached and math.ceil(nch / blk) <= 16) else 0
    batch = max(1, min(4, math.ceil(nch / blk)))
    k.comment(f"rows: {R} x {C}, {vec}-wide, {ns} state(s), register cache {kmax} chunk(s)")
    k.shared(f"\t.shared .align 16 .b8 row_slots[{2 * 32 * ns * 4}];")
    mod = Module(comment=f"emmy-b200 rows template for {spec.entry}")

    tid, ntid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ntid.x", "%ctaid.x", "%nctaid.x"))
    _require_whole_warps(k, ntid, mod)
    # a launch that overlaps its predecessor (emmy_launch_ex) may be
    # scheduled now: a row only reads until its combine is done
    k("griddepcontrol.launch_dependents")
    lo.run(plan.pre)
    consts = _preload_consts(lo, spec, base, [lb for lb in (lb1, lb2) if lb is not None])
    row = k.reg("u32")
    parity = k.reg("u32")
    k(f"mov.u32 {row}, {cta}")
    k(f"mov.u32 {parity}, 0")
    p = k.reg("pred")
    rloop, rend = k.label("row"), k.label("rowend")
    k.place(rloop)
    k(f"setp.ge.u32 {p}, {row}, {R}")
    k(f"@{p} bra {rend}")
    rowv = k.reg("s32")
    k(f"mov.u32 {rowv}, {row}")
    lo.bind(plan.row, Val(rowv, "s32"))
    co = k.reg("s32")
    k(f"mov.u32 {co}, {tid}")
    lo.bind(plan.coop, Val(co, "s32"))
    lo.write_hook = _scalar_write_hook(lo, spec, base, row_reg=(plan.row, row))
    # row base addresses
    rowaddr = {}
    for b in sorted(set(row_bufs1 + row_bufs2 + out_bufs)):
        eb = dtype_info(spec.args[b].dtype)[2]
        a = k.reg("u64")
        k(f"mad.wide.u32 {a}, {row}, {C * eb}, {base[b]}")
        rowaddr[b] = a
    for b in col_bufs:
        rowaddr[b] = base[b]
    lo.seed_accums(lb1.loop.body, bool(lb1.loop.seed))
    ident = _state_identities(lo, lb1.loop.body, states)

    def load_chunks(bufs, chunk_regs, tag):
        """Issue the vector loads of ``bufs`` for each chunk register."""
        got = {}
        for jj, c in enumerate(chunk_regs):
            for b in bufs:
                eb = dtype_info(spec.args[b].dtype)[2]
                a = k.addr(rowaddr[b], c, eb * vec)
                sk = storage_kind(spec.args[b].dtype)
                if vec == 4:
                    rs = k.regs("f32" if sk == "f32" else "s32", 4)
                    t = "f32" if sk == "f32" else "b32"
                    nc = ".nc" if spec.args[b].output is False else ""
                    k(f"ld.global{nc}.v4.{t} {{{', '.join(rs)}}}, [{a}]")
                    for e in range(4):
                        got[(jj, b, e)] = Val(rs[e], sk)
                else:
                    got[(jj, b, 0)] = _load_scalar(lo, a, spec.args[b].dtype, sk)
        return got

    def run_pass(lb, chunk_regs, got, stores):
        for jj, c in enumerate(chunk_regs):
            outs = {}
            for e in range(vec):
                def hook(st, jj=jj, e=e):
                    cls, buf, _ = lb.loads[id(st)]
                    dk = value_kind(st.dtype) if st.dtype is not None else value_kind(spec.args[buf].dtype)
                    if cls == "const":
                        lo.bind(st.names[0], lo.coerce(consts[buf], dk))
                    else:
                        lo.bind(st.names[0], lo.coerce(got[(jj, buf, e)], dk))

                def whook(st, e=e, outs=outs):
                    # snapshot: the name's register is reused by the next element
                    v = lo.env[st.values[0]]
                    r = k.reg(v.kind)
                    k(f"mov.{lo._mov_t(v.kind)} {r}, {v.reg}")
                    outs[(st.output, e)] = Val(r, v.kind)
                lo.load_hook, lo.write_hook = hook, whook
                ax = k.reg("s32")
                k(f"mad.lo.u32 {ax}, {c}, {vec}, {e}")
                lo.bind(lb.axis, Val(ax, "s32"))
                lo.run(lb.loop.body)
            for ob in sorted({o for o, _ in outs}):
                eb = dtype_info(spec.args[ob].dtype)[2]
                a = k.addr(rowaddr[ob], c, eb * vec)
                sk = storage_kind(spec.args[ob].dtype)
                if vec == 4:
                    vals = [lo.coerce(outs[(ob, e)], sk).reg for e in range(4)]
                    t = "f32" if sk == "f32" else "b32"
                    k(f"st.global.v4.{t} [{a}], {{{', '.join(vals)}}}")
                else:
                    _store_scalar(lo, a, spec.args[ob].dtype, outs[(ob, 0)])
        lo.load_hook = _const_load_hook(lo, spec, base)
        lo.write_hook = _scalar_write_hook(lo, spec, base, row_reg=(plan.row, row))

    def streamed(lb, bufs):
        """for c = tid; c < nch; c += ntid*batch: a batch of chunks per trip."""
        c0 = k.reg("u32")
        k(f"mov.u32 {c0}, {tid}")
        lp, lpe = k.label("chunks"), k.label("chunksend")
        one, onee = k.label("chunk1"), k.label("chunk1end")
        stepb = k.reg("u32")
        k(f"mul.lo.u32 {stepb}, {ntid}, {batch}")
        last = k.reg("u32")
        k.place(lp)
        # full batch only if its last chunk is in range
        k(f"mad.lo.u32 {last}, {ntid}, {batch - 1}, {c0}")
        k(f"setp.ge.u32 {p}, {last}, {nch}")
        k(f"@{p} bra {lpe}")
        regs = [c0]
        for b_ in range(1, batch):
            r = k.reg("u32")
            k(f"mad.lo.u32 {r}, {ntid}, {b_}, {c0}")
            regs.append(r)
        got = load_chunks(bufs, regs, "s")
        run_pass(lb, regs, got, True)
        k(f"add.u32 {c0}, {c0}, {stepb}")
        k(f"bra.uni {lp}")
        k.place(lpe)
        k.place(one)
        k(f"setp.ge.u32 {p}, {c0}, {nch}")
        k(f"@{p} bra {onee}")
        got = load_chunks(bufs, [c0], "s1")
        run_pass(lb, [c0], got, True)
        k(f"add.u32 {c0}, {c0}, {ntid}")
        k(f"bra.uni {one}")
        k.place(onee)

    use_cache = k.reg("pred")
    if kmax:
        capn = k.reg("u32")
        k(f"mul.lo.u32 {capn}, {ntid}, {kmax}")
        k(f"setp.ge.u32 {use_cache}, {capn}, {nch}")
    else:
        k(f"setp.ne.u32 {use_cache}, 0, 0")
    slow, join = k.label("uncached"), k.label("rowjoin")

    if kmax:
        k(f"@!{use_cache} bra {slow}")
        # ---- cached path: every chunk of this thread held in registers ----
        cregs, valid = [], []
        for jj in range(kmax):
            c = k.reg("u32")
            k(f"mad.lo.u32 {c}, {ntid}, {jj}, {tid}")
            pv = k.reg("pred")
            k(f"setp.lt.u32 {pv}, {c}, {nch}")
            cregs.append(c)
            valid.append(pv)
        cache = {}
        for jj in range(kmax):
            # clamp out-of-range chunks to chunk 0 so every load stays in bounds
            cc = k.reg("u32")
            k(f"selp.u32 {cc}, {cregs[jj]}, 0, {valid[jj]}")
            g = load_chunks(row_bufs1 + [b for b in col_bufs if b in
                                         {c[1] for c in lb1.loads.values()}], [cc], "c")
            for (x, b, e), v in g.items():
                cache[(jj, b, e)] = v
        for jj in range(kmax):
            sk = k.label("skipc")
            k(f"@!{valid[jj]} bra {sk}")
            run_pass(lb1, [cregs[jj]], {(0, b, e): cache[(jj, b, e)]
                                        for (x, b, e) in cache if x == jj}, False)
            k.place(sk)
        _block_combine(lo, k, ws, "row_slots", parity, ident)
        # before the row's first global write: an overlapped launch's
        # predecessor has completed (returns at once otherwise)
        k("griddepcontrol.wait")
        lo.run(plan.mid)
        if lb2 is not None:
            for jj in range(kmax):
                sk = k.label("skipc2")
                k(f"@!{valid[jj]} bra {sk}")
                extra = [b for b in row_bufs2 if b not in row_bufs1] + \
                        [b for b in col_bufs if b in {c[1] for c in lb2.loads.values()}
                         and b not in {c[1] for c in lb1.loads.values()}]
                g = load_chunks(extra, [cregs[jj]], "c2") if extra else {}
                got = {(0, b, e): cache[(jj, b, e)] for (x, b, e) in cache if x == jj}
                got.update(g)
                run_pass(lb2, [cregs[jj]], got, True)
                k.place(sk)
        else:
            lo.run(plan.post)
        k(f"bra.uni {join}")
        k.place(slow)
        # accumulators restart for the uncached path
        lo.seed_accums(lb1.loop.body, bool(lb1.loop.seed))
    # ---- streamed path: chunks in batches, second pass re-reads ----------
    l1_bufs = row_bufs1 + [b for b in col_bufs if b in {c[1] for c in lb1.loads.values()}]
    streamed(lb1, l1_bufs)
    _block_combine(lo, k, ws, "row_slots", parity, ident)
    k("griddepcontrol.wait")
    lo.run(plan.mid)
    if lb2 is not None:
        l2_bufs = row_bufs2 + [b for b in col_bufs if b in {c[1] for c in lb2.loads.values()}]
        streamed(lb2, l2_bufs)
    else:
        lo.run(plan.post)
    k.place(join)
    k(f"xor.b32 {parity}, {parity}, 1")
    k(f"add.u32 {row}, {row}, {ncta}")
    k(f"bra.uni {rloop}")
    k.place(rend)
    mod.kernels.append(k)
    mod.plan = {"entry": spec.entry, "kind": "rows", "block": blk, "grid_max": R,
                "grid_per_sm": 0, "smem": 0,
                # rows read only their inputs before griddepcontrol.wait
                "overlap": True}
    return mod
