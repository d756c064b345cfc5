"""Statement-by-statement sm_100a lowering of any Kernel IR.

The correctness floor behind the templates: any IR in the vocabulary of
``TASK.md:89-187`` that no template accepts is lowered statement by statement
under meta.json's launch, with the semantics of the golden model
(``ptxgen/interp.py``):

* ``Tile``: one cell per thread, ``gid = ctaid * ntid + tid``; lanes with
  ``gid >= N`` keep running on a clamped cell with every side effect masked
  off (``interp.py:634-663``), so block-wide barriers and shuffles always see
  the whole block;
* ``Cond`` narrows the mask instead of branching (``interp.py:858-864``);
  loads of masked-off lanes read element 0, register writes of masked-off
  lanes do not land (predicated moves), stores are predicated;
* ``Loop``/``StridedLoop`` seed their accumulators (``interp.py:782-856``);
  a loop whose trip count depends on the thread exits per thread (such a
  loop may not contain a barrier);
* ``WarpShuffle`` is an XOR butterfly over ``activemask`` in which an
  inactive partner yields the caller's own value (``interp.py:868-888``);
* ``TreeHalve`` is the shared-memory halving tree with a barrier per level
  and a broadcast of slot 0 (``interp.py:890-926``);
* ``cp.async`` copies land at once (``interp.py:930-958``): plain 4/8/16-byte
  loads and shared stores, the commit/wait statements are no-ops and the
  IR's own ``Sync`` orders them;
* shared-memory buffers are static, or one dynamic pool when meta.json
  gives a dynamic size, with the XOR swizzle of ``interp.py:578-586``;
* ``TmaLoad`` (with its ``TmaDescriptor``) is a real asynchronous copy by the
  bulk-copy (TMA) engine: one ``cp.async.bulk`` per box row, or per 16-byte
  chunk under a swizzle, each completing bytes on the IR's mbarrier; parts
  of the box outside the source are copied from a zeroed module buffer, so
  every byte arrives through the engine.  No host-built tensor map is
  needed, so the kernel runs under any launcher.  ``Mbarrier*`` lower to the
  ``mbarrier`` instructions, the wait bounded by ``%globaltimer`` (2 s,
  ``emmy_err`` 0x304); a malformed copy (misaligned inner coordinate or
  destination, box outside its Smem buffer) is skipped with ``emmy_err``
  0x305 and its bytes completed so no wait is left hanging.  ``SetMaxNReg``
  lowers to nothing: this lowering does not specialise warps, and the same
  budget change on every warp of the block can only lower the registers
  ptxas allotted or, as an increase, wait on registers nobody releases;
* ``RegFragment`` / ``LdmatrixLoad`` / ``MmaSyncPtx`` / ``RegStore`` (the
  m16n8k16 atom, bf16 or f16 A/B, f32 C) are per-thread registers,
  ``ldmatrix`` (``.trans`` for a [K][N] B), ``mma.sync`` and per-lane stores
  in the PTX fragment layout; loads and products update every lane of the
  warp whatever the mask, stores honour it; a fragment access outside its
  buffer is skipped with ``emmy_err`` 0x306;
* ``Wgmma*`` run on the 5th-generation tensor cores: each warpgroup's
  accumulator fragments live in its own TMEM columns while products are in
  flight (``tcgen05.st`` of the registers before the first product,
  ``tcgen05.ld`` back after ``WgmmaWait``, the ``16x256b`` shape whose
  per-thread layout is the warpgroup accumulator's); one thread of the
  group issues ``tcgen05.mma.cta_group::1.kind::f16`` (M = 64) from the
  descriptors' shared-memory operands, ``WgmmaCommit`` is a
  ``tcgen05.commit`` to a per-warpgroup mbarrier and ``WgmmaWait`` a
  bounded wait on it.  The CTA allocates its TMEM once at the start and
  frees it at the end.  An operand outside its buffer or misaligned skips
  the product with ``emmy_err`` 0x307.
"""

from __future__ import annotations

from . import ir, ops
from .analysis import NoMatch, numel
from .lower import Lowerer, LowerError, Val, storage_kind, value_kind
from .model import KernelSpec, dtype_info
from .ptx import Kernel, Module, f32_hex, f64_hex

_PTX_T = {"f32": "f32", "f64": "f64", "s32": "s32", "s64": "s64", "f16": "b16", "bf16": "b16",
          "pred": "u8"}
_SWZ = {"B128": (6, 0x7), "B64": (6, 0x3), "B32": (6, 0x1)}


def _collective(body) -> bool:
    return any(isinstance(s, (ir.Sync, ir.TreeHalve, ir.WarpShuffle)) for s in ir.walk(body))


ERR_OOB = 0x301          # checked mode: an index outside its buffer (access skipped)
ERR_MBAR_WAIT = 0x304    # an mbarrier wait ran past its limit
ERR_TMA = 0x305          # a TMA box copy that breaks its alignment or bounds (skipped)
ERR_FRAG = 0x306         # a fragment load or store outside its buffer (skipped)
ERR_WGMMA = 0x307        # a wgmma operand outside its buffer or misaligned (skipped)
ERR_SMEM = 0x308         # launched with less dynamic shared memory than the layout needs
_WG_LAYOUT = {"NONE": 0, "B32": 6, "B64": 4, "B128": 2}   # tcgen05 descriptor bits 61-63


def plan_carries(body):
    """(carrier -> (seed, dtype), id(loop body) -> carriers whose carrying
    loop it is, id(loop body) -> carriers with a Carry inside it, carriers
    set outside every loop): a carrier's carrying loop is the innermost loop
    holding all its Carry statements."""
    stacks: dict[str, list] = {}
    info: dict[str, tuple] = {}

    def walk(stmts, stack):
        for st in stmts:
            if isinstance(st, ir.Carry):
                stacks.setdefault(st.name, []).append(stack)
                seed = st.seed.value if isinstance(st.seed, ir.Literal) else st.seed
                got = (float(seed), st.dtype if st.dtype is not None else "f32")
                if info.setdefault(st.name, got) != got:
                    raise LowerError(f"carrier {st.name!r}: Carry seeds or dtypes differ")
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


def wgmma_n(shape) -> int:
    """N of an ``m64nNk16`` shape string (0 for any other)."""
    s = str(shape)
    if s.startswith("m64n") and s.endswith("k16") and s[4:-3].isdigit():
        n = int(s[4:-3])
        if n % 8 == 0 and 8 <= n <= 256:
            return n
    return 0
MBAR_WAIT_NS = 2_000_000_000
_TMA_SPAN = {"NONE": 0, "B32": 32, "B64": 64, "B128": 128}


def check_tma_descriptor(d: ir.TmaDescriptor, buf_numel: int, eb: int) -> None:
    """The limits of a box copy: rank 1..5, box extents 1..256, rows of the
    view and of the box whole multiples of 16 bytes, a view that stays in its
    buffer, and under a swizzle a box row exactly the swizzle span."""
    shape = tuple(int(e) for e in d.src_shape)
    box = tuple(int(e) for e in d.box_extents)
    span = _TMA_SPAN.get(str(d.swizzle or "NONE"))
    if span is None:
        raise LowerError(f"TMA swizzle {d.swizzle!r}")
    if not 1 <= len(shape) <= 5 or len(box) != len(shape):
        raise LowerError("TMA descriptor rank must be 1..5 with a box of the same rank")
    if min(shape) < 1 or numel(shape) > buf_numel:
        raise LowerError(f"TMA view {shape} exceeds buffer {d.src_buf!r}")
    if any(not 1 <= b <= 256 for b in box):
        raise LowerError("TMA box extents must be 1..256")
    if (shape[-1] * eb) % 16 or (box[-1] * eb) % 16:
        raise LowerError("TMA row and box row must be multiples of 16 bytes")
    if span and box[-1] * eb != span:
        raise LowerError(f"TMA swizzle {d.swizzle} needs a {span}-byte box row")


class Generic:
    def __init__(self, spec: KernelSpec, checked: bool = False):
        self.spec = spec
        self.checked = checked
        self.last_ok = None
        self.mod = Module(comment=f"emmy-b200 generic lowering for {spec.entry}"
                                  + (" (checked)" if checked else ""))
        self.mod.add_global(".visible .global .align 4 .u32 emmy_err;")
        if checked:
            # first violation: buffer id + 1 (see plan "oob_names") and its index
            self.mod.add_global(".visible .global .align 4 .u32 emmy_oob_buf;")
            self.mod.add_global(".visible .global .align 4 .s32 emmy_oob_index;")
        params = []
        for n in spec.arg_order:
            a = spec.args[n]
            if a.scalar:
                params.append((f"p_{n}", "." + {"f32": "f32", "f64": "f64", "s32": "s32",
                                                "s64": "s64"}[value_kind(a.dtype)]))
            else:
                params.append((f"p_{n}", ".u64"))
        self.k = Kernel(spec.entry, params)
        self.lo = Lowerer(self.k)
        self.lo.load_hook = self.do_load
        self.lo.write_hook = self.do_write
        self.lo.extra = {
            ir.Tile: self.do_tile, ir.Loop: self.do_loop, ir.StridedLoop: self.do_strided,
            ir.Cond: self.do_cond, ir.Sync: self.do_sync, ir.Smem: lambda st: None,
            ir.WarpShuffle: self.do_shuffle, ir.TreeHalve: self.do_tree,
            ir.CpAsyncCopy: self.do_cp_async, ir.CpAsyncCommit: lambda st: None,
            ir.CpAsyncWait: lambda st: None, ir.Select: self.do_select,
            ir.ZeroPrologue: self.do_zero_prologue,
            ir.TmaDescriptor: lambda st: None, ir.TmaLoad: self.do_tma_load,
            ir.MbarrierInit: self.do_mbar_init, ir.MbarrierArriveExpectTx: self.do_mbar_expect,
            ir.MbarrierArrive: self.do_mbar_arrive, ir.MbarrierWait: self.do_mbar_wait,
            ir.SetMaxNReg: lambda st: None, ir.RegFragment: self.do_reg_fragment,
            ir.LdmatrixLoad: self.do_ldmatrix, ir.MmaSyncPtx: self.do_mma_sync,
            ir.RegStore: self.do_reg_store, ir.WgmmaDescriptor: self.do_wgmma_desc,
            ir.WgmmaMma: self.do_wgmma, ir.WgmmaFence: lambda st: None,
            ir.WgmmaCommit: self.do_wgmma_commit, ir.WgmmaWait: self.do_wgmma_wait,
            ir.FragmentApply: self.do_frag_apply, ir.FragmentRowReduce: self.do_frag_rowreduce,
            ir.FragmentRepack: self.do_frag_repack, ir.Pre: self.do_pre, ir.Carry: self.do_carry,
            ir.FragmentPromote: self.do_frag_promote,
        }
        (self.carriers, self.carry_home, self.carry_inside,
         self.carry_top) = plan_carries(spec.op.body)
        self.carry_regs: dict[tuple, tuple] = {}     # (carrier, cell) -> (cur, nxt)
        self.frags: dict[str, tuple] = {}    # name -> (role, dtype, [[regs] per cell])
        self.wg = None                       # warpgroup tensor-core state (setup_wgmma)
        self.wgdesc: dict[str, tuple] = {}
        self.frag_shape: dict[str, str] = {}
        self.tma = {st.name: st for st in ir.walk(spec.op.body)
                    if isinstance(st, ir.TmaDescriptor)}
        for d in self.tma.values():
            if d.src_buf not in spec.args or spec.args[d.src_buf].scalar:
                raise LowerError(f"TMA descriptor {d.name!r}: no buffer {d.src_buf!r}")
            a = spec.args[d.src_buf]
            check_tma_descriptor(d, numel(a.shape), dtype_info(a.dtype)[2])
        if self.tma:
            row = max(int(d.box_extents[-1]) * dtype_info(spec.args[d.src_buf].dtype)[2]
                      for d in self.tma.values())
            # the source of every box byte outside its view: never written
            self.mod.add_global(f".visible .global .align 16 .b8 emmy_zeros[{row}];")
        self.smem: dict[str, tuple] = {}     # name -> (shape, dtype, offset)
        self.base: dict[str, str] = {}

    # -- set-up --------------------------------------------------------------

    def layout_smem(self) -> None:
        decls = [s for s in ir.walk(self.spec.op.body) if isinstance(s, ir.Smem)]
        off = 0
        for d in decls:
            if d.name in self.smem:
                continue
            eb = dtype_info(d.dtype)[2]
            al = max(int(d.align or 0), eb, 4)
            off = (off + al - 1) // al * al
            shape = tuple(int(e) for e in d.extents)
            self.smem[d.name] = (shape, d.dtype, off)
            off += numel(shape) * eb
        self.smem_bytes = off
        k = self.k
        if not self.smem:
            return
        al = 1024 if self.tma else 16
        if self.spec.smem_bytes > 0 or off > 48 * 1024:
            self.mod.add_global(f".extern .shared .align {al} .b8 emmy_dyn_smem[];")
            self.dyn = True
            # a launch with less dynamic shared memory than the layout uses
            # (meta.json's smem_bytes may be smaller) reports and returns at
            # once, before any shared access or barrier
            dsz, ok = k.reg("u32"), k.reg("pred")
            fine = k.label("smem_ok")
            k(f"mov.u32 {dsz}, %dynamic_smem_size")
            k(f"setp.ge.u32 {ok}, {dsz}, {off}")
            k(f"@{ok} bra {fine}")
            k(f"st.global.u32 [emmy_err], {ERR_SMEM}")
            k("ret")
            k.place(fine)
            r = k.reg("u32")
            k(f"mov.u32 {r}, emmy_dyn_smem")
        else:
            self.dyn = False
            k.shared(f"\t.shared .align {al} .b8 emmy_smem[{max(16, off)}];")
            r = k.reg("u32")
            k(f"mov.u32 {r}, emmy_smem")
        self.smem_base = r

    def emit(self) -> Module:
        k, lo, spec = self.k, self.lo, self.spec
        for n in spec.arg_order:
            a = spec.args[n]
            if a.scalar:
                kind = value_kind(a.dtype)
                r = k.reg(kind)
                k(f"ld.param.{_PTX_T[kind]} {r}, [p_{n}]")
                lo.bind(n, Val(r, kind))
            else:
                self.base[n] = k.param_ptr(f"p_{n}")
        self.layout_smem()
        tid = k.sreg("%tid.x")
        lane, warp = k.reg("s32"), k.reg("s32")
        k(f"and.b32 {lane}, {tid}, 31")
        k(f"shr.u32 {warp}, {tid}, 5")
        lo.bind("lane", Val(lane, "s32"))
        lo.bind("warp", Val(warp, "s32"))
        self.tid = tid
        # carried-state registers are seeded here (lines inserted at this
        # point as cells are first met)
        self.carry_at = len(k.lines)
        self.setup_wgmma()
        lo.run(spec.op.body)
        self.finish_wgmma()
        self.mod.kernels.append(k)
        self.mod.plan = {"entry": spec.entry, "kind": "generic", "block": int(spec.block[0]),
                         "grid_max": int(spec.grid[0] * spec.grid[1] * spec.grid[2]),
                         "grid_per_sm": 0,
                         "smem": int(max(spec.smem_bytes, self.smem_bytes)
                                     if self.smem and self.dyn else 0),
                         "geometry": "meta"}
        if self.checked:
            self.mod.plan["checked"] = True
            self.mod.plan["oob_names"] = self.buf_names()
        if tuple(spec.block[1:]) != (1, 1):
            raise NoMatch("1-D blocks only")
        return self.mod

    # -- masks -----------------------------------------------------------------

    def and_mask(self, p: str | None) -> str | None:
        cur = self.lo.mask
        if p is None:
            return cur
        if cur is None:
            return p
        r = self.k.reg("pred")
        self.k(f"and.pred {r}, {cur}, {p}")
        return r

    def guard(self) -> str:
        return f"@{self.lo.mask} " if self.lo.mask is not None else ""

    # -- addressing ------------------------------------------------------------

    def shape_of(self, name: str):
        if name in self.smem:
            return self.smem[name][0]
        return self.spec.args[name].shape

    def flat(self, index, shape) -> Val:
        """Row-major element offset as s32 (``interp.py:559-576``)."""
        lo, k = self.lo, self.k
        n = len(index)
        if n == 0:
            return lo.const(0, "s32")
        dims = [1] * max(0, n - len(shape)) + [int(d) for d in shape]
        dims = dims[len(dims) - n:]
        total = None
        stride = 1
        for e, d in zip(reversed(index), reversed(dims)):
            v = lo.coerce(lo.ev(e), "s32")
            if stride != 1:
                t = k.reg("s32")
                k(f"mul.lo.s32 {t}, {v.reg}, {stride}")
                v = Val(t, "s32")
            if total is None:
                total = v
            else:
                t = k.reg("s32")
                k(f"add.s32 {t}, {total.reg}, {v.reg}")
                total = Val(t, "s32")
            stride *= d
        return total

    def swizzle(self, idx: Val, mode) -> Val:
        base, _, sh = str(mode or "NONE").partition("@")
        if base not in _SWZ:
            return idx
        shift, msk = _SWZ[base]
        if sh:
            shift = int(sh)
        k = self.k
        t, r = k.reg("s32"), k.reg("s32")
        k(f"shr.s32 {t}, {idx.reg}, {shift}")
        k(f"and.b32 {t}, {t}, {msk}")
        k(f"shl.b32 {t}, {t}, 3")
        k(f"xor.b32 {r}, {idx.reg}, {t}")
        return Val(r, "s32")

    def clamp_masked(self, idx: Val) -> Val:
        """Masked-off lanes read element 0 (``interp.py:697-701``)."""
        if self.lo.mask is None:
            return idx
        r = self.k.reg("s32")
        self.k(f"selp.s32 {r}, {idx.reg}, 0, {self.lo.mask}")
        return Val(r, "s32")

    def buf_names(self) -> list[str]:
        """Buffer ids of checked mode: arguments in arg_order, then Smem."""
        return list(self.spec.arg_order) + list(self.smem)

    def bounds(self, name: str, idx: Val, j: int, count: int) -> tuple[Val, str]:
        """Checked mode: (index clamped to 0 when elements idx+j .. idx+j+count-1
        leave ``name``, in-range predicate).  An active lane out of range
        records the first violation and raises ``emmy_err`` to ERR_OOB; the
        access itself is then skipped by the caller."""
        k = self.k
        n = numel(self.shape_of(name))
        lim = n - j - count + 1
        if lim <= 0:
            raise LowerError(f"{name}: access of {count} element(s) at +{j} can never be "
                             f"inside its {n} elements")
        ok, viol = k.reg("pred"), k.reg("pred")
        k(f"setp.lt.u32 {ok}, {idx.reg}, {lim}")
        k(f"not.pred {viol}, {ok}")
        if self.lo.mask is not None:
            k(f"and.pred {viol}, {viol}, {self.lo.mask}")
        skip = k.label("inb")
        old, won = k.reg("u32"), k.reg("pred")
        k(f"@!{viol} bra {skip}")
        k(f"atom.global.cas.b32 {old}, [emmy_oob_buf], 0, {self.buf_names().index(name) + 1}")
        k(f"setp.eq.u32 {won}, {old}, 0")
        k(f"@{won} st.global.s32 [emmy_oob_index], {idx.reg}")
        k(f"atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_OOB}")
        k.place(skip)
        safe = k.reg("s32")
        k(f"selp.s32 {safe}, {idx.reg}, 0, {ok}")
        return Val(safe, "s32"), ok

    def addr(self, name: str, idx: Val, j: int = 0, count: int = 1) -> tuple[str, bool, object]:
        """(address register, shared?, dtype) of element idx+j of ``name``; in
        checked mode ``self.last_ok`` is the in-range predicate of elements
        idx+j .. idx+j+count-1 (else None)."""
        k = self.k
        self.last_ok = None
        if self.checked:
            idx, self.last_ok = self.bounds(name, idx, j, count)
        if name in self.smem:
            shape, dt, off = self.smem[name]
            eb = dtype_info(dt)[2]
            a = k.reg("u32")
            k(f"mad.lo.u32 {a}, {idx.reg}, {eb}, {self.smem_base}")
            if off + j * eb:
                k(f"add.u32 {a}, {a}, {off + j * eb}")
            return a, True, dt
        if name not in self.base:
            raise LowerError(f"unknown buffer {name!r}")
        dt = self.spec.args[name].dtype
        eb = dtype_info(dt)[2]
        a = k.reg("u64")
        k(f"mad.wide.s32 {a}, {idx.reg}, {eb}, {self.base[name]}")
        if j:
            k(f"add.u64 {a}, {a}, {j * eb}")
        return a, False, dt

    def load_elem(self, a: str, shared: bool, dt, kind: str) -> Val:
        k, lo = self.k, self.lo
        sk = storage_kind(dt)
        sp = "shared" if shared else "global"
        if sk in ("f16", "bf16"):
            h, r = k.reg("b16"), k.reg("f32")
            k(f"ld.{sp}.b16 {h}, [{a}]")
            k(f"cvt.f32.{sk} {r}, {h}")
            v = Val(r, "f32")
        elif sk == "pred":
            b, pr = k.reg("s32"), k.reg("pred")
            k(f"ld.{sp}.u8 {b}, [{a}]")
            k(f"setp.ne.s32 {pr}, {b}, 0")
            v = Val(pr, "pred")
        else:
            r = k.reg(sk)
            k(f"ld.{sp}.{_PTX_T[sk]} {r}, [{a}]")
            v = Val(r, sk)
        return lo.coerce(v, kind)

    def store_elem(self, a: str, shared: bool, dt, v: Val, atomic: bool = False,
                   ok: str | None = None) -> None:
        k, lo = self.k, self.lo
        sk = storage_kind(dt)
        sp = "shared" if shared else "global"
        p = self.and_mask(ok)
        g = f"@{p} " if p is not None else ""
        if atomic:
            if shared or sk not in ("f32", "s32"):
                raise LowerError("atomic add supports f32/s32 global buffers")
            s = lo.coerce(v, sk)
            k(f"{g}red.global.add.{sk} [{a}], {s.reg}")
            return
        if sk in ("f16", "bf16"):
            f = lo.coerce(v, "f32")
            h = k.reg("b16")
            k(f"cvt.rn.{sk}.f32 {h}, {f.reg}")
            k(f"{g}st.{sp}.b16 [{a}], {h}")
        elif sk == "pred":
            s = lo.coerce(v, "s32")
            k(f"{g}st.{sp}.u8 [{a}], {s.reg}")
        else:
            s = lo.coerce(v, sk)
            k(f"{g}st.{sp}.{_PTX_T[sk]} [{a}], {s.reg}")

    # -- statements ------------------------------------------------------------

    def do_tile(self, st: ir.Tile) -> None:
        k, lo = self.k, self.lo
        ext = [int(a.extent.as_static()) for a in st.axes]
        n = 1
        for e in ext:
            n *= e
        cta, ntid = k.sreg("%ctaid.x"), k.sreg("%ntid.x")
        gid, safe = k.reg("u32"), k.reg("u32")
        k(f"mad.lo.u32 {gid}, {cta}, {ntid}, {self.tid}")
        act = k.reg("pred")
        k(f"setp.lt.u32 {act}, {gid}, {n}")
        k(f"min.u32 {safe}, {gid}, {max(0, n - 1)}")
        stride = 1
        for axis, e in reversed(list(zip(st.axes, ext))):
            r = k.reg("s32")
            if e == 1:
                k(f"mov.u32 {r}, 0")
            elif stride == 1:
                k(f"rem.u32 {r}, {safe}, {e}")
            else:
                k(f"div.u32 {r}, {safe}, {stride}")
                k(f"rem.u32 {r}, {r}, {e}")
            lo.env[axis.name] = Val(r, "s32")
            stride *= e
        saved = lo.mask
        lo.mask = self.and_mask(act)
        lo.run(st.body)
        lo.mask = saved

    def do_load(self, st: ir.Load) -> None:
        lo = self.lo
        if st.dtype is not None:
            kind = value_kind(st.dtype)
        elif st.input in self.smem:
            kind = value_kind(self.smem[st.input][1])
        else:
            kind = value_kind(self.spec.args[st.input].dtype)
        idx = self.clamp_masked(self.flat(st.index, self.shape_of(st.input)))
        for j, name in enumerate(st.names):
            e = idx
            if j:
                t = self.k.reg("s32")
                self.k(f"add.s32 {t}, {idx.reg}, {j}")
                e = Val(t, "s32")
            if st.input in self.smem:
                e = self.swizzle(e, getattr(st, "swizzle", "NONE"))
            a, sh, dt = self.addr(st.input, e)
            ok = self.last_ok
            v = self.load_elem(a, sh, dt, kind)
            if ok is not None:                 # checked: out of range reads 0
                v = lo.select(Val(ok, "pred"), v, lo.const(0, v.kind))
            lo.bind(name, v)

    def do_write(self, st: ir.Write) -> None:
        idx = self.flat(st.index, self.shape_of(st.output))
        shared = st.output in self.smem
        for j, name in enumerate(st.values):
            e = idx
            if j:
                t = self.k.reg("s32")
                self.k(f"add.s32 {t}, {idx.reg}, {j}")
                e = Val(t, "s32")
            if shared:
                e = self.swizzle(e, getattr(st, "swizzle", "NONE"))
            a, sh, dt = self.addr(st.output, e)
            self.store_elem(a, sh, dt, self.lo.env[name], atomic=bool(st.atomic) and not sh,
                            ok=self.last_ok)

    def _loop(self, axis: str, start: Val, bound: Val, step: Val, body, seed: bool,
              uniform: bool) -> None:
        k, lo = self.k, self.lo
        lo.seed_accums(body, seed)
        var = k.reg("s32")
        k(f"mov.b32 {var}, {start.reg}")
        saved_env = lo.env.get(axis)
        head, done = k.label("lp"), k.label("lpend")
        # carried cells are seeded once as their carrying loop starts
        for c in self.carry_home.get(id(body), ()):
            self.carry_reset(c, body)
        k.place(head)
        p = k.reg("pred")
        k(f"setp.ge.s32 {p}, {var}, {bound.reg}")
        if uniform:
            k(f"@{p} bra.uni {done}")
        else:
            k(f"@{p} bra {done}")
            if lo.mask is not None:
                k(f"@!{lo.mask} bra {done}")
        lo.env[axis] = Val(var, "s32")
        before = self.wg_state()
        lo.run(body)
        if self.wg_state() != before:
            raise LowerError("wgmma products must be committed and waited for inside each "
                             "loop iteration")
        for c in sorted(self.carry_inside.get(id(body), ())):
            self.carry_commit(c)
        k(f"add.s32 {var}, {var}, {step.reg}")
        k(f"bra {head}")
        k.place(done)
        if saved_env is None:
            lo.env.pop(axis, None)
        else:
            lo.env[axis] = saved_env

    def _thread_free(self, e) -> bool:
        """Expression independent of the thread (literals only)."""
        return isinstance(e, ir.Literal) or (hasattr(e, "free_vars") and not e.free_vars)

    def do_loop(self, st: ir.Loop) -> None:
        lo = self.lo
        ext = int(st.axis.extent.as_static())
        self._loop(st.axis.name, lo.const(0, "s32"), lo.const(ext, "s32"), lo.const(1, "s32"),
                   st.body, bool(st.seed), uniform=True)

    def do_strided(self, st: ir.StridedLoop) -> None:
        lo = self.lo
        ext = int(st.axis.extent.as_static())
        start = lo.coerce(lo.ev(st.start), "s32")
        step = lo.coerce(lo.ev(st.step) if hasattr(st.step, "free_vars") else
                         lo.const(int(st.step), "s32"), "s32")
        bound = lo.coerce(lo.ev(st.end), "s32") if st.end is not None else lo.const(ext, "s32")
        uniform = self._thread_free(st.start) and self._thread_free(st.step) and (
            st.end is None or self._thread_free(st.end))
        if not uniform and _collective(st.body):
            raise LowerError("barrier inside a loop whose trip count depends on the thread")
        self._loop(st.axis.name, start, bound, step, st.body, bool(st.seed), uniform)

    def do_cond(self, st: ir.Cond) -> None:
        lo, k = self.lo, self.k
        c = lo.truthy(lo.ev(st.cond))
        saved = lo.mask
        lo.mask = self.and_mask(c.reg)
        lo.run(st.body)
        lo.mask = saved
        if st.else_body:
            n = k.reg("pred")
            k(f"not.pred {n}, {c.reg}")
            lo.mask = self.and_mask(n)
            lo.run(st.else_body)
            lo.mask = saved

    def do_sync(self, st: ir.Sync) -> None:
        if st.warp:
            self.k("bar.warp.sync -1")
        elif st.count is not None:
            self.k(f"barrier.sync {int(st.barrier_id or 0)}, {int(st.count)}")
        else:
            self.k(f"barrier.sync {int(st.barrier_id or 0)}")

    def do_shuffle(self, st: ir.WarpShuffle) -> None:
        k, lo = self.k, self.lo
        am = k.reg("u32")
        k(f"activemask.b32 {am}")
        lane = k.sreg("%laneid")
        off = int(st.length) // 2
        while off > 0:
            src, bit = k.reg("u32"), k.reg("u32")
            k(f"xor.b32 {src}, {lane}, {off}")
            k(f"shr.u32 {bit}, {am}, {src}")
            k(f"and.b32 {bit}, {bit}, 1")
            ok = k.reg("pred")
            k(f"setp.ne.u32 {ok}, {bit}, 0")
            for s, sb in zip(st.state, st.state_b):
                cur = lo.env[s]
                if cur.kind not in ("f32", "s32"):
                    raise LowerError("shuffle of a non-32-bit state")
                r, out = k.reg(cur.kind), k.reg(cur.kind)
                k(f"shfl.sync.bfly.b32 {r}, {cur.reg}, {off}, 31, {am}")
                k(f"selp.{'f32' if cur.kind == 'f32' else 'b32'} {out}, {r}, {cur.reg}, {ok}")
                lo.bind(sb, Val(out, cur.kind))
            lo.run(st.combine_states)
            off //= 2

    def do_tree(self, st: ir.TreeHalve) -> None:
        k, lo = self.k, self.lo
        if st.inner is not None:
            raise LowerError("TreeHalve(inner=...)")
        t = lo.coerce(lo.env[st.tid_var], "s32")
        kinds = {s: lo.env[s].kind for s in st.state}
        length = int(st.length)
        half = length // 2
        bar = f"barrier.sync {int(st.barrier_id or 0)}"
        if st.barrier_count is not None:
            bar += f", {int(st.barrier_count)}"
        while half > 0:
            k(bar)
            inner = k.reg("pred")
            k(f"setp.lt.s32 {inner}, {t.reg}, {half}")
            for b, s, sb in zip(st.bufs, st.state, st.state_b):
                size = numel(self.smem[b][0])
                i0, i1 = k.reg("s32"), k.reg("s32")
                k(f"min.s32 {i0}, {t.reg}, {size - 1}")
                k(f"max.s32 {i0}, {i0}, 0")
                k(f"add.s32 {i1}, {t.reg}, {half}")
                k(f"min.s32 {i1}, {i1}, {size - 1}")
                k(f"max.s32 {i1}, {i1}, 0")
                bk = value_kind(self.smem[b][1])
                a0, sh, dt = self.addr(b, Val(i0, "s32"))
                a1, _, _ = self.addr(b, Val(i1, "s32"))
                lo.bind(s, self.load_elem(a0, True, dt, bk))
                lo.bind(sb, self.load_elem(a1, True, dt, bk))
            k(bar)
            saved = lo.mask
            lo.mask = self.and_mask(inner)
            lo.run(st.combine_states)
            for b, s in zip(st.bufs, st.state):
                size = numel(self.smem[b][0])
                i0 = k.reg("s32")
                k(f"min.s32 {i0}, {t.reg}, {size - 1}")
                k(f"max.s32 {i0}, {i0}, 0")
                a0, _, dt = self.addr(b, Val(i0, "s32"))
                self.store_elem(a0, True, dt, lo.env[s])
            lo.mask = saved
            half //= 2
        k(bar)
        for b, s in zip(st.bufs, st.state):
            z = lo.const(0, "s32")
            a0, _, dt = self.addr(b, z)
            lo.bind(s, lo.coerce(self.load_elem(a0, True, dt, value_kind(dt)), kinds[s]))

    def do_cp_async(self, st: ir.CpAsyncCopy) -> None:
        k, lo = self.k, self.lo
        if st.smem not in self.smem:
            raise LowerError(f"cp.async into non-Smem {st.smem!r}")
        shape = self.smem[st.smem][0]
        dst = self.flat(st.smem_index, shape)
        if st.lane_index is not None:
            cols = int(shape[-1]) if shape else 1
            ln = lo.coerce(lo.ev(st.lane_index[0]), "s32")
            cl = lo.coerce(lo.ev(st.lane_index[1]), "s32")
            t = k.reg("s32")
            k(f"mad.lo.s32 {t}, {ln.reg}, {cols}, {dst.reg}")
            k(f"add.s32 {t}, {t}, {cl.reg}")
            dst = Val(t, "s32")
        dst = self.swizzle(dst, st.swizzle)
        src = self.clamp_masked(self.flat(st.src_index, self.shape_of(st.src)))
        nb = int(st.nbytes)
        eb = dtype_info(self.spec.args[st.src].dtype)[2]
        src_elems = max(1, nb // eb)
        dst_elems = max(1, nb // dtype_info(self.smem[st.smem][1])[2])
        sa, _, _ = self.addr(st.src, src, count=src_elems)
        ok_s = self.last_ok
        da, _, _ = self.addr(st.smem, dst, count=dst_elems)
        ok_d = self.last_ok
        p = self.lo.mask
        for extra in (ok_s, ok_d):
            if extra is not None:
                q = k.reg("pred")
                k(f"and.pred {q}, {p}, {extra}") if p is not None else k(f"mov.pred {q}, {extra}")
                p = q
        g = f"@{p} " if p is not None else ""
        words = nb // 4
        regs = k.regs("b32", words)
        if words == 4:
            k(f"ld.global.v4.b32 {{{', '.join(regs)}}}, [{sa}]")
            k(f"{g}st.shared.v4.b32 [{da}], {{{', '.join(regs)}}}")
        elif words == 2:
            k(f"ld.global.v2.b32 {{{', '.join(regs)}}}, [{sa}]")
            k(f"{g}st.shared.v2.b32 [{da}], {{{', '.join(regs)}}}")
        elif words == 1:
            k(f"ld.global.b32 {regs[0]}, [{sa}]")
            k(f"{g}st.shared.b32 [{da}], {regs[0]}")
        else:
            raise LowerError(f"cp.async of {nb} bytes")

    def do_select(self, st: ir.Select) -> None:
        lo = self.lo
        br = list(st.branches)
        kind = lo.env[br[-1].value].kind
        for b in br[:-1]:
            kk = lo.env[b.value].kind
            kind = ("f64" if "f64" in (kk, kind) else "f32") if ("f32" in (kk, kind) or
                                                                  "f64" in (kk, kind)) else "s32"
        res = lo.coerce(lo.env[br[-1].value], kind)
        for b in reversed(br[:-1]):
            c = lo.truthy(lo.ev(b.select))
            res = lo.select(c, lo.coerce(lo.env[b.value], kind), res)
        lo.bind(st.name, res)

    def do_zero_prologue(self, st: ir.ZeroPrologue) -> None:
        k = self.k
        a = self.spec.args[st.dst]
        words = min(int(st.words), (a.nbytes + 3) // 4)
        cta, ntid = k.sreg("%ctaid.x"), k.sreg("%ntid.x")
        p = k.reg("pred")
        skip = k.label("nozp")
        k(f"setp.ne.u32 {p}, {cta}, 0")
        k(f"@{p} bra {skip}")
        i = k.reg("u32")
        k(f"mov.u32 {i}, {self.tid}")
        lp = k.label("zp")
        k.place(lp)
        k(f"setp.ge.u32 {p}, {i}, {words}")
        k(f"@{p} bra {skip}")
        ad = k.addr(self.base[st.dst], i, 4)
        k(f"st.global.u32 [{ad}], 0")
        k(f"add.u32 {i}, {i}, {ntid}")
        k(f"bra {lp}")
        k.place(skip)
        k("barrier.sync 0")


    # -- bulk-async transport and mbarriers ----------------------------------

    def mbar_addr(self, name: str, slot) -> str:
        k = self.k
        if name not in self.smem or dtype_info(self.smem[name][1])[2] != 8:
            raise LowerError(f"mbarrier {name!r} is not a Smem array of 8-byte elements")
        a = k.reg("u32")
        k(f"add.u32 {a}, {self.smem_base}, {self.smem[name][2]}")
        if slot is not None:
            sl = self.lo.coerce(self.lo.ev(slot), "s32")
            k(f"mad.lo.u32 {a}, {sl.reg}, 8, {a}")
        return a

    def do_mbar_init(self, st: ir.MbarrierInit) -> None:
        k = self.k
        a = self.mbar_addr(st.mbar, st.slot)
        n = self.lo.coerce(self.lo.ev(st.count) if hasattr(st.count, "free_vars")
                           else self.lo.const(int(st.count), "s32"), "s32")
        k(f"{self.guard()}mbarrier.init.shared::cta.b64 [{a}], {n.reg}")
        # the initialised barrier is visible to the copy engine's completions
        k("fence.mbarrier_init.release.cluster")

    def do_mbar_expect(self, st: ir.MbarrierArriveExpectTx) -> None:
        k = self.k
        a = self.mbar_addr(st.mbar, st.slot)
        n = self.lo.coerce(self.lo.ev(st.bytes_) if hasattr(st.bytes_, "free_vars")
                           else self.lo.const(int(st.bytes_), "s32"), "s32")
        k(f"{self.guard()}mbarrier.arrive.expect_tx.shared::cta.b64 _, [{a}], {n.reg}")

    def do_mbar_arrive(self, st: ir.MbarrierArrive) -> None:
        a = self.mbar_addr(st.mbar, st.slot)
        self.k(f"{self.guard()}mbarrier.arrive.shared::cta.b64 _, [{a}]")

    def do_mbar_wait(self, st: ir.MbarrierWait) -> None:
        """Wait for the completion of phase ``phase`` (parity phase & 1),
        bounded: past MBAR_WAIT_NS the lane records ERR_MBAR_WAIT and goes on."""
        k, lo = self.k, self.lo
        a = self.mbar_addr(st.mbar, st.slot)
        ph = lo.coerce(lo.ev(st.phase) if hasattr(st.phase, "free_vars")
                       else lo.const(int(st.phase), "s32"), "s32")
        par = k.reg("u32")
        k(f"and.b32 {par}, {ph.reg}, 1")
        done, loop = k.label("mbw_done"), k.label("mbw")
        p = k.reg("pred")
        if lo.mask is not None:
            k(f"@!{lo.mask} bra {done}")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{a}], {par}")
        k(f"@{p} bra {done}")
        t0, t1 = k.reg("u64"), k.reg("u64")
        k(f"mov.u64 {t0}, %globaltimer")
        k.place(loop)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{a}], {par}, 100000")
        k(f"@{p} bra {done}")
        k(f"mov.u64 {t1}, %globaltimer")
        k(f"sub.u64 {t1}, {t1}, {t0}")
        k(f"setp.lt.u64 {p}, {t1}, {MBAR_WAIT_NS}")
        k(f"@{p} bra {loop}")
        old = k.reg("u32")
        k(f"atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_MBAR_WAIT}")
        k.place(done)

    def do_tma_load(self, st: ir.TmaLoad) -> None:
        """The box of ``st.desc`` at ``st.coords`` into Smem ``st.smem`` at
        element ``st.smem_index``, completing its bytes on ``st.mbar``."""
        k, lo = self.k, self.lo
        d = self.tma.get(st.desc)
        if d is None:
            raise LowerError(f"unknown TMA descriptor {st.desc!r}")
        if st.smem not in self.smem:
            raise LowerError(f"TMA destination {st.smem!r} is not a Smem buffer")
        shape = [int(e) for e in d.src_shape]
        box = [int(e) for e in d.box_extents]
        if len(st.coords) != len(shape):
            raise LowerError("TMA coords and descriptor rank differ")
        eb = dtype_info(self.spec.args[d.src_buf].dtype)[2]
        sshape, sdt, soff = self.smem[st.smem]
        if dtype_info(sdt)[2] != eb:
            raise LowerError("TMA source and destination element sizes differ")
        span = _TMA_SPAN[str(d.swizzle or "NONE")]
        bi, W = box[-1], shape[-1]
        row_bytes = bi * eb
        nbox = numel(box)
        rows = nbox // bi
        if nbox > numel(sshape):
            raise LowerError(f"TMA box of {nbox} elements exceeds Smem {st.smem!r}")
        done = k.label("tma_done")
        if lo.mask is not None:
            k(f"@!{lo.mask} bra {done}")
        coords = [lo.coerce(lo.ev(c), "s32").reg for c in st.coords]
        idx = st.smem_index if isinstance(st.smem_index, tuple) else (st.smem_index,)
        dshape = sshape if isinstance(st.smem_index, tuple) else (numel(sshape),)
        di = self.flat(idx, dshape)
        bar = self.mbar_addr(st.mbar, st.mbar_slot)
        dst = k.reg("u32")
        k(f"mad.lo.u32 {dst}, {di.reg}, {eb}, {self.smem_base}")
        k(f"add.u32 {dst}, {dst}, {soff}")
        # checks: inner coordinate on 16 bytes, destination aligned, box inside Smem
        bad, q = k.reg("pred"), k.reg("pred")
        t = k.reg("u32")
        k(f"mul.lo.u32 {t}, {coords[-1]}, {eb}")
        k(f"and.b32 {t}, {t}, 15")
        k(f"setp.ne.u32 {bad}, {t}, 0")
        k(f"and.b32 {t}, {dst}, {(1024 if span else 16) - 1}")
        k(f"setp.ne.or.u32 {bad}, {t}, 0, {bad}")
        k(f"setp.gt.u32 {q}, {di.reg}, {numel(sshape) - nbox}")
        k(f"or.pred {bad}, {bad}, {q}")
        ok_l = k.label("tma_ok")
        k(f"@!{bad} bra {ok_l}")
        old = k.reg("u32")
        k(f"atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_TMA}")
        k(f"mbarrier.complete_tx.relaxed.cta.shared::cta.b64 [{bar}], {nbox * eb}")
        k(f"bra {done}")
        k.place(ok_l)
        # generic-proxy accesses to the destination come before the copies
        k("fence.proxy.async.shared::cta")
        zeros = k.reg("u64")
        k(f"mov.u64 {zeros}, emmy_zeros")
        base = self.base[d.src_buf]
        # x range of the box that lies inside the view: [lo, hi)
        xlo, xhi, xend = k.reg("s32"), k.reg("s32"), k.reg("s32")
        k(f"add.s32 {xend}, {coords[-1]}, {bi}")
        k(f"max.s32 {xlo}, {coords[-1]}, 0")
        k(f"min.s32 {xlo}, {xlo}, {xend}")
        k(f"min.s32 {xhi}, {xend}, {W}")
        ri = k.reg("u32")
        k(f"mov.u32 {ri}, 0")
        head = k.label("tma_row")
        k.place(head)
        # outer coordinates of row ri; inside the view?
        inrow = k.reg("pred")
        k("setp.eq.u32 {}, 0, 0".format(inrow))
        rowoff = k.reg("s64")
        k(f"mov.s64 {rowoff}, 0")
        rem = k.reg("u32")
        k(f"mov.u32 {rem}, {ri}")
        # row-major decode of ri over box[:-1] (innermost outer dim first)
        outer = []
        for dim in range(len(shape) - 2, -1, -1):
            o, oc = k.reg("u32"), k.reg("s32")
            if dim == 0:
                k(f"mov.u32 {o}, {rem}")
            else:
                k(f"rem.u32 {o}, {rem}, {box[dim]}")
                k(f"div.u32 {rem}, {rem}, {box[dim]}")
            k(f"add.s32 {oc}, {coords[dim]}, {o}")
            k(f"setp.lt.and.u32 {inrow}, {oc}, {shape[dim]}, {inrow}")
            outer.append((dim, oc))
        stride = W
        for dim, oc in outer:          # innermost outer dim first
            w = k.reg("s64")
            k(f"mul.wide.s32 {w}, {oc}, {stride}")
            k(f"add.s64 {rowoff}, {rowoff}, {w}")
            stride *= shape[dim]
        lo_r, hi_r = k.reg("s32"), k.reg("s32")
        k(f"selp.s32 {lo_r}, {xlo}, {coords[-1]}, {inrow}")
        k(f"selp.s32 {hi_r}, {xhi}, {coords[-1]}, {inrow}")
        k(f"max.s32 {hi_r}, {hi_r}, {lo_r}")
        # the source address of element x of this row is base + (rowoff + x) * eb
        srow = k.reg("u64")
        k(f"mad.lo.s64 {srow}, {rowoff}, {eb}, {base}")
        drow = k.reg("u32")
        k(f"mad.lo.u32 {drow}, {ri}, {row_bytes}, {dst}")
        cp = "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes"
        if not span:
            # zeros [x0, lo), the view's part [lo, hi), zeros [hi, x0 + bi)
            for a_, b_, from_src in ((coords[-1], lo_r, False), (lo_r, hi_r, True),
                                     (hi_r, xend, False)):
                n_, dd, sz = k.reg("s32"), k.reg("u32"), k.reg("u32")
                skip = k.reg("pred")
                k(f"sub.s32 {n_}, {b_}, {a_}")
                k(f"setp.le.s32 {skip}, {n_}, 0")
                k(f"mul.lo.u32 {sz}, {n_}, {eb}")
                k(f"sub.s32 {dd}, {a_}, {coords[-1]}")
                k(f"mad.lo.u32 {dd}, {dd}, {eb}, {drow}")
                if from_src:
                    sa = k.reg("u64")
                    k(f"mad.wide.s32 {sa}, {a_}, {eb}, {srow}")
                    k(f"@!{skip} {cp} [{dd}], [{sa}], {sz}, [{bar}]")
                else:
                    k(f"@!{skip} {cp} [{dd}], [{zeros}], {sz}, [{bar}]")
        else:
            m = span // 16 - 1
            for j in range(row_bytes // 16):
                # chunk j of the row: inside the view when lo <= x0 + j*16/eb < hi
                x, o, ph, dd = k.reg("s32"), k.reg("u32"), k.reg("u32"), k.reg("u32")
                inside, p2 = k.reg("pred"), k.reg("pred")
                k(f"add.s32 {x}, {coords[-1]}, {j * 16 // eb}")
                k(f"setp.ge.s32 {inside}, {x}, {lo_r}")
                k(f"setp.lt.and.s32 {inside}, {x}, {hi_r}, {inside}")
                k(f"mad.lo.u32 {o}, {ri}, {row_bytes}, {j * 16}")
                k(f"shr.u32 {ph}, {o}, 7")
                k(f"and.b32 {ph}, {ph}, {m}")
                k(f"shl.b32 {ph}, {ph}, 4")
                k(f"xor.b32 {o}, {o}, {ph}")
                k(f"add.u32 {dd}, {dst}, {o}")
                sa = k.reg("u64")
                k(f"mad.wide.s32 {sa}, {x}, {eb}, {srow}")
                k(f"selp.b64 {sa}, {sa}, {zeros}, {inside}")
                k(f"{cp} [{dd}], [{sa}], 16, [{bar}]")
        k(f"add.u32 {ri}, {ri}, 1")
        p3 = k.reg("pred")
        k(f"setp.lt.u32 {p3}, {ri}, {rows}")
        k(f"@{p3} bra {head}")
        k.place(done)


    # -- warp-level tensor-core fragments (mma.sync) ------------------------

    def frag_cell(self, ref, index=None) -> tuple[str, list]:
        name, _, rest = str(ref).partition("[")
        cell = int(rest.rstrip("]")) if rest else 0
        if index is not None:
            if rest:
                raise LowerError(f"fragment {ref!r} indexed twice")
            if not isinstance(index, (int, ir.Literal)):
                raise LowerError("fragment_index must be a literal")
            cell = int(index.value if isinstance(index, ir.Literal) else index)
        if name not in self.frags:
            raise LowerError(f"undeclared fragment {name!r}")
        cells = self.frags[name][2]
        if not 0 <= cell < len(cells):
            raise LowerError(f"fragment cell {cell} of {name!r}")
        return name, cells[cell]

    def frag_error(self, ok: str) -> None:
        """Record ERR_FRAG for a lane whose fragment access left its buffer."""
        k = self.k
        skip, old = k.label("frag_ok"), k.reg("u32")
        k(f"@{ok} bra {skip}")
        k(f"atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_FRAG}")
        k.place(skip)

    def do_reg_fragment(self, st: ir.RegFragment) -> None:
        k = self.k
        role = str(st.role).lower()
        wg_n = wgmma_n(st.shape)
        if str(st.shape) != "m16n8k16" and not (role == "c" and wg_n):
            raise LowerError(f"{role} fragment shape {st.shape!r}")
        dt = dtype_info(st.dtype)[0]
        if (role in ("a", "b") and dt not in ("bf16", "f16")) or (
                role == "c" and dt != "f32" and not (dt == "f16" and not wg_n)):
            raise LowerError(f"{role} fragment of {st.dtype!r}")
        # an f16 c cell is two packed f16 pairs
        nregs = {"a": 4, "b": 2, "c": wg_n // 2 if wg_n else (2 if dt == "f16" else 4)}[role]
        if st.name not in self.frags:
            cells = [k.regs("f32" if role == "c" and dt == "f32" else "b32", nregs)
                     for _ in range(int(st.count or 1))]
            self.frags[st.name] = (role, dt, cells)
            self.frag_shape[st.name] = str(st.shape)
        role0, dt0, cells = self.frags[st.name]
        if (role0, dt0, len(cells)) != (role, dt, int(st.count or 1)):
            raise LowerError(f"fragment {st.name!r} declared twice differently")
        for cell in cells:
            for r in cell:
                k(f"mov.b32 {r}, 0")

    def do_ldmatrix(self, st: ir.LdmatrixLoad) -> None:
        k, lo = self.k, self.lo
        for opt in ("staged", "gmem_guard", "k_zero", "pair_frag", "byte_slab",
                    "scale_buffer", "scale_index", "scale_ldm", "fragment_layout"):
            if getattr(st, opt) not in (None, False, "NONE"):
                raise LowerError(f"LdmatrixLoad option {opt}")
        name, regs = self.frag_cell(st.frag, st.fragment_index)
        role = self.frags[name][0]
        if role != str(st.role).lower() or role not in ("a", "b"):
            raise LowerError(f"LdmatrixLoad role {st.role!r} into {role} fragment {name!r}")
        if st.src_buffer not in self.smem or dtype_info(self.smem[st.src_buffer][1])[2] != 2:
            raise LowerError("LdmatrixLoad reads a 16-bit Smem buffer")
        shape, _, off = self.smem[st.src_buffer]
        ldm = int(st.ldm) if st.ldm is not None else int(shape[-1])
        lane = lo.env["lane"].reg
        r, c = k.reg("s32"), k.reg("s32")
        # the row this lane addresses: A rows 0-15 for k 0-7 (lanes 0-15) and
        # k 8-15 (lanes 16-31); B [N][K]: n 0-7 for k 0-7 and 8-15 (lanes
        # 0-15); B [K][N] (.trans): k 0-15 (lanes 0-15)
        if role == "a":
            k(f"and.b32 {r}, {lane}, 15")
            k(f"shr.b32 {c}, {lane}, 4")
            k(f"shl.b32 {c}, {c}, 3")
        elif st.b_trans:
            k(f"and.b32 {r}, {lane}, 15")
            k(f"mov.b32 {c}, 0")
        else:
            k(f"and.b32 {r}, {lane}, 7")
            k(f"shr.b32 {c}, {lane}, 3")
            k(f"and.b32 {c}, {c}, 1")
            k(f"shl.b32 {c}, {c}, 3")
        r0 = lo.coerce(lo.ev(st.src_index[0]), "s32").reg
        c0 = lo.coerce(lo.ev(st.src_index[1]), "s32").reg
        flat = k.reg("s32")
        k(f"add.s32 {r}, {r}, {r0}")
        k(f"add.s32 {c}, {c}, {c0}")
        k(f"mad.lo.s32 {flat}, {r}, {ldm}, {c}")
        fl = self.swizzle(Val(flat, "s32"), st.swizzle).reg
        ok = k.reg("pred")
        k(f"setp.le.u32 {ok}, {fl}, {numel(shape) - 8}")
        self.frag_error(ok)
        safe, a = k.reg("s32"), k.reg("u32")
        k(f"selp.s32 {safe}, {fl}, 0, {ok}")
        k(f"mad.lo.u32 {a}, {safe}, 2, {self.smem_base}")
        if off:
            k(f"add.u32 {a}, {a}, {off}")
        if role == "a":
            k(f"ldmatrix.sync.aligned.m8n8.x4.shared.b16 {{{', '.join(regs)}}}, [{a}]")
        else:
            tr = ".trans" if st.b_trans else ""
            k(f"ldmatrix.sync.aligned.m8n8.x2{tr}.shared.b16 {{{', '.join(regs)}}}, [{a}]")

    def do_mma_sync(self, st: ir.MmaSyncPtx) -> None:
        if str(st.shape) != "m16n8k16" or st.b_row_major or st.sfa_frag or st.sfb_frag:
            raise LowerError("MmaSyncPtx: m16n8k16, B column-major, no scales")
        an, a = self.frag_cell(st.a_frag)
        bn, b = self.frag_cell(st.b_frag)
        cn, c = self.frag_cell(st.c_frag)
        if (self.frags[an][0], self.frags[bn][0], self.frags[cn][0]) != ("a", "b", "c"):
            raise LowerError("MmaSyncPtx takes a, b and c fragments")
        ab = self.frags[an][1]
        if self.frags[bn][1] != ab:
            raise LowerError("MmaSyncPtx: A and B of different types")
        if self.frags[cn][1] == "f16":
            if ab != "f16":
                raise LowerError("an f16 accumulator takes f16 A and B")
            self.k(f"mma.sync.aligned.m16n8k16.row.col.f16.f16.f16.f16 "
                   f"{{{', '.join(c)}}}, {{{', '.join(a)}}}, {{{', '.join(b)}}}, "
                   f"{{{', '.join(c)}}}")
            return
        self.k(f"mma.sync.aligned.m16n8k16.row.col.f32.{ab}.{ab}.f32 "
               f"{{{', '.join(c)}}}, {{{', '.join(a)}}}, {{{', '.join(b)}}}, "
               f"{{{', '.join(c)}}}")

    def do_reg_store(self, st: ir.RegStore) -> None:
        k, lo = self.k, self.lo
        for opt in ("epilogue", "extra_frags", "fragment_layout", "volta_interleaved",
                    "row_dim", "col_dim"):
            if getattr(st, opt) not in (None, False, (), []):
                raise LowerError(f"RegStore option {opt}")
        if str(st.swizzle or "NONE") != "NONE":
            raise LowerError("RegStore swizzle")
        name, regs = self.frag_cell(st.frag, st.fragment_index)
        if self.frags[name][0] != "c":
            raise LowerError("RegStore stores a c fragment")
        if self.frags[name][1] == "f16":
            regs = self.unpack_f16(regs)
        if st.dst_buffer not in self.base:
            raise LowerError(f"RegStore into {st.dst_buffer!r}")
        shape = self.spec.args[st.dst_buffer].shape
        ldm = int(st.ldm) if st.ldm is not None else int(shape[-1])
        lane = lo.env["lane"].reg
        g, t = k.reg("s32"), k.reg("s32")
        k(f"shr.b32 {g}, {lane}, 2")
        k(f"and.b32 {t}, {lane}, 3")
        k(f"shl.b32 {t}, {t}, 1")
        r0 = lo.coerce(lo.ev(st.dst_index[0]), "s32").reg
        c0 = lo.coerce(lo.ev(st.dst_index[1]), "s32").reg
        if wgmma_n(self.frag_shape.get(name)):
            # warpgroup accumulator: warp w of the group holds rows 16w..16w+15
            wr = k.reg("s32")
            k(f"shr.b32 {wr}, {self.tid}, 5")
            k(f"and.b32 {wr}, {wr}, 3")
            k(f"mad.lo.s32 {g}, {wr}, 16, {g}")
        mg = lo.coerce(lo.ev(st.m_guard), "s32").reg if st.m_guard is not None else None
        ng = lo.coerce(lo.ev(st.n_guard), "s32").reg if st.n_guard is not None else None
        dt = self.spec.args[st.dst_buffer].dtype
        for e, v in enumerate(regs):
            j, i = e // 4, e % 4
            row, col, idx = k.reg("s32"), k.reg("s32"), k.reg("s32")
            k(f"add.s32 {row}, {r0}, {g}")
            if i // 2:
                k(f"add.s32 {row}, {row}, 8")
            k(f"add.s32 {col}, {c0}, {t}")
            if i % 2 or j:
                k(f"add.s32 {col}, {col}, {8 * j + i % 2}")
            k(f"mad.lo.s32 {idx}, {row}, {ldm}, {col}")
            want = k.reg("pred")
            k("setp.eq.u32 {}, 0, 0".format(want))
            if mg is not None:
                k(f"setp.lt.and.s32 {want}, {row}, {mg}, {want}")
            if ng is not None:
                k(f"setp.lt.and.s32 {want}, {col}, {ng}, {want}")
            if lo.mask is not None:
                k(f"and.pred {want}, {want}, {lo.mask}")
            inb, ok = k.reg("pred"), k.reg("pred")
            k(f"setp.lt.u32 {inb}, {idx}, {numel(shape)}")
            # a wanted element outside the buffer is an error, not a store
            k(f"not.pred {ok}, {want}")
            k(f"or.pred {ok}, {ok}, {inb}")
            self.frag_error(ok)
            k(f"and.pred {want}, {want}, {inb}")
            safe = k.reg("s32")
            k(f"selp.s32 {safe}, {idx}, 0, {inb}")
            a, sh, _ = self.addr(st.dst_buffer, Val(safe, "s32"))
            saved = lo.mask
            lo.mask = want
            self.store_elem(a, sh, dt, Val(v, "f32"), atomic=bool(st.atomic))
            lo.mask = saved


    def c_cell(self, ref, dtype="f32") -> list:
        name, regs = self.frag_cell(ref)
        if (self.frags[name][0], self.frags[name][1]) != ("c", dtype) or \
                self.frag_shape[name] != "m16n8k16":
            raise LowerError(f"{ref!r} is not an m16n8 {dtype} c fragment")
        return regs

    def unpack_f16(self, regs) -> list:
        """Four f32 values of a packed f16 c cell (element 2j in the low half)."""
        k, out = self.k, []
        for r in regs:
            lo16, hi16 = k.reg("b16"), k.reg("b16")
            k(f"mov.b32 {{{lo16}, {hi16}}}, {r}")
            for h in (lo16, hi16):
                f = k.reg("f32")
                k(f"cvt.f32.f16 {f}, {h}")
                out.append(f)
        return out

    def do_frag_promote(self, st: ir.FragmentPromote) -> None:
        k = self.k
        dst = self.c_cell(st.dst)
        src = self.c_cell(st.src, "f16")
        vals = self.unpack_f16(src)
        g = self.guard()
        for d, v in zip(dst, vals):
            t = k.reg("f32")
            k(f"add.rn.f32 {t}, {d}, {v}")
            k(f"{g}mov.f32 {d}, {t}")
        for r in src:
            k(f"{g}mov.b32 {r}, 0")

    def do_frag_apply(self, st: ir.FragmentApply) -> None:
        """op per element of an m16n8 c cell with the IR's op lowering;
        "row" arguments give top to elements 0-1 (row g), bot to 2-3."""
        k, lo = self.k, self.lo
        if st.layout is not None or st.post is not None:
            raise LowerError("FragmentApply layout / post")
        out = self.c_cell(st.out)
        if len(st.args) != len(st.kinds):
            raise LowerError("FragmentApply args and kinds differ in length")
        cols = []
        if st.in_place:
            cols.append(lambda e: Val(out[e], "f32"))
        for a, kd in zip(st.args, st.kinds):
            if kd == "frag":
                src = self.c_cell(a)
                cols.append(lambda e, src=src: Val(src[e], "f32"))
            elif kd == "row":
                top, bot = (lo.env[x] for x in a)
                cols.append(lambda e, top=top, bot=bot: bot if e >= 2 else top)
            elif kd == "scalar":
                v = lo.env[a] if isinstance(a, str) else lo.ev(a)
                cols.append(lambda e, v=v: v)
            else:
                raise LowerError(f"FragmentApply argument kind {kd!r}")
        opname = getattr(st.op, "name", st.op)
        res = [lo.coerce(lo.apply(opname, [f(e) for f in cols]), "f32") for e in range(4)]
        g = self.guard()
        for e in range(4):
            k(f"{g}mov.f32 {out[e]}, {res[e].reg}")

    def do_frag_rowreduce(self, st: ir.FragmentRowReduce) -> None:
        k, lo = self.k, self.lo
        refs = [st.frags] if isinstance(st.frags, str) else list(st.frags)
        cells = [self.c_cell(r) for r in refs]
        opname = ops.canon(getattr(st.op, "name", st.op))
        if opname not in ("add", "maximum", "minimum"):
            raise LowerError(f"FragmentRowReduce op {st.op!r}")
        for half, name in ((0, st.top), (1, st.bot)):
            v = None
            for c in cells:
                for e in (2 * half, 2 * half + 1):
                    x = Val(c[e], "f32")
                    v = x if v is None else lo.coerce(lo.apply(opname, [v, x]), "f32")
            for x in (1, 2):
                t = k.reg("f32")
                k(f"shfl.sync.bfly.b32 {t}, {v.reg}, {x}, 31, -1")
                v = lo.coerce(lo.apply(opname, [v, Val(t, "f32")]), "f32")
            lo.bind(name, v)

    def do_frag_repack(self, st: ir.FragmentRepack) -> None:
        k = self.k
        if st.fragment_layout is not None or st.part is not None:
            raise LowerError("FragmentRepack layout / part")
        name, regs = self.frag_cell(st.frag)
        role, dt = self.frags[name][0], self.frags[name][1]
        if role != "a" or dtype_info(st.ab_dtype)[0] != dt:
            raise LowerError("FragmentRepack fills an a fragment of its own type")
        if len(st.srcs) != 2:
            raise LowerError("FragmentRepack takes two c cells")
        src = self.c_cell(st.srcs[0]) + self.c_cell(st.srcs[1])
        for j in range(4):
            # element 2j in the low half, 2j + 1 in the high half
            k(f"cvt.rn.{dt}x2.f32 {regs[j]}, {src[2 * j + 1]}, {src[2 * j]}")

    # -- carried state (Pre / Carry) ----------------------------------------

    def carry_cell(self, index) -> tuple:
        idx = index if isinstance(index, tuple) else (() if index is None else (index,))
        out = []
        for e in idx:
            v = e.value if isinstance(e, ir.Literal) else e
            if not isinstance(v, int) or isinstance(v, bool):
                raise LowerError("carried-state cells take literal indices")
            out.append(int(v))
        return tuple(out)

    def carry_pair(self, c: str, cell: tuple) -> tuple:
        """(state, next state) registers of one cell, seeded where first used
        (the prologue runs before any loop, so a cell read before its
        carrying loop holds the seed)."""
        if (c, cell) not in self.carry_regs:
            seed, dt = self.carriers[c]
            kind = value_kind(dt)
            if kind == "f32":
                imm = f32_hex(float(seed))
            elif kind == "f64":
                imm = f64_hex(float(seed))
            elif kind in ("s32", "s64"):
                imm = str(int(seed))
            else:
                raise LowerError(f"carrier {c!r} of dtype {dt!r}")
            cur, nxt = self.k.reg(kind), self.k.reg(kind)
            # registers set in the kernel's first lines, ahead of every loop
            t = {"f32": "f32", "f64": "f64", "s32": "b32", "s64": "b64"}[kind]
            self.k.lines.insert(self.carry_at, f"\tmov.{t} {cur}, {imm};")
            self.k.lines.insert(self.carry_at, f"\tmov.{t} {nxt}, {imm};")
            self.carry_regs[(c, cell)] = (cur, nxt, kind, imm)
        return self.carry_regs[(c, cell)]

    def carry_reset(self, c: str, body) -> None:
        """Seed every cell of ``c`` as its carrying loop starts (cells first
        met inside the loop included)."""
        for st in ir.walk(body):
            if isinstance(st, ir.Carry) and st.name == c:
                self.carry_pair(c, self.carry_cell(st.index))
            elif isinstance(st, ir.Pre) and st.carrier == c:
                self.carry_pair(c, self.carry_cell(st.index))
        g = self.guard()
        for (cc, cell), (cur, nxt, kind, imm) in list(self.carry_regs.items()):
            if cc == c:
                t = {"f32": "f32", "f64": "f64", "s32": "b32", "s64": "b64"}[kind]
                self.k(f"{g}mov.{t} {cur}, {imm}")
                self.k(f"{g}mov.{t} {nxt}, {imm}")

    def carry_commit(self, c: str) -> None:
        for (cc, cell), (cur, nxt, kind, _) in list(self.carry_regs.items()):
            if cc == c:
                t = {"f32": "f32", "f64": "f64", "s32": "b32", "s64": "b64"}[kind]
                self.k(f"mov.{t} {cur}, {nxt}")

    def do_pre(self, st: ir.Pre) -> None:
        if st.carrier not in self.carriers:
            raise LowerError(f"carrier {st.carrier!r} has no Carry")
        cur, _, kind, _ = self.carry_pair(st.carrier, self.carry_cell(st.index))
        self.lo.bind(st.name, Val(cur, kind))

    def do_carry(self, st: ir.Carry) -> None:
        cur, nxt, kind, _ = self.carry_pair(st.name, self.carry_cell(st.index))
        if st.value not in self.lo.env:
            raise LowerError(f"undefined name {st.value!r}")
        v = self.lo.coerce(self.lo.env[st.value], kind)
        t = {"f32": "f32", "f64": "f64", "s32": "b32", "s64": "b64"}[kind]
        g = self.guard()
        self.k(f"{g}mov.{t} {nxt}, {v.reg}")
        if st.name in self.carry_top:
            self.k(f"{g}mov.{t} {cur}, {v.reg}")

    # -- warpgroup products on tcgen05 ----------------------------------------

    def setup_wgmma(self) -> None:
        """TMEM for every warpgroup's accumulators, allocated once by warp 0,
        and one commit mbarrier per warpgroup."""
        mmas = [st for st in ir.walk(self.spec.op.body) if isinstance(st, ir.WgmmaMma)]
        if not mmas:
            return
        k = self.k
        block = int(self.spec.block[0])
        if block % 128:
            raise LowerError("wgmma needs whole warpgroups (blocks of 128 threads)")
        nwg = block // 128
        cols: dict[str, int] = {}
        for st in mmas:
            n = wgmma_n(st.shape)
            if not n:
                raise LowerError(f"WgmmaMma shape {st.shape!r}")
            name = str(st.c_frags).partition("[")[0]
            cols[name] = max(cols.get(name, 0), n)
        offs, total = {}, 0
        for name, n in cols.items():
            offs[name] = total
            total += n
        per_wg = max(32, 1 << (total - 1).bit_length())
        ncols = max(32, 1 << (nwg * per_wg - 1).bit_length())
        if ncols > 512:
            raise LowerError(f"wgmma accumulators need {ncols} TMEM columns (512 at most)")
        k.shared(f"\t.shared .align 8 .b64 emmy_wg_bar[{nwg}];")
        k.shared("\t.shared .align 4 .u32 emmy_tmem_slot;")
        p = k.reg("pred")
        warp, wg = k.reg("u32"), k.reg("u32")
        k(f"shr.u32 {warp}, {self.tid}, 5")
        k(f"shr.u32 {wg}, {self.tid}, 7")
        skip = k.label("wg_init")
        k(f"setp.ne.u32 {p}, {self.tid}, 0")
        k(f"@{p} bra {skip}")
        for i in range(nwg):
            k(f"mbarrier.init.shared::cta.b64 [emmy_wg_bar+{8 * i}], 1")
        k("fence.mbarrier_init.release.cluster")
        k.place(skip)
        skip2 = k.label("wg_alloc")
        k(f"setp.ne.u32 {p}, {warp}, 0")
        k(f"@{p} bra {skip2}")
        slot = k.reg("u32")
        k(f"mov.u32 {slot}, emmy_tmem_slot")
        k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], {ncols}")
        k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
        k.place(skip2)
        k("tcgen05.fence::before_thread_sync")
        k("barrier.sync 0")
        k("tcgen05.fence::after_thread_sync")
        tmem, tcol, lanef, bar, ph, issuer = (k.reg("u32") for _ in range(6))
        k(f"ld.shared.u32 {tmem}, [emmy_tmem_slot]")
        k(f"mad.lo.u32 {tcol}, {wg}, {per_wg}, {tmem}")
        k(f"and.b32 {lanef}, {warp}, 3")
        k(f"shl.b32 {lanef}, {lanef}, 21")          # (32 * (warp % 4)) << 16
        k(f"mov.u32 {bar}, emmy_wg_bar")
        k(f"mad.lo.u32 {bar}, {wg}, 8, {bar}")
        k(f"mov.u32 {ph}, 0")
        ip = k.reg("pred")
        k(f"and.b32 {issuer}, {self.tid}, 127")
        k(f"setp.eq.u32 {ip}, {issuer}, 0")
        self.wg = {"ncols": ncols, "offs": offs, "tmem": tmem, "tcol": tcol, "lane": lanef,
                   "bar": bar, "ph": ph, "issuer": ip, "wg": wg, "resident": set(),
                   "pending": False}

    def finish_wgmma(self) -> None:
        if self.wg is None:
            return
        k = self.k
        if self.wg["resident"] or self.wg["pending"]:
            raise LowerError("wgmma products left in flight at the end of the kernel")
        k("tcgen05.fence::before_thread_sync")
        k("barrier.sync 0")
        p, warp = k.reg("pred"), k.reg("u32")
        skip = k.label("wg_free")
        k(f"shr.u32 {warp}, {self.tid}, 5")
        k(f"setp.ne.u32 {p}, {warp}, 0")
        k(f"@{p} bra {skip}")
        k("tcgen05.fence::after_thread_sync")
        k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {self.wg['tmem']}, {self.wg['ncols']}")
        k.place(skip)

    def wg_state(self):
        return None if self.wg is None else (frozenset(self.wg["resident"]), self.wg["pending"])

    def do_wgmma_desc(self, st: ir.WgmmaDescriptor) -> None:
        k, lo = self.k, self.lo
        if st.smem not in self.smem or dtype_info(self.smem[st.smem][1])[2] != 2:
            raise LowerError("wgmma descriptors address a 16-bit Smem buffer")
        swz = str(st.swizzle or "NONE")
        if swz not in _WG_LAYOUT:
            raise LowerError(f"wgmma descriptor swizzle {swz!r}")
        shape, _, off = self.smem[st.smem]
        if swz != "NONE" and off % 1024:
            raise LowerError(f"swizzled wgmma operand {st.smem!r} needs 1024-byte alignment")
        idx = st.smem_index if st.smem_index is not None else ir.Literal(0, None)
        tup = idx if isinstance(idx, tuple) else (idx,)
        el = self.flat(tup, shape if len(tup) > 1 else (numel(shape),)).reg
        a, d = k.reg("u32"), k.reg("u64")
        k(f"mad.lo.u32 {a}, {el}, 2, {self.smem_base}")
        if off:
            k(f"add.u32 {a}, {a}, {off}")
        lbo, sbo = int(st.lbo_bytes or 0), int(st.sbo_bytes or 0)
        fixed = ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1 << 46) | (_WG_LAYOUT[swz] << 61)
        t = k.reg("u32")
        k(f"shr.u32 {t}, {a}, 4")
        k(f"and.b32 {t}, {t}, 16383")
        k(f"cvt.u64.u32 {d}, {t}")
        k(f"or.b64 {d}, {d}, 0x{fixed:016X}")
        self.wgdesc[st.name] = (d, el, st.smem, swz, lbo, sbo)

    def wg_operand_ok(self, name: str, rows: int) -> str:
        """Predicate: the operand's first byte is 16-byte aligned and every
        byte the product reads lies inside its Smem buffer."""
        k = self.k
        if name not in self.wgdesc:
            raise LowerError(f"unknown wgmma descriptor {name!r}")
        _, el, smem, swz, lbo, sbo = self.wgdesc[name]
        size = numel(self.smem[smem][0]) * 2
        span = {"NONE": 0, "B32": 32, "B64": 64, "B128": 128}[swz]
        b, t = k.reg("u32"), k.reg("u32")
        ok, q = k.reg("pred"), k.reg("pred")
        k(f"shl.b32 {b}, {el}, 1")
        k(f"and.b32 {t}, {b}, 15")
        k(f"setp.eq.u32 {ok}, {t}, 0")
        if span:
            # the 16-deep K slice stays inside one swizzled row
            k(f"rem.u32 {t}, {b}, {span}")
            k(f"setp.le.and.u32 {ok}, {t}, {span - 32}, {ok}")
            k(f"sub.u32 {t}, {b}, {t}")
            end = (rows // 8 - 1) * sbo + 8 * span
        else:
            k(f"mov.u32 {t}, {b}")
            end = (rows // 8 - 1) * sbo + lbo + 8 * 16
        k(f"setp.le.u32 {q}, {t}, {max(-1, size - end)}")
        k(f"and.pred {ok}, {ok}, {q}")
        if size - end < 0:
            k(f"setp.ne.u32 {ok}, 0, 0")
        return ok

    def do_wgmma(self, st: ir.WgmmaMma) -> None:
        k, lo, wg = self.k, self.lo, self.wg
        n = wgmma_n(st.shape)
        if wg is None or not n:
            raise LowerError(f"WgmmaMma shape {st.shape!r}")
        if st.a_frag is not None or st.a_desc is None or st.trans_a or st.trans_b:
            raise LowerError("WgmmaMma: A and B K-major from shared-memory descriptors")
        name, regs = self.frag_cell(st.c_frags)
        if self.frags[name][0] != "c" or wgmma_n(self.frag_shape[name]) != n:
            raise LowerError("WgmmaMma needs a c fragment of its own shape")
        ab = dtype_info(st.ab_dtype)[0]
        if ab not in ("bf16", "f16"):
            raise LowerError(f"WgmmaMma of {st.ab_dtype!r}")
        ok = self.wg_operand_ok(st.a_desc, 64)
        okb = self.wg_operand_ok(st.b_desc, n)
        k(f"and.pred {ok}, {ok}, {okb}")
        col = k.reg("u32")
        k(f"add.u32 {col}, {wg['tcol']}, {wg['offs'][name]}")
        if name not in wg["resident"]:
            ta = k.reg("u32")
            k(f"add.u32 {ta}, {col}, {wg['lane']}")
            k(f"tcgen05.st.sync.aligned.16x256b.x{n // 8}.b32 [{ta}], {{{', '.join(regs)}}}")
            k("tcgen05.wait::st.sync.aligned")
            wg["resident"].add(name)
        # operands (written through either proxy) and C visible to the MMA
        k("fence.proxy.async.shared::cta")
        k("tcgen05.fence::before_thread_sync")
        bid = "15" if int(self.spec.block[0]) == 128 else self.wg_barrier_id()
        k(f"barrier.sync {bid}, 128")
        k("tcgen05.fence::after_thread_sync")
        sd = (lo.truthy(lo.ev(st.scale_d)).reg if hasattr(st.scale_d, "free_vars") else None)
        if sd is None:
            sd = k.reg("pred")
            k(f"setp.ne.u32 {sd}, {1 if st.scale_d else 0}, 0")
        fmt = 1 if ab == "bf16" else 0
        idesc = (1 << 4) | (fmt << 7) | (fmt << 10) | ((n >> 3) << 17) | ((64 >> 4) << 24)
        idr = k.reg("u32")
        k(f"mov.u32 {idr}, {idesc}")
        go, bad = k.reg("pred"), k.reg("pred")
        k(f"and.pred {go}, {wg['issuer']}, {ok}")
        k(f"not.pred {bad}, {ok}")
        k(f"and.pred {bad}, {bad}, {wg['issuer']}")
        old = k.reg("u32")
        k(f"@{bad} atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_WGMMA}")
        k(f"@{go} tcgen05.mma.cta_group::1.kind::f16 [{col}], {self.wgdesc[st.a_desc][0]}, "
          f"{self.wgdesc[st.b_desc][0]}, {idr}, {sd}")

    def wg_barrier_id(self) -> str:
        """Named barrier of this thread's warpgroup: 15 - warpgroup."""
        k = self.k
        r = k.reg("u32")
        k(f"sub.u32 {r}, 15, {self.wg['wg']}")
        return r

    def do_wgmma_commit(self, st: ir.WgmmaCommit) -> None:
        wg = self.wg
        if wg is None:
            raise LowerError("WgmmaCommit without a WgmmaMma")
        if wg["pending"]:
            raise LowerError("two WgmmaCommit without a WgmmaWait between them")
        self.k(f"@{wg['issuer']} tcgen05.commit.cta_group::1.mbarrier::arrive::one."
               f"shared::cluster.b64 [{wg['bar']}]")
        wg["pending"] = True

    def do_wgmma_wait(self, st: ir.WgmmaWait) -> None:
        k, wg = self.k, self.wg
        if int(st.group or 0) != 0:
            raise LowerError("WgmmaWait with groups left in flight")
        if wg is None:
            return
        if not wg["pending"]:
            if wg["resident"]:
                raise LowerError("WgmmaWait on products that were never committed")
            return
        # bounded wait for this commit's phase, then the accumulators back
        done, loop = k.label("wgw_done"), k.label("wgw")
        p = k.reg("pred")
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{wg['bar']}], {wg['ph']}")
        k(f"@{p} bra {done}")
        t0, t1 = k.reg("u64"), k.reg("u64")
        k(f"mov.u64 {t0}, %globaltimer")
        k.place(loop)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{wg['bar']}], {wg['ph']}, 100000")
        k(f"@{p} bra {done}")
        k(f"mov.u64 {t1}, %globaltimer")
        k(f"sub.u64 {t1}, {t1}, {t0}")
        k(f"setp.lt.u64 {p}, {t1}, {MBAR_WAIT_NS}")
        k(f"@{p} bra {loop}")
        old = k.reg("u32")
        k(f"atom.global.cas.b32 {old}, [emmy_err], 0, {ERR_MBAR_WAIT}")
        k.place(done)
        k(f"xor.b32 {wg['ph']}, {wg['ph']}, 1")
        k("tcgen05.fence::after_thread_sync")
        for name in sorted(wg["resident"]):
            regs = self.frags[name][2][0]
            n = 2 * len(regs)
            ta = k.reg("u32")
            k(f"add.u32 {ta}, {wg['tcol']}, {wg['offs'][name]}")
            k(f"add.u32 {ta}, {ta}, {wg['lane']}")
            k(f"tcgen05.ld.sync.aligned.16x256b.x{n // 8}.b32 {{{', '.join(regs)}}}, [{ta}]")
        k("tcgen05.wait::ld.sync.aligned")
        wg["resident"].clear()
        wg["pending"] = False


def emit_generic(spec: KernelSpec, checked: bool = False) -> Module:
    return Generic(spec, checked=checked).emit()
