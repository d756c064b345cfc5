"""Dense f32 matmul on the 5th-generation tensor cores (tcgen05 + TMEM + TMA).

IR family: m01 (``C = A.B`` with a cp.async ring) and m02 (split-K slices
accumulated with atomic writes into a zeroed C).  The IR's arithmetic is a
sum over K of ``multiply(b, a)`` in f32; on B200 it runs as **3xTF32**:
every operand x is split into ``hi = x & 0xffffe000`` (exactly representable
in TF32) and ``lo = x - hi`` (exact in f32), and the tile product is
``hi.hi + hi.lo + lo.hi`` accumulated in f32 in tensor memory -- about
2^-21 relative error per product, well inside the 1e-4 budget for fp32
contractions (the dropped ``lo.lo`` term is ~2^-22 relative).

Pre-passes write the TF32 hi/lo halves of A and of B (B transposed to
K-major) into a launcher-owned workspace.  Kernel (one persistent CTA per SM,
192 threads):

* warp 0, one lane -- TMA producer: per K block of 16, the A hi/lo boxes
  (128x16) and the B hi/lo boxes (BNx16), K-major with the 64-byte swizzle,
  into a 4-stage shared-memory ring, ``mbarrier`` complete_tx;
* warp 1 -- allocates 2 x BN TMEM columns (two accumulators) and issues, per
  8-deep K step, three ``tcgen05.mma.cta_group::1.kind::tf32`` (M=128,
  N=BN) reading smem matrix descriptors; ``tcgen05.commit`` frees the stage
  and, after the last K block, publishes the accumulator;
* warps 2-5 -- epilogue: ``tcgen05.ld.32x32b`` of the accumulator (each warp
  its 32-lane quadrant) 32 columns at a time, written into one of two
  shared-memory staging buffers (128-byte swizzle) and stored by one thread
  with a TMA tensor store (``cp.reduce.async.bulk.tensor .add`` for split-K
  into the launcher-zeroed C), then the accumulator is handed back --
  overlapping the next tile's main loop.  An output the 3xTF32 sum leaves
  infinite or NaN is recomputed there in plain f32 in K order, so
  infinities and NaNs come out as the IR's f32 arithmetic gives them
  (``_emit_nonfinite_fix``).

Every wait is an ``mbarrier.try_wait`` loop bounded by ``%globaltimer``; on
expiry the kernel raises a shared abort flag and writes ``emmy_err``, every
role leaves its loop, in-flight copies and MMAs are drained with bounded
waits, TMEM is freed and the kernel returns.

The tcgen05 path needs the launcher's plan: tensor maps filled in module
globals (the operand halves in the workspace, and C), ``emmy_plan`` set, 192
threads and the stated dynamic shared memory.  Any other launch (for
example meta.json's geometry) takes a SIMT path that computes each C element
as the IR does -- ``acc = acc + b*a`` in K order, rounded per op -- so the
PTX is correct under every launch.
"""

from __future__ import annotations

import math

from . import ir
from .analysis import NoMatch, flat_affine, numel
from .model import KernelSpec, dtype_info
from .ptx import Kernel, Module, Reg

PLAN_MAGIC = 0x454D4D59          # "EMMY"
ERR_WAIT_TIMEOUT = 0x201
WAIT_LIMIT_NS = 4_000_000_000    # 4 s: far above any legal wait in these kernels

BM, BK, STAGES = 128, 16, 4
THREADS = 192                    # warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
EPI_THREADS = 128
EPI_COLS = 32                    # C columns per epilogue chunk (128 bytes of f32)
EPI_BUF = BM * EPI_COLS * 4      # one staging buffer: 128 rows x 128 bytes, 128-byte swizzle
EPI_ISSUER = 64                  # thread that issues the C stores (warp 2, lane 0)
W_PROD, W_MMA = 0, 1


# A's TF32 hi part is A itself: a kind::tf32 MMA reads only the top 19 bits
# of each 32-bit operand, so it sees exactly x & 0xffffe000; the pre-pass
# then writes only A_lo (B must be transposed to K-major anyway).
RAW_A_HI = True


class MatmulPlan:
    pass


def match_matmul(spec: KernelSpec) -> MatmulPlan:
    body = spec.op.body
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        raise NoMatch("needs one Tile")
    tile = body[0]
    stmts = list(ir.walk(tile.body))
    inits = [s for s in stmts if isinstance(s, ir.Init)]
    copies = [s for s in stmts if isinstance(s, ir.CpAsyncCopy)]
    writes = [s for s in stmts if isinstance(s, ir.Write) and s.output in spec.args]
    if not inits or not copies or not writes:
        raise NoMatch("not the matmul shape (Init + cp.async + Write)")
    # innermost loop: loads from smem, multiply, Accum(add)
    loops = [s for s in stmts if isinstance(s, ir.Loop)]
    inner = None
    for lp in loops:
        if any(isinstance(x, ir.Accum) for x in lp.body):
            inner = lp
    if inner is None:
        raise NoMatch("no accumulation loop")
    kvar = inner.axis.name
    smem_names = {s.name for s in stmts if isinstance(s, ir.Smem)}
    loads = {s.names[0]: s for s in inner.body if isinstance(s, ir.Load)}
    a_smem = b_smem = None
    for ld in loads.values():
        if ld.input not in smem_names:
            raise NoMatch("inner loop reads global memory")
        last = ld.index[-1]
        if isinstance(last, ir.Var) and last.name == kvar:
            a_smem = ld.input
        elif isinstance(ld.index[0], ir.BinaryExpr) or isinstance(ld.index[0], ir.Var):
            b_smem = ld.input
    if a_smem is None or b_smem is None or a_smem == b_smem:
        raise NoMatch("cannot tell the A and B tiles apart")
    assigns = {s.name: s for s in inner.body if isinstance(s, ir.Assign)}
    accs = [s for s in inner.body if isinstance(s, ir.Accum)]
    for acc in accs:
        if acc.op.name != "add" or acc.base is not None:
            raise NoMatch("accumulation is not a plain sum")
        v = assigns.get(acc.value)
        if v is None or v.op.name != "multiply" or len(v.args) != 2:
            raise NoMatch("accumulated value is not a product")
        srcs = {loads[a].input for a in v.args if a in loads}
        if srcs != {a_smem, b_smem}:
            raise NoMatch("product is not of an A and a B element")
    src_of = {}
    for c in copies:
        src_of.setdefault(c.smem, set()).add(c.src)
    if len(src_of.get(a_smem, ())) != 1 or len(src_of.get(b_smem, ())) != 1:
        raise NoMatch("smem tiles fed by several buffers")
    a_buf, b_buf = next(iter(src_of[a_smem])), next(iter(src_of[b_smem]))
    outs = {w.output for w in writes}
    if len(outs) != 1:
        raise NoMatch("writes to several buffers")
    c_buf = outs.pop()
    atomic = {w.atomic for w in writes}
    if len(atomic) != 1:
        raise NoMatch("mixed atomic and plain writes")
    atomic = atomic.pop()
    for b in (a_buf, b_buf, c_buf):
        if spec.args[b].dtype != "f32" or len(spec.args[b].shape) != 2:
            raise NoMatch("matmul template is f32 2-D")
    m, k = spec.args[a_buf].shape
    k2, n = spec.args[b_buf].shape
    if k != k2 or tuple(spec.args[c_buf].shape) != (m, n):
        raise NoMatch("operand shapes do not chain")
    if atomic and c_buf not in spec.zero_outputs:
        raise NoMatch("atomic matmul without a zeroed output")
    # split-K slices: Tile axes that no write index uses
    used = set()
    for w in writes:
        for e in w.index:
            used |= set(e.free_vars)
    slices = 1
    if atomic:
        for axd in tile.axes:
            if axd.name not in used:
                slices *= int(axd.extent.as_static())
    plan = MatmulPlan()
    plan.a, plan.b, plan.c, plan.m, plan.n, plan.k = a_buf, b_buf, c_buf, m, n, k
    plan.atomic, plan.slices = atomic, max(1, slices)
    plan.bn = _choose_bn(m, n)
    plan.partial_n = bool(plan.bn) and n % plan.bn != 0
    slice_k = k // plan.slices if plan.slices and k % plan.slices == 0 else k
    # slices shorter than a K block are merged (same sum, other association)
    while plan.slices > 1 and (slice_k % BK or slice_k < 4 * BK):
        plan.slices //= 2
        slice_k = k // plan.slices
    if plan.bn and m % BM == 0 and k % BK == 0:
        plan.slices = _choose_slices(k, (m // BM) * -(-n // plan.bn), plan.slices,
                                     atomic=plan.atomic)
        slice_k = k // plan.slices
    plan.slice_k = slice_k
    plan.tc = (m % BM == 0 and plan.bn > 0 and k % 32 == 0 and slice_k % BK == 0
               and m * n < 2 ** 31 and m * k < 2 ** 31 and k * n < 2 ** 31)
    return plan


BN_RAGGED = (256, 224, 192, 160)   # widths a ragged N edge may use


def _choose_bn(m: int, n: int) -> int:
    """The C tile width (the MMA's N): 256 or 128 where it divides N; for
    other N that are multiples of 32 a full-rate width -- N itself up to
    256, else 256 -- with the N edge tile sticking out past N: its B rows
    load as zeros (the tensor map's bounds) and its C columns past N are
    not stored (every 32-column store chunk is wholly in or out).  Other N
    take the largest of 64, 32 that divides them.  Narrower widths chosen
    to fill the last wave of a few-tile product (224 for the 8-GPU row shard
    of 8192^3, 160 or 128 for the rect shards) measured no faster, or much
    slower, than 256 on B200, so the width is not chosen by wave count.
    ``EMMY_MATMUL_BN`` (read when the kernel is compiled) forces a width of
    ``BN_RAGGED`` or 128 for measurements."""
    import os
    forced = os.environ.get("EMMY_MATMUL_BN", "").strip()
    exact = next((bn for bn in (256, 128, 64, 32) if n % bn == 0), 0)
    if forced and n % 32 == 0 and int(forced) in BN_RAGGED + (128,):
        return int(forced)
    if exact >= 128 or n % 32:
        return exact
    if n <= 256:
        return n if n >= 128 else exact
    return 256


# K slices.  On B200 the kind::tf32 accumulation truncates each MMA's sum,
# so a C tile's error grows with the number of MMAs it accumulates.  Cutting
# K into slices of at most EMMY_MATMUL_MAX_SLICE_K (reduce-added into a
# launcher-cleared C with f32 TMA reduce-adds, rounded to nearest) keeps a
# K = 8192 product near a K = 1024 one.  Measured on B200, 8192^3: per-16-row
# max|err| / max|ref| 7.1e-5 unsliced, 1.7e-5 with 4 slices, 8.7e-6 with 8;
# but 4.18 ms unsliced against 4.79 and 5.10 ms.  Both are inside the
# 1e-4 contraction bound, so slicing is opt-in (environment variable, read
# when the kernel is compiled); the default favours speed.
MIN_SLICE_K = 256     # the shortest K range worth a unit of its own


def _max_slice_k() -> int:
    import os
    v = os.environ.get("EMMY_MATMUL_MAX_SLICE_K", "").strip()
    return int(v) if v else 0


def _wave_eff(units: int) -> float:
    """Fraction of SM slots busy over the waves ``units`` take on 148 SMs."""
    return units / (math.ceil(units / SM_COUNT) * SM_COUNT)


def _choose_slices(k: int, tiles: int, ir_slices: int, atomic: bool) -> int:
    """How many K slices the units of one C tile take.

    Atomic (split-K) IR: a divisor of its own slice count -- a CTA
    accumulates a group of the IR's slices in TMEM before its one add (the
    same sum, another association) -- the fewest that give every SM a unit
    (measured: more slices than that only add reduce-add traffic; at 256
    tiles, 2 slices took 0.088 ms against 0.074 unsliced).  Other IR: one
    slice, or with ``EMMY_MATMUL_MAX_SLICE_K`` set, the fewest slices no
    longer than it (C cleared by the launcher, slices reduce-added)."""
    maxk = _max_slice_k()
    cands = []
    s = 1
    limit = ir_slices if atomic else max(1, k // MIN_SLICE_K)
    while s <= limit:
        if (k % s == 0 and (k // s) % BK == 0 and k // s >= 4 * BK
                and (atomic or s == 1 or k // s >= MIN_SLICE_K)):
            cands.append(s)
        s *= 2
    if not cands:
        return ir_slices if atomic else 1
    if maxk:
        short = [c for c in cands if k // c <= maxk]
        cands = short or cands[-1:]
    if not atomic:
        return cands[0] if maxk else 1
    fill = [c for c in cands if tiles * c >= SM_COUNT]
    return fill[0] if fill else cands[-1]


# ---------------------------------------------------------------------------
# emission helpers
# ---------------------------------------------------------------------------


class _Ctx:
    """Bounded mbarrier waits.  ``limit``: a register holding the limit in
    ns (read from a module global the launcher may lower), or None for the
    fixed ``WAIT_LIMIT_NS``."""

    def __init__(self, k: Kernel, limit: str | None = None):
        self.k = k
        self.abort_label = None
        self.limit = limit if limit is not None else str(WAIT_LIMIT_NS)

    def wait(self, bar_addr: str, parity: str, abort_label: str, code: int = ERR_WAIT_TIMEOUT):
        """Bounded wait for the phase of parity ``parity`` of an mbarrier."""
        k = self.k
        p = k.reg("pred")
        t0, t1 = k.reg("u64"), k.reg("u64")
        ab = k.reg("u32")
        loop, done, to = k.label("wt"), k.label("wtok"), k.label("wtto")
        # fast path: a phase that is already complete costs one try_wait
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar_addr}], {parity}")
        k(f"@{p} bra {done}")
        k(f"mov.u64 {t0}, %globaltimer")
        k.place(loop)
        # the hint lets the warp sleep (up to SUSPEND_HINT_NS) until the phase
        # completes instead of spinning on issue slots its neighbours need
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {p}, [{bar_addr}], {parity}, {SUSPEND_HINT_NS}")
        k(f"@{p} bra {done}")
        k(f"ld.volatile.shared.u32 {ab}, [abort_flag]")
        k(f"setp.ne.u32 {p}, {ab}, 0")
        k(f"@{p} bra {abort_label}")
        k(f"mov.u64 {t1}, %globaltimer")
        k(f"sub.u64 {t1}, {t1}, {t0}")
        k(f"setp.gt.u64 {p}, {t1}, {self.limit}")
        k(f"@!{p} bra {loop}")
        k(f"st.volatile.shared.u32 [abort_flag], 1")
        k(f"st.global.u32 [emmy_err], {code}")
        k(f"bra.uni {abort_label}")
        k.place(done)


SUSPEND_HINT_NS = 100000
SM_COUNT = 148                   # B200 (sm_100a)


def _desc_const(lbo: int, sbo: int, layout: int) -> int:
    """Fixed fields of a tcgen05 shared-memory matrix descriptor: leading and
    stride byte offsets (16-byte units), version 1 (bit 46), swizzle
    layout (bits 61-63; 2 = 128B, 4 = 64B)."""
    return ((lbo >> 4) << 16) | ((sbo >> 4) << 32) | (1 << 46) | (layout << 61)


def _idesc_tf32(m: int, n: int) -> int:
    """Instruction descriptor of kind::tf32: D f32 (bits 4-5 = 1), A and B TF32
    (bits 7-9 and 10-12 = 2), A and B K-major (bits 15 and 16 = 0), N>>3 at
    bits 17-22, M>>4 at bits 24-28.  (On this B200 a TF32 B operand marked
    MN-major produced no result at all, so B is transposed once by the
    pre-pass and read K-major.)"""
    return (1 << 4) | (2 << 7) | (2 << 10) | ((n >> 3) << 17) | ((m >> 4) << 24)


def _decode_unit(k: Kernel, u: str, plan, mt: int, nt: int, group: int = 16):
    """unit -> (tile_m, tile_n, k_begin): split-minor, then tiles grouped by
    ``group`` tile rows so concurrent CTAs share A and B panels in L2."""
    S = plan.slices
    ks, t = k.reg("u32"), k.reg("u32")
    if S > 1:
        k(f"rem.u32 {ks}, {u}, {S}")
        k(f"div.u32 {t}, {u}, {S}")
    else:
        k(f"mov.u32 {ks}, 0")
        k(f"mov.u32 {t}, {u}")
    gsz = group * nt
    g, r, first, gm, tm, tn, kb = (k.reg("u32") for _ in range(7))
    k(f"div.u32 {g}, {t}, {gsz}")
    k(f"rem.u32 {r}, {t}, {gsz}")
    k(f"mul.lo.u32 {first}, {g}, {group}")
    k(f"sub.u32 {gm}, {mt}, {first}")
    k(f"min.u32 {gm}, {gm}, {group}")
    k(f"rem.u32 {tm}, {r}, {gm}")
    k(f"add.u32 {tm}, {tm}, {first}")
    k(f"div.u32 {tn}, {r}, {gm}")
    k(f"mul.lo.u32 {kb}, {ks}, {plan.slice_k}")
    return tm, tn, kb


def emit_matmul(spec: KernelSpec, plan: MatmulPlan) -> Module:
    params = [(f"p_{n}", ".u64") for n in spec.arg_order]
    k = Kernel(spec.entry, params)
    mod = Module(comment=f"emmy-b200 tcgen05 3xTF32 matmul template for {spec.entry}")
    mod.add_global(".visible .global .align 4 .u32 emmy_err;")
    mod.add_global(".visible .global .align 4 .u32 emmy_plan;")
    mod.add_global(".visible .global .align 8 .u64 emmy_ws;")
    for t in ("ahi", "alo", "bhi", "blo", "c"):
        mod.add_global(f".visible .global .align 64 .b8 tmap_{t}[128];")
    # the mbarrier wait limit, and a test hook: with emmy_test_stall set, the
    # MMA issuer first waits on a barrier nothing arrives on, so a test can
    # make the bounded wait run out (emmy_err 0x201) and check that the
    # kernel drains, frees TMEM and returns
    mod.add_global(f".visible .global .align 8 .u64 emmy_wait_ns = {WAIT_LIMIT_NS};")
    mod.add_global(".visible .global .align 4 .u32 emmy_test_stall;")
    M, N, K = plan.m, plan.n, plan.k
    BN = plan.bn or 32
    a_bytes = BM * BK * 4
    b_bytes = BN * BK * 4
    stage_bytes = 2 * (a_bytes + b_bytes)
    # the operand ring, then two staging buffers for the TMA stores of C
    dyn_smem = STAGES * stage_bytes + 2 * EPI_BUF + 1024
    # the two TMEM accumulators sit a power of two apart (BN rounded up), as
    # every other accumulator in these kernels does
    acc_stride = 1 << (BN - 1).bit_length()
    tcols = max(32, 2 * acc_stride)
    mt, nt = M // BM, (-(-N // BN) if plan.bn else 1)
    units = mt * nt * plan.slices
    kblocks = plan.slice_k // BK

    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    A, B, C = base[plan.a], base[plan.b], base[plan.c]
    tid, ntid = k.sreg("%tid.x"), k.sreg("%ntid.x")
    cta, ncta = k.sreg("%ctaid.x"), k.sreg("%nctaid.x")
    p = k.reg("pred")
    simt = k.label("simt")
    if plan.tc:
        mod.add_global(".extern .shared .align 1024 .b8 dsmem[];")
        flag, dsz = k.reg("u32"), k.reg("u32")
        k(f"ld.global.u32 {flag}, [emmy_plan]")
        k(f"setp.ne.u32 {p}, {flag}, {PLAN_MAGIC}")
        k(f"@{p} bra {simt}")
        k(f"setp.ne.u32 {p}, {ntid}, {THREADS}")
        k(f"@{p} bra {simt}")
        k(f"mov.u32 {dsz}, %dynamic_smem_size")
        k(f"setp.lt.u32 {p}, {dsz}, {dyn_smem}")
        k(f"@{p} bra {simt}")
        _emit_tc(k, plan, A, B, C, tid, cta, ncta, BN, acc_stride, a_bytes, b_bytes, stage_bytes,
                 tcols,
                 mt, nt, units, kblocks)
        k("ret")
    k.place(simt)
    _emit_simt(k, plan, A, B, C, tid, ntid, cta, ncta)
    mod.kernels.append(k)
    plan_d = {"entry": spec.entry, "kind": "matmul", "smem": 0, "block": 256,
              "grid_per_sm": 8, "grid_max": max(1, math.ceil(M * N / 256))}
    if plan.tc:
        mod.kernels.append(_emit_split_a(spec, plan))
        mod.kernels.append(_emit_split_b(spec, plan))
        o_alo, o_bhi = M * K * 4, 2 * M * K * 4
        o_blo = o_bhi + N * K * 4
        ws = o_blo + N * K * 4

        def tm(sym, off, rows, box_rows):
            return {"sym": sym, "buf": "@ws", "offset": off, "dtype": "f32", "dims": [K, rows],
                    "strides": [K * 4], "box": [BK, box_rows], "swizzle": 64}

        plan_d.update({
            "block": THREADS, "grid_per_sm": 1, "grid_max": units, "smem": dyn_smem,
            "workspace": {"sym": "emmy_ws", "bytes": ws},
            "pre": [
                {"entry": f"{spec.entry}_split_a", "block": 256, "grid_per_sm": 8,
                 "grid_max": max(1, math.ceil(M * K // 4 / 256))},
                {"entry": f"{spec.entry}_split_b", "block": 256, "grid_per_sm": 8,
                 "grid_max": (K // 32) * (N // 32)},
            ],
            "tmaps": [({"sym": "tmap_ahi", "buf": plan.a, "offset": 0, "dtype": "f32",
                        "dims": [K, M], "strides": [K * 4], "box": [BK, BM], "swizzle": 64}
                       if RAW_A_HI else tm("tmap_ahi", 0, M, BM)),
                      tm("tmap_alo", o_alo, M, BM),
                      tm("tmap_bhi", o_bhi, N, BN), tm("tmap_blo", o_blo, N, BN),
                      {"sym": "tmap_c", "buf": plan.c, "offset": 0, "dtype": "f32",
                       "dims": [N, M], "strides": [N * 4], "box": [EPI_COLS, BM],
                       "swizzle": 128}],
            "flags": [{"sym": "emmy_plan", "value": PLAN_MAGIC}],
            "flops": 2 * M * N * K, "tile": [BM, BN, BK], "stages": STAGES,
            "split_k": plan.slices,
        })
        if plan.slices == 1:
            # every C element is written once by a plain TMA store: C needs
            # no clearing before a launch even when the IR adds into it
            plan_d["overwrites"] = [plan.c]
        elif not plan.atomic:
            # K slices reduce-add into C: the launcher clears it first
            plan_d["zero"] = [plan.c]
    mod.plan = plan_d
    return mod


def _split_vec4(k: Kernel, x: list, hi: list, lo: list) -> None:
    for e in range(4):
        k(f"and.b32 {hi[e]}, {x[e]}, -8192")
        k(f"sub.rn.f32 {lo[e]}, {x[e]}, {hi[e]}")


def _emit_split_a(spec: KernelSpec, plan) -> Kernel:
    """A [M, K] -> A_hi, A_lo [M, K] in the workspace (elementwise)."""
    k = Kernel(f"{spec.entry}_split_a", [(f"p_{n}", ".u64") for n in spec.arg_order])
    A = k.param_ptr(f"p_{plan.a}")
    ws = k.reg("u64")
    k("ld.global.u64 {}, [emmy_ws]".format(ws))
    nvec = plan.m * plan.k // 4
    tid, ntid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ntid.x", "%ctaid.x", "%nctaid.x"))
    i, st = k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {i}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {st}, {ncta}, {ntid}")
    p = k.reg("pred")
    lp, end = k.label("sa"), k.label("saend")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {i}, {nvec}")
    k(f"@{p} bra {end}")
    a = k.addr(A, i, 16)
    x = k.regs("b32", 4)
    hi = k.regs("b32", 4)
    lo = k.regs("f32", 4)
    k(f"ld.global.nc.L1::no_allocate.v4.b32 {{{', '.join(x)}}}, [{a}]")
    _split_vec4(k, x, hi, lo)
    w = k.addr(ws, i, 16)
    if not RAW_A_HI:
        k(f"st.global.v4.b32 [{w}], {{{', '.join(hi)}}}")
    k(f"st.global.v4.f32 [{w}+{plan.m * plan.k * 4}], {{{', '.join(lo)}}}")
    k(f"add.u32 {i}, {i}, {st}")
    k(f"bra.uni {lp}")
    k.place(end)
    return k


def _emit_split_b(spec: KernelSpec, plan) -> Kernel:
    """B [K, N] -> B_hi^T, B_lo^T [N, K] in the workspace: 32x32 tiles through
    shared memory so both the reads (along N) and the writes (along K) are
    coalesced; 256 threads, 4 elements each."""
    k = Kernel(f"{spec.entry}_split_b", [(f"p_{n}", ".u64") for n in spec.arg_order])
    k.shared("\t.shared .align 4 .f32 tr_tile[1056];")   # 32 x 33
    M, N, K = plan.m, plan.n, plan.k
    B = k.param_ptr(f"p_{plan.b}")
    ws = k.reg("u64")
    k("ld.global.u64 {}, [emmy_ws]".format(ws))
    o_bhi = 2 * M * K * 4
    o_blo = o_bhi + N * K * 4
    tid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ctaid.x", "%nctaid.x"))
    tx, ty = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {tx}, {tid}, 31")
    k(f"shr.u32 {ty}, {tid}, 5")
    ntn = N // 32
    tiles = (K // 32) * ntn
    t = k.reg("u32")
    k(f"mov.u32 {t}, {cta}")
    p = k.reg("pred")
    lp, end = k.label("sb"), k.label("sbend")
    base_s = k.reg("u32")
    k(f"mov.u32 {base_s}, tr_tile")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {t}, {tiles}")
    k(f"@{p} bra {end}")
    tk, tn = k.reg("u32"), k.reg("u32")
    k(f"div.u32 {tk}, {t}, {ntn}")
    k(f"rem.u32 {tn}, {t}, {ntn}")
    for j in range(4):
        r, g, sa = k.reg("u32"), k.reg("u32"), k.reg("u32")
        k(f"add.u32 {r}, {ty}, {8 * j}")
        # global (tk*32 + r) * N + tn*32 + tx
        k(f"mad.lo.u32 {g}, {tk}, 32, {r}")
        k(f"mul.lo.u32 {g}, {g}, {N}")
        k(f"mad.lo.u32 {g}, {tn}, 32, {g}")
        k(f"add.u32 {g}, {g}, {tx}")
        a = k.addr(B, g, 4)
        v = k.reg("f32")
        k(f"ld.global.nc.f32 {v}, [{a}]")
        k(f"mad.lo.u32 {sa}, {r}, 33, {tx}")
        k(f"mad.lo.u32 {sa}, {sa}, 4, {base_s}")
        k(f"st.shared.f32 [{sa}], {v}")
    k("bar.sync 0")
    for j in range(4):
        r, g, sa = k.reg("u32"), k.reg("u32"), k.reg("u32")
        k(f"add.u32 {r}, {ty}, {8 * j}")
        # element B[tk*32 + tx][tn*32 + r] -> BT[(tn*32 + r) * K + tk*32 + tx]
        k(f"mad.lo.u32 {sa}, {tx}, 33, {r}")
        k(f"mad.lo.u32 {sa}, {sa}, 4, {base_s}")
        x, hi, lo = k.reg("b32"), k.reg("b32"), k.reg("f32")
        k(f"ld.shared.b32 {x}, [{sa}]")
        k(f"and.b32 {hi}, {x}, -8192")
        k(f"sub.rn.f32 {lo}, {x}, {hi}")
        k(f"mad.lo.u32 {g}, {tn}, 32, {r}")
        k(f"mul.lo.u32 {g}, {g}, {K}")
        k(f"mad.lo.u32 {g}, {tk}, 32, {g}")
        k(f"add.u32 {g}, {g}, {tx}")
        w = k.addr(ws, g, 4)
        k(f"st.global.b32 [{w}+{o_bhi}], {hi}")
        k(f"st.global.f32 [{w}+{o_blo}], {lo}")
    k("bar.sync 0")
    k(f"add.u32 {t}, {t}, {ncta}")
    k(f"bra.uni {lp}")
    k.place(end)
    return k


def _emit_simt(k: Kernel, plan, A, B, C, tid, ntid, cta, ncta):
    """Any launch: one C element per thread-iteration, acc = acc + b*a in K order."""
    M, N, K = plan.m, plan.n, plan.k
    gid, stride, i = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {gid}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {stride}, {ncta}, {ntid}")
    k(f"mov.u32 {i}, {gid}")
    p = k.reg("pred")
    lp, end = k.label("simt_el"), k.label("simt_end")
    mrow, ncol, kk = k.reg("u32"), k.reg("u32"), k.reg("u32")
    acc, av, bv, prod = (k.reg("f32") for _ in range(4))
    pa, pb, pc = k.reg("u64"), k.reg("u64"), k.reg("u64")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {i}, {M * N}")
    k(f"@{p} bra {end}")
    k(f"div.u32 {mrow}, {i}, {N}")
    k(f"rem.u32 {ncol}, {i}, {N}")
    k(f"mov.f32 {acc}, 0f00000000")
    k(f"mul.lo.u32 {kk}, {mrow}, {K}")
    k(f"mad.wide.u32 {pa}, {kk}, 4, {A}")
    k(f"mad.wide.u32 {pb}, {ncol}, 4, {B}")
    kl, kend = k.label("simt_k"), k.label("simt_kend")
    cnt = k.reg("u32")
    k(f"mov.u32 {cnt}, 0")
    k.place(kl)
    k(f"ld.global.nc.f32 {av}, [{pa}]")
    k(f"ld.global.nc.f32 {bv}, [{pb}]")
    k(f"mul.rn.f32 {prod}, {bv}, {av}")
    k(f"add.rn.f32 {acc}, {acc}, {prod}")
    k(f"add.u64 {pa}, {pa}, 4")
    k(f"add.u64 {pb}, {pb}, {N * 4}")
    k(f"add.u32 {cnt}, {cnt}, 1")
    k(f"setp.lt.u32 {p}, {cnt}, {K}")
    k(f"@{p} bra {kl}")
    k(f"mad.wide.u32 {pc}, {i}, 4, {C}")
    if plan.atomic:
        k(f"red.global.add.f32 [{pc}], {acc}")
    else:
        k(f"st.global.f32 [{pc}], {acc}")
    k(f"add.u32 {i}, {i}, {stride}")
    k(f"bra.uni {lp}")
    k.place(end)


def _any_nonfinite(k: Kernel, regs: list) -> Reg:
    """Predicate: some value in ``regs`` is an infinity or a NaN (all
    exponent bits set)."""
    m = k.reg("u32")
    k(f"mov.u32 {m}, 0")
    for r in regs:
        t = k.reg("u32")
        k(f"mov.b32 {t}, {r}")
        k(f"and.b32 {t}, {t}, 0x7F800000")
        k(f"max.u32 {m}, {m}, {t}")
    p = k.reg("pred")
    k(f"setp.eq.u32 {p}, {m}, 0x7F800000")
    return p


def _emit_nonfinite_fix(k: Kernel, plan, A, B, special, sbuf, rowq, r7, row0, col0, c0, kb):
    """Outputs the 3xTF32 product leaves non-finite are recomputed as the IR
    computes them: ``acc = acc + b*a`` over this unit's K range in K order,
    one rounding per op (``ptxgen/interp.py:196-206``, the m01/m02 loop).

    The split cannot carry an infinity: ``lo = inf - inf`` is NaN, and a
    zero ``lo`` meets an infinite ``hi`` in a cross term (``inf * 0``), so
    an output the f32 arithmetic makes +-inf would come out NaN.  Every
    output an infinite or NaN operand reaches is non-finite after the
    tensor-core pass (its ``hi.hi`` term already is), so recomputing exactly
    the non-finite outputs gives the f32 result wherever an operand is not
    finite; all-finite operands never take this path unless a sum
    overflows, and then the K-order sum is the IR's own.  A NaN
    accumulator stops the loop early (it stays NaN).

    The values sit in this thread's row of the staging buffer (16-byte
    chunk j/4 at (j/4) ^ (row % 8)); the fix rewrites them there before the
    buffer is stored."""
    N, K = plan.n, plan.k
    skip = k.label("nf_skip")
    k(f"@!{special} bra {skip}")
    j, off, t, v = k.reg("u32"), k.reg("u32"), k.reg("u32"), k.reg("b32")
    sa = k.reg("u32")
    p = k.reg("pred")
    row, col = k.reg("u32"), k.reg("u32")
    k(f"add.u32 {row}, {row0}, {rowq}")
    jl, jn = k.label("nf_j"), k.label("nf_next")
    k(f"mov.u32 {j}, 0")
    k.place(jl)
    k(f"shr.u32 {off}, {j}, 2")
    k(f"xor.b32 {off}, {off}, {r7}")
    k(f"shl.b32 {off}, {off}, 4")
    k(f"and.b32 {t}, {j}, 3")
    k(f"mad.lo.u32 {off}, {t}, 4, {off}")
    k(f"mad.lo.u32 {off}, {rowq}, {EPI_COLS * 4}, {off}")
    k(f"add.u32 {sa}, {sbuf}, {off}")
    k(f"ld.shared.b32 {v}, [{sa}]")
    k(f"and.b32 {t}, {v}, 0x7F800000")
    k(f"setp.ne.u32 {p}, {t}, 0x7F800000")
    k(f"@{p} bra {jn}")
    # C[row, col] over K rows kb .. kb + slice_k of this unit
    k(f"add.u32 {col}, {col0}, {c0}")
    k(f"add.u32 {col}, {col}, {j}")
    ia, ib = k.reg("u32"), k.reg("u32")
    pa, pb = k.reg("u64"), k.reg("u64")
    k(f"mad.lo.u32 {ia}, {row}, {K}, {kb}")
    k(f"mad.lo.u32 {ib}, {kb}, {N}, {col}")
    k(f"mad.wide.u32 {pa}, {ia}, 4, {A}")
    k(f"mad.wide.u32 {pb}, {ib}, 4, {B}")
    acc = k.reg("f32")
    k(f"mov.f32 {acc}, 0f00000000")
    cnt = k.reg("u32")
    k(f"mov.u32 {cnt}, 0")
    kl, kd = k.label("nf_k"), k.label("nf_kdone")
    k.place(kl)
    # four products per trip (slice_k is a multiple of 16), loads issued first
    av, bv = k.regs("f32", 4), k.regs("f32", 4)
    for e in range(4):
        k(f"ld.global.nc.f32 {av[e]}, [{pa}+{4 * e}]")
        k(f"ld.global.nc.f32 {bv[e]}, [{pb}+{4 * N * e}]")
    pr = k.reg("f32")
    for e in range(4):
        k(f"mul.rn.f32 {pr}, {bv[e]}, {av[e]}")
        k(f"add.rn.f32 {acc}, {acc}, {pr}")
    k(f"add.u64 {pa}, {pa}, 16")
    k(f"add.u64 {pb}, {pb}, {16 * N}")
    k(f"add.u32 {cnt}, {cnt}, 4")
    k(f"testp.notanumber.f32 {p}, {acc}")
    k(f"@{p} bra {kd}")
    k(f"setp.lt.u32 {p}, {cnt}, {plan.slice_k}")
    k(f"@{p} bra {kl}")
    k.place(kd)
    k(f"st.shared.f32 [{sa}], {acc}")
    k.place(jn)
    k(f"add.u32 {j}, {j}, 1")
    k(f"setp.lt.u32 {p}, {j}, {EPI_COLS}")
    k(f"@{p} bra {jl}")
    k.place(skip)


def _emit_tc(k: Kernel, plan, A, B, C, tid, cta, ncta, BN, acc_stride, a_bytes, b_bytes,
             stage_bytes, tcols, mt, nt, units, kblocks):
    M, N, K = plan.m, plan.n, plan.k
    wlim = k.reg("u64")
    k(f"ld.global.u64 {wlim}, [emmy_wait_ns]")
    cx = _Ctx(k, wlim)
    k.shared(f"\t.shared .align 8 .b64 bar_full[{STAGES}];")
    k.shared(f"\t.shared .align 8 .b64 bar_empty[{STAGES}];")
    k.shared("\t.shared .align 8 .b64 bar_tfull[2];")
    k.shared("\t.shared .align 8 .b64 bar_tempty[2];")
    k.shared("\t.shared .align 8 .b64 bar_drain;")
    k.shared("\t.shared .align 8 .b64 bar_stall;")
    k.shared("\t.shared .align 4 .u32 tmem_slot;")
    k.shared("\t.shared .align 4 .u32 abort_flag;")
    warp, lane = k.reg("u32"), k.reg("u32")
    k(f"shr.u32 {warp}, {tid}, 5")
    k(f"and.b32 {lane}, {tid}, 31")
    p, q = k.reg("pred"), k.reg("pred")
    ring = k.reg("u32")
    k(f"mov.u32 {ring}, dsmem")
    k(f"add.u32 {ring}, {ring}, 1023")
    k(f"and.b32 {ring}, {ring}, -1024")
    tmaps = {}
    for t in ("ahi", "alo", "bhi", "blo", "c"):
        r = k.reg("u64")
        k(f"mov.u64 {r}, tmap_{t}")
        k(f"cvta.global.u64 {r}, {r}")
        tmaps[t] = r

    def bar(name, idx):
        r = k.reg("u32")
        k(f"mov.u32 {r}, {name}")
        k(f"mad.lo.u32 {r}, {idx}, 8, {r}")
        return r

    # ---- set-up: barriers (thread 0), TMEM (warp 1) ----
    skip = k.label("noinit")
    k(f"setp.ne.u32 {p}, {tid}, 0")
    k(f"@{p} bra {skip}")
    for s_ in range(STAGES):
        k(f"mbarrier.init.shared::cta.b64 [bar_full+{8 * s_}], 1")
        k(f"mbarrier.init.shared::cta.b64 [bar_empty+{8 * s_}], 1")
    for a in range(2):
        k(f"mbarrier.init.shared::cta.b64 [bar_tfull+{8 * a}], 1")
        k(f"mbarrier.init.shared::cta.b64 [bar_tempty+{8 * a}], {EPI_THREADS}")
    k("mbarrier.init.shared::cta.b64 [bar_drain], 1")
    k("mbarrier.init.shared::cta.b64 [bar_stall], 1")
    k("st.shared.u32 [abort_flag], 0")
    for t in tmaps.values():
        k(f"prefetch.tensormap [{t}]")
    k("fence.mbarrier_init.release.cluster")
    k.place(skip)
    skip2 = k.label("noalloc")
    k(f"setp.ne.u32 {p}, {warp}, {W_MMA}")
    k(f"@{p} bra {skip2}")
    slot = k.reg("u32")
    k(f"mov.u32 {slot}, tmem_slot")
    k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], {tcols}")
    k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
    k.place(skip2)
    k("tcgen05.fence::before_thread_sync")
    k("barrier.sync 0")
    k("tcgen05.fence::after_thread_sync")
    tmem = k.reg("u32")
    k(f"ld.shared.u32 {tmem}, [tmem_slot]")

    teardown, abort_l = k.label("teardown"), k.label("abort")
    role_mma, role_epi = k.label("rmma"), k.label("repi")

    # ================= producer: warp 0, one lane =================
    k(f"setp.ne.u32 {p}, {warp}, {W_PROD}")
    k(f"@{p} bra {role_mma}")
    k(f"setp.ne.u32 {p}, {lane}, 0")
    k(f"@{p} bra {teardown}")
    it, u = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {it}, 0")
    k(f"mov.u32 {u}, {cta}")
    ul, ue = k.label("p_unit"), k.label("p_unitend")
    k.place(ul)
    k(f"setp.ge.u32 {p}, {u}, {units}")
    k(f"@{p} bra {ue}")
    tm, tn, kb0 = _decode_unit(k, u, plan, mt, nt)
    rowA, rowB = k.reg("u32"), k.reg("u32")
    k(f"mul.lo.u32 {rowA}, {tm}, {BM}")
    k(f"mul.lo.u32 {rowB}, {tn}, {BN}")
    kb = k.reg("u32")
    k(f"mov.u32 {kb}, 0")
    kl = k.label("p_kb")
    k.place(kl)
    s, ph, tmp = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"rem.u32 {s}, {it}, {STAGES}")
    k(f"div.u32 {ph}, {it}, {STAGES}")
    k(f"and.b32 {ph}, {ph}, 1")
    k(f"xor.b32 {tmp}, {ph}, 1")
    cx.wait(bar("bar_empty", s), tmp, abort_l)
    fb = bar("bar_full", s)
    k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {stage_bytes}")
    dst = k.reg("u32")
    k(f"mad.lo.u32 {dst}, {s}, {stage_bytes}, {ring}")
    kc = k.reg("u32")
    k(f"mad.lo.u32 {kc}, {kb}, {BK}, {kb0}")
    for name, off, row in (("ahi", 0, rowA), ("alo", a_bytes, rowA),
                           ("bhi", 2 * a_bytes, rowB), ("blo", 2 * a_bytes + b_bytes, rowB)):
        d2 = k.reg("u32")
        k(f"add.u32 {d2}, {dst}, {off}")
        k(f"cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
          f"[{d2}], [{tmaps[name]}, {{{kc}, {row}}}], [{fb}]")
    k(f"add.u32 {it}, {it}, 1")
    k(f"add.u32 {kb}, {kb}, 1")
    k(f"setp.lt.u32 {p}, {kb}, {kblocks}")
    k(f"@{p} bra {kl}")
    k(f"add.u32 {u}, {u}, {ncta}")
    k(f"bra.uni {ul}")
    k.place(ue)
    k(f"bra.uni {teardown}")

    # ================= MMA issuer: warp 1, one lane =================
    k.place(role_mma)
    k(f"setp.ne.u32 {p}, {warp}, {W_MMA}")
    k(f"@{p} bra {role_epi}")
    k(f"setp.ne.u32 {p}, {lane}, 0")
    k(f"@{p} bra {teardown}")
    stall, nostall = k.reg("u32"), k.label("nostall")
    k(f"ld.global.u32 {stall}, [emmy_test_stall]")
    k(f"setp.eq.u32 {p}, {stall}, 0")
    k(f"@{p} bra {nostall}")
    sb0 = k.reg("u32")
    k(f"mov.u32 {sb0}, bar_stall")
    cx.wait(sb0, "0", abort_l)
    k.place(nostall)
    kmaj = _desc_const(16, 512, 4)   # K-major, 64-byte swizzle, 8-row groups 512 B apart
    idr = k.reg("u32")
    k(f"mov.u32 {idr}, {_idesc_tf32(BM, BN)}")
    yes = k.reg("pred")
    k(f"setp.eq.u32 {yes}, 0, 0")
    it2, acc_it, u2 = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {it2}, 0")
    k(f"mov.u32 {acc_it}, 0")
    k(f"mov.u32 {u2}, {cta}")
    ml, me = k.label("m_unit"), k.label("m_unitend")
    k.place(ml)
    k(f"setp.ge.u32 {p}, {u2}, {units}")
    k(f"@{p} bra {me}")
    a_i, aph = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {a_i}, {acc_it}, 1")
    k(f"shr.u32 {aph}, {acc_it}, 1")
    k(f"and.b32 {aph}, {aph}, 1")
    k(f"xor.b32 {aph}, {aph}, 1")
    cx.wait(bar("bar_tempty", a_i), aph, abort_l)
    k("tcgen05.fence::after_thread_sync")
    dt = k.reg("u32")
    k(f"mad.lo.u32 {dt}, {a_i}, {acc_stride}, {tmem}")
    kb2 = k.reg("u32")
    k(f"mov.u32 {kb2}, 0")
    mkl = k.label("m_kb")
    k.place(mkl)
    s2, ph2 = k.reg("u32"), k.reg("u32")
    k(f"rem.u32 {s2}, {it2}, {STAGES}")
    k(f"div.u32 {ph2}, {it2}, {STAGES}")
    k(f"and.b32 {ph2}, {ph2}, 1")
    cx.wait(bar("bar_full", s2), ph2, abort_l)
    k("tcgen05.fence::after_thread_sync")
    sb = k.reg("u32")
    k(f"mad.lo.u32 {sb}, {s2}, {stage_bytes}, {ring}")
    first = k.reg("pred")
    k(f"setp.ne.u32 {first}, {kb2}, 0")
    for kk in range(BK // 8):
        d = {}
        for name, off in (("ahi", 0), ("alo", a_bytes), ("bhi", 2 * a_bytes),
                          ("blo", 2 * a_bytes + b_bytes)):
            ad, r = k.reg("u32"), k.reg("u64")
            k(f"add.u32 {ad}, {sb}, {off + kk * 32}")
            k(f"shr.u32 {ad}, {ad}, 4")
            k(f"and.b32 {ad}, {ad}, 16383")
            k(f"cvt.u64.u32 {r}, {ad}")
            k(f"or.b64 {r}, {r}, 0x{kmaj:016X}")
            d[name] = r
        acc = first if kk == 0 else yes
        k(f"tcgen05.mma.cta_group::1.kind::tf32 [{dt}], {d['ahi']}, {d['bhi']}, {idr}, {acc}")
        k(f"tcgen05.mma.cta_group::1.kind::tf32 [{dt}], {d['ahi']}, {d['blo']}, {idr}, {yes}")
        k(f"tcgen05.mma.cta_group::1.kind::tf32 [{dt}], {d['alo']}, {d['bhi']}, {idr}, {yes}")
    eb = bar("bar_empty", s2)
    k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{eb}]")
    k(f"add.u32 {it2}, {it2}, 1")
    k(f"add.u32 {kb2}, {kb2}, 1")
    k(f"setp.lt.u32 {p}, {kb2}, {kblocks}")
    k(f"@{p} bra {mkl}")
    tfb = bar("bar_tfull", a_i)
    k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{tfb}]")
    k(f"add.u32 {acc_it}, {acc_it}, 1")
    k(f"add.u32 {u2}, {u2}, {ncta}")
    k(f"bra.uni {ml}")
    k.place(me)
    k(f"bra.uni {teardown}")

    # ================= epilogue: warps 2-5 =================
    k.place(role_epi)
    quad, rowq, lane_off = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"and.b32 {quad}, {warp}, 3")
    k(f"mad.lo.u32 {rowq}, {quad}, 32, {lane}")
    k(f"mul.lo.u32 {lane_off}, {quad}, {32 << 16}")
    acc_e, u4 = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {acc_e}, 0")
    k(f"mov.u32 {u4}, {cta}")
    is_iss = k.reg("pred")
    k(f"setp.eq.u32 {is_iss}, {tid}, {EPI_ISSUER}")
    ec, epi_base = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {ec}, 0")
    k(f"add.u32 {epi_base}, {ring}, {STAGES * stage_bytes}")
    # this thread's row in a staging buffer: 16-byte chunk j at j ^ (row % 8)
    swz_off = []
    r7 = k.reg("u32")
    k(f"and.b32 {r7}, {rowq}, 7")
    for j in range(EPI_COLS // 4):
        o = k.reg("u32")
        k(f"xor.b32 {o}, {r7}, {j}")
        k(f"shl.b32 {o}, {o}, 4")
        k(f"mad.lo.u32 {o}, {rowq}, {EPI_COLS * 4}, {o}")
        swz_off.append(o)
    el, ee = k.label("e_unit"), k.label("e_unitend")
    k.place(el)
    k(f"setp.ge.u32 {p}, {u4}, {units}")
    k(f"@{p} bra {ee}")
    tm4, tn4, kb4 = _decode_unit(k, u4, plan, mt, nt)
    a4, aph4 = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {a4}, {acc_e}, 1")
    k(f"shr.u32 {aph4}, {acc_e}, 1")
    k(f"and.b32 {aph4}, {aph4}, 1")
    cx.wait(bar("bar_tfull", a4), aph4, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    col0 = k.reg("u32")
    k(f"mul.lo.u32 {col0}, {tn4}, {BN}")
    tbase = k.reg("u32")
    k(f"mad.lo.u32 {tbase}, {a4}, {acc_stride}, {tmem}")
    k(f"add.u32 {tbase}, {tbase}, {lane_off}")
    row0 = k.reg("u32")
    k(f"mul.lo.u32 {row0}, {tm4}, {BM}")
    # C leaves through shared memory: per 32 columns every thread writes its
    # accumulator row (128 bytes, 128-byte swizzle) into one of two staging
    # buffers and one thread issues a TMA tensor store of the 128 x 32 box,
    # so C is written in whole lines instead of one 16-byte piece per row per
    # store.  Split-K IR adds into a zeroed C: a TMA reduce-add while several
    # CTAs share a tile, a plain store once each tile's K slices are all
    # accumulated in one CTA (0 + x == x; only a -0.0 sum keeps its sign)
    for c in range(BN // EPI_COLS):
        regs = k.regs("f32", EPI_COLS)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {tbase}, {c * EPI_COLS}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{EPI_COLS}.b32 {{{', '.join(regs)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        special = _any_nonfinite(k, regs)
        inb = None
        if plan.partial_n:
            # a chunk past N (an edge tile's overhang) is neither fixed up
            # nor stored
            cc0, inb = k.reg("u32"), k.reg("pred")
            k(f"add.u32 {cc0}, {col0}, {c * EPI_COLS}")
            k(f"setp.lt.u32 {inb}, {cc0}, {N}")
            k(f"and.pred {special}, {special}, {inb}")
        # the buffer is free once the store that used it two chunks ago read it
        k(f"@{is_iss} cp.async.bulk.wait_group.read 1")
        k(f"bar.sync 1, {EPI_THREADS}")
        sbuf = k.reg("u32")
        k(f"and.b32 {sbuf}, {ec}, 1")
        k(f"mad.lo.u32 {sbuf}, {sbuf}, {EPI_BUF}, {epi_base}")
        for j in range(EPI_COLS // 4):
            sa = k.reg("u32")
            k(f"add.u32 {sa}, {sbuf}, {swz_off[j]}")
            k(f"st.shared.v4.f32 [{sa}], {{{', '.join(regs[4 * j:4 * j + 4])}}}")
        _emit_nonfinite_fix(k, plan, A, B, special, sbuf, rowq, r7, row0, col0, c * EPI_COLS,
                            kb4)
        k("fence.proxy.async.shared::cta")
        k(f"bar.sync 1, {EPI_THREADS}")
        cc = k.reg("u32")
        k(f"add.u32 {cc}, {col0}, {c * EPI_COLS}")
        st_p = is_iss
        if inb is not None:
            st_p = k.reg("pred")
            k(f"and.pred {st_p}, {is_iss}, {inb}")
        if plan.slices > 1:
            k(f"@{st_p} cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group "
              f"[{tmaps['c']}, {{{cc}, {row0}}}], [{sbuf}]")
        else:
            k(f"@{st_p} cp.async.bulk.tensor.2d.global.shared::cta.bulk_group "
              f"[{tmaps['c']}, {{{cc}, {row0}}}], [{sbuf}]")
        k(f"@{is_iss} cp.async.bulk.commit_group")
        k(f"add.u32 {ec}, {ec}, 1")
    k("tcgen05.fence::before_thread_sync")
    teb = bar("bar_tempty", a4)
    k(f"mbarrier.arrive.shared::cta.b64 _, [{teb}]")
    k(f"add.u32 {acc_e}, {acc_e}, 1")
    k(f"add.u32 {u4}, {u4}, {ncta}")
    k(f"bra.uni {el}")
    k.place(ee)
    k(f"bra.uni {teardown}")

    # ================= abort and teardown =================
    k.place(abort_l)
    k("st.volatile.shared.u32 [abort_flag], 1")
    k.place(teardown)
    # the C store issuer: every TMA store it issued has completed
    k(f"setp.ne.u32 {q}, {tid}, {EPI_ISSUER}")
    nw = k.label("nostorewait")
    k(f"@{q} bra {nw}")
    k("cp.async.bulk.wait_group 0")
    k.place(nw)
    k("barrier.sync 0")
    ab = k.reg("u32")
    k(f"ld.volatile.shared.u32 {ab}, [abort_flag]")
    drained = k.label("drained")
    k(f"setp.eq.u32 {p}, {ab}, 0")
    k(f"@{p} bra {drained}")
    k(f"setp.ne.u32 {q}, {tid}, 0")
    k(f"@{q} bra {drained}")
    # after an abort, let the producer's copies in flight land (bounded: 50 ms)
    t0, t1 = k.reg("u64"), k.reg("u64")
    lw = k.label("drain")
    k(f"mov.u64 {t0}, %globaltimer")
    k.place(lw)
    k(f"mov.u64 {t1}, %globaltimer")
    k(f"sub.u64 {t1}, {t1}, {t0}")
    k(f"setp.lt.u64 {p}, {t1}, 50000000")
    k(f"@{p} bra {lw}")
    k.place(drained)
    # MMA lane: every issued MMA has completed before TMEM is freed (bounded)
    k(f"setp.ne.u32 {q}, {tid}, {W_MMA * 32}")
    nd = k.label("nodrain")
    k(f"@{q} bra {nd}")
    k("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_drain]")
    pp2 = k.reg("pred")
    t2, t3 = k.reg("u64"), k.reg("u64")
    lw2, ld2 = k.label("mdrain"), k.label("mdraindone")
    k(f"mov.u64 {t2}, %globaltimer")
    k.place(lw2)
    k(f"mbarrier.try_wait.parity.shared::cta.b64 {pp2}, [bar_drain], 0")
    k(f"@{pp2} bra {ld2}")
    k(f"mov.u64 {t3}, %globaltimer")
    k(f"sub.u64 {t3}, {t3}, {t2}")
    k(f"setp.lt.u64 {pp2}, {t3}, 1000000000")
    k(f"@{pp2} bra {lw2}")
    k(f"st.global.u32 [emmy_err], {ERR_WAIT_TIMEOUT + 1}")
    k.place(ld2)
    k.place(nd)
    k("barrier.sync 0")
    fin = k.label("fin")
    k(f"setp.ne.u32 {p}, {warp}, {W_MMA}")
    k(f"@{p} bra {fin}")
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {tcols}")
    k.place(fin)
