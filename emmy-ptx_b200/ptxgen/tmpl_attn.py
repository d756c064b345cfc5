"""Fused online-softmax attention on tcgen05 (a01/a02 family, and [B,H,S,D]).

IR family: ``out[.., i, c] = sum_j softmax_j(q_i . k_j * (1/c0)) v[.., j, c]``
with the online-softmax update per key (``a02``: Loop over keys, inner Loop
over the head dimension, coupled max/sum Accums, final multiply by the
reciprocal of the sum).  K is given either transposed (``kt [D, S]``, the
shipped problems) or as ``k [.., S, D]``.

B200 kernel (one persistent CTA per SM, 352 threads -- 224 when shared memory
allows one softmax thread per row only; a unit is one batch*head and 128
query rows):

* the last warp -- TMA: the unit's Q tile once (bf16), then per key block the
  K block and the V^T block (all K-major, 128-byte swizzle) into as many
  stages as shared memory holds, with separate full/empty barriers for K and
  V;
* warp 0 -- issues ``S = Q . K^T`` into one of two TMEM S buffers as soon as
  the K block is in and the buffer is free (f32: Q from TMEM, two MMAs per
  K-step); warp 1 -- allocates TMEM and issues ``O += P . V^T`` with P read
  from TMEM once the softmax warps have written it (kind::tf32 in hi/lo
  passes for f32 data, kind::f16 on bf16 data).  Two issuing warps on two SM
  sub-partitions split the issue cost;
* warps 2-9 (2-5 when shared memory is short) -- one or two threads per
  query row (f32: first its Q row, split into TF32 hi/lo, into TMEM):
  ``tcgen05.ld`` of its S columns, row max (swapped with the partner thread),
  ``p = exp(s/c0 - m)``, running sum, P written over its S columns in TMEM as
  the A operand of the P . V MMA (hi/lo TF32 or packed bf16), rescale of its
  O columns in TMEM only when the row max grew by more than 8 (``m`` is
  otherwise kept, so ``p <= e^8``; the result is the same sum, only rounded
  differently), and at the end ``O / l`` to global memory.

A pre-pass writes the hi/lo TF32 halves of K (f32 only) and V^T (and K from
K^T when the IR gives K transposed) into a launcher-owned workspace.
Every wait is bounded by ``%globaltimer`` and reports through ``emmy_err``.

Any other launch -- meta.json's geometry, or shapes the tensor-core path
does not tile (S not a multiple of 128) -- takes a SIMT path that evaluates
each output element with the IR's own per-key statements.
"""

from __future__ import annotations

import math
import os

from . import ir
from .analysis import NoMatch, flat_affine, numel
from .lower import Lowerer, Val
from .model import KernelSpec, dtype_info
from .ptx import Kernel, Module, f32_hex
from .tmpl_mma import ERR_WAIT_TIMEOUT, PLAN_MAGIC, _Ctx, _desc_const


def _late_import():
    from . import tmpl_attn2h, tmpl_attn2q
    return tmpl_attn2q, tmpl_attn2h

LOG2E = 1.4426950408889634
SMEM_MAX = 232448            # shared memory per CTA, static + dynamic
XCH_STATIC = 4096            # static shared memory of the two-threads-per-row form
W_QK, W_PV = 0, 1           # S = Q.K^T issuer, O += P.V^T issuer (and TMEM owner)
BQ = 128
RESCALE_T = 8.0
SPLIT_O_DEFAULT = True


class AttnPlan:
    pass


def match_attention(spec: KernelSpec) -> AttnPlan:
    body = spec.op.body
    if len(body) != 1 or not isinstance(body[0], ir.Tile):
        raise NoMatch("needs one Tile")
    tile = body[0]
    stmts = list(ir.walk(tile.body))
    loops = [s for s in tile.body if isinstance(s, ir.Loop)]
    if len(loops) != 1:
        raise NoMatch("attention has one key loop at the top of the tile")
    kloop = loops[0]
    kvar = kloop.axis.name
    inner = [s for s in kloop.body if isinstance(s, ir.Loop)]
    if not inner:
        raise NoMatch("no dot-product loop")
    dvar = inner[0].axis.name
    ops_used = {s.op.name for s in stmts if isinstance(s, ir.Assign)}
    if not {"exp", "maximum", "reciprocal", "multiply"} <= ops_used:
        raise NoMatch("not an online softmax")
    loads = [s for s in stmts if isinstance(s, ir.Load)]
    writes = [s for s in stmts if isinstance(s, ir.Write)]
    if not writes or any(w.atomic for w in writes):
        raise NoMatch("attention writes plainly")
    out = {w.output for w in writes}
    if len(out) != 1:
        raise NoMatch("one output")
    out = out.pop()
    consts = [l for l in loads if numel(spec.args[l.input].shape) == 1]
    if len(consts) != 1:
        raise NoMatch("one scale constant")
    scale_buf = consts[0].input
    q_buf = k_buf = v_buf = None
    k_trans = False
    for ld in loads:
        if ld.input == scale_buf:
            continue
        names = [getattr(e, "name", None) for e in ld.index]
        if ld in inner[0].body or any(ld in lp.body for lp in inner):
            # dot-product operands: q[.., row, d] and k[.., j, d] or kt[d, j]
            if names[-2:] == [dvar, kvar]:
                k_buf, k_trans = ld.input, True
            elif names[-2:] == [kvar, dvar]:
                k_buf = ld.input
            elif names[-1] == dvar:
                q_buf = ld.input
        elif names and kvar in names:
            v_buf = ld.input
    if None in (q_buf, k_buf, v_buf):
        raise NoMatch("cannot identify q, k and v")
    qs, ks, vs, os_ = (tuple(spec.args[b].shape) for b in (q_buf, k_buf, v_buf, out))
    if len(qs) not in (2, 4) or qs != vs or qs != os_:
        raise NoMatch("q, v and out must share one [.., S, D] shape")
    s_len, d = qs[-2], qs[-1]
    if k_trans and ks != qs[:-2] + (d, s_len):
        raise NoMatch("kt shape")
    if not k_trans and ks != qs:
        raise NoMatch("k shape")
    dts = {spec.args[b].dtype for b in (q_buf, k_buf, v_buf, out)}
    if len(dts) != 1 or dts.pop() not in ("f32", "bf16"):
        raise NoMatch("attention template handles f32 or bf16 tensors")
    plan = AttnPlan()
    plan.q, plan.k, plan.v, plan.out, plan.scale = q_buf, k_buf, v_buf, out, scale_buf
    plan.k_trans = k_trans
    plan.bh = int(numel(qs[:-2])) if len(qs) == 4 else 1
    plan.s, plan.d = int(s_len), int(d)
    plan.dtype = spec.args[q_buf].dtype
    plan.e = 4 if plan.dtype == "f32" else 2
    plan.atom = 128 // plan.e                      # elements per 128-byte swizzle row
    plan.bkv = 32 if plan.dtype == "f32" else 128
    plan.passes = 3 if plan.dtype == "f32" else 1
    plan.tc = (plan.s % BQ == 0 and plan.s % plan.bkv == 0 and plan.d % plan.atom == 0
               and plan.d % 32 == 0 and 32 <= plan.d <= 256 and plan.s % 32 == 0
               and plan.bh * plan.s * plan.d < 2 ** 31)
    return plan


# ---------------------------------------------------------------------------
# kernel emission
# ---------------------------------------------------------------------------


def _idesc(kind: str, m: int, n: int) -> int:
    """kind::tf32 (formats 2) or kind::f16 with bf16 operands (formats 1); D f32,
    both operands K-major, N>>3 at bits 17-22, M>>4 at bits 24-28."""
    fmt = 2 if kind == "tf32" else 1
    return (1 << 4) | (fmt << 7) | (fmt << 10) | ((n >> 3) << 17) | ((m >> 4) << 24)


def _p_col(key: int, bkv: int, split: int, f32: bool) -> int:
    """TMEM column (from the S buffer's first) of P for key ``key`` of a key
    block: each softmax thread of a row writes P over its own ``bkv // split``
    score columns -- f32 one column per key, bf16 two keys per column in the
    first half of them."""
    if f32:
        return key
    hs = bkv // split
    return (key // hs) * hs + (key % hs) // 2


def _split_o_on() -> bool:
    v = os.environ.get("EMMY_ATTN_SPLIT_O")
    return SPLIT_O_DEFAULT if v is None else v not in ("0", "")


def _layout(plan):
    """Shared-memory regions (bytes) of one unit: Q (resident), ``kvst``
    stages of the K block and the V^T block, and P; each ``halves`` deep
    (hi, lo) for f32."""
    e, atom, bkv, d = plan.e, plan.atom, plan.bkv, plan.d
    halves = 2 if plan.dtype == "f32" else 1
    q_chunk = BQ * 128                 # one 128-byte-wide column chunk of 128 rows
    q_bytes = (d // atom) * q_chunk
    k_chunk = bkv * 128
    k_bytes = (d // atom) * k_chunk
    v_chunk = d * 128                  # V^T: d rows, one atom of keys wide
    v_bytes = max(1, bkv // atom) * v_chunk
    # (P is not staged here: it lives in TMEM over its own S columns)
    # f32 Q (TF32 hi/lo) lives in TMEM too when the columns allow, as the A
    # operand of S = Q . K^T: then shared memory holds only K/V stages
    s_cols = max(32, bkv * (2 if plan.dtype == "f32" else 1))
    q_tmem = plan.dtype == "f32" and 2 * s_cols + 3 * d <= 512
    base = 0 if q_tmem else halves * q_bytes
    per_stage = halves * (k_bytes + v_bytes)
    kvst = 1
    for cand in (3, 2):
        if base + cand * per_stage + 1024 + XCH_STATIC <= SMEM_MAX:
            kvst = cand
            break
    lay = {"q_tmem": q_tmem, "s_cols": s_cols}
    off = 0
    for h in range(0 if q_tmem else halves):
        lay[("q", h)] = off
        off += q_bytes
    for st in range(kvst):
        for name, size in (("k", k_bytes), ("v", v_bytes)):
            for h in range(halves):
                lay[(name, st, h)] = off
                off += size
    lay["total"] = off
    # two softmax threads per query row (warps 2-9) when the exchange slots
    # fit beside the dynamic layout, else one (warps 2-5)
    split = 2 if off + 1024 + XCH_STATIC <= SMEM_MAX else 1
    lay["split"] = split
    # split O (bf16): the row's two threads keep their own running max and
    # sum over their half of each key block and accumulate into their own O
    # (O_A: keys [0, BKV/2), O_B: the rest), merged once in the epilogue --
    # no per-block exchange of partial maxima.  TMEM: 2 S + 2 O columns.
    lay["split_o"] = (plan.dtype != "f32" and split == 2 and bkv // atom == 2
                      and 2 * s_cols + 2 * d <= 512 and _split_o_on())
    # warps 0-1 MMA issue, 2 .. 1+4*split softmax, then one TMA warp
    lay["threads"] = 96 + 128 * split
    lay["w_prod"] = 2 + 4 * split
    lay.update(q_bytes=q_bytes, k_bytes=k_bytes, v_bytes=v_bytes,
               q_chunk=q_chunk, k_chunk=k_chunk, v_chunk=v_chunk,
               halves=halves, kvst=kvst)
    return lay


def _tmap_names(plan, lay):
    names = ["kh", "kl", "vh", "vl"] if plan.dtype == "f32" else ["kh", "vh"]
    if not lay["q_tmem"]:
        names = (["qh", "ql"] if plan.dtype == "f32" else ["qh"]) + names
    return names


def emit_attention(spec: KernelSpec, plan: AttnPlan) -> Module:
    params = [(f"p_{n}", ".u64") for n in spec.arg_order]
    k = Kernel(spec.entry, params)
    mod = Module(comment=f"emmy-b200 tcgen05 attention template for {spec.entry}")
    mod.add_global(".visible .global .align 4 .u32 emmy_err;")
    mod.add_global(".visible .global .align 4 .u32 emmy_plan;")
    mod.add_global(".visible .global .align 8 .u64 emmy_ws;")
    lay = _layout(plan)
    tnames = _tmap_names(plan, lay)
    for t in tnames:
        mod.add_global(f".visible .global .align 64 .b8 tmap_{t}[128];")
    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    tid, ntid = k.sreg("%tid.x"), k.sreg("%ntid.x")
    cta, ncta = k.sreg("%ctaid.x"), k.sreg("%nctaid.x")
    p = k.reg("pred")
    simt = k.label("simt")
    # bf16 with D = 128: two query tiles per unit (tmpl_attn2q)
    # bf16 with D = 128: two query tiles per unit on 64-key blocks with two
    # S buffers per tile (tmpl_attn2h), else on 128-key blocks (tmpl_attn2q)
    tmpl_attn2q, tmpl_attn2h = _late_import()
    half = tmpl_attn2h.eligible(plan)
    two_q = half or tmpl_attn2q.eligible(plan)
    tq = tmpl_attn2h if half else tmpl_attn2q
    dyn = tq.SMEM_DYN if two_q else lay["total"] + 1024
    threads = tq.THREADS if two_q else lay["threads"]
    if plan.tc and dyn <= 232448 - 1024:
        mod.add_global(".extern .shared .align 1024 .b8 dsmem[];")
        flag, dsz = k.reg("u32"), k.reg("u32")
        k(f"ld.global.u32 {flag}, [emmy_plan]")
        k(f"setp.ne.u32 {p}, {flag}, {PLAN_MAGIC}")
        k(f"@{p} bra {simt}")
        k(f"setp.ne.u32 {p}, {ntid}, {threads}")
        k(f"@{p} bra {simt}")
        k(f"mov.u32 {dsz}, %dynamic_smem_size")
        k(f"setp.lt.u32 {p}, {dsz}, {dyn}")
        k(f"@{p} bra {simt}")
        if half:
            tmpl_attn2h.emit_tc2h(k, spec, plan, base, tid, cta, ncta)
        elif two_q:
            tmpl_attn2q.emit_tc2q(k, spec, plan, base, tid, cta, ncta)
        else:
            _emit_tc(k, spec, plan, lay, base, tid, cta, ncta)
        k("ret")
        tc_ok = True
    else:
        tc_ok = False
    k.place(simt)
    _emit_simt(k, spec, plan, base, tid, ntid, cta, ncta)
    mod.kernels.append(k)
    S, D, BH = plan.s, plan.d, plan.bh
    total = BH * S * D
    plan_d = {"entry": spec.entry, "kind": "attention", "smem": 0, "block": 128,
              "grid_per_sm": 16, "grid_max": max(1, math.ceil(total / 128)),
              "flops": 4 * BH * S * S * D}
    if tc_ok:
        plan.v_direct = half or (two_q and tmpl_attn2q.v_direct())
        plan.kv_box = tmpl_attn2h.BKV if half else plan.bkv
        pre, ws_bytes, tm = _emit_pre(mod, spec, plan, lay)
        plan_d.update({
            "block": threads, "grid_per_sm": 1,
            "grid_max": BH * (S // (2 * BQ if two_q else BQ)), "smem": dyn,
            "workspace": {"sym": "emmy_ws", "bytes": ws_bytes}, "pre": pre, "tmaps": tm,
            "flags": [{"sym": "emmy_plan", "value": PLAN_MAGIC}],
            "tile": [2 * BQ if two_q else BQ, plan.bkv, D], "passes": plan.passes,
            "schedule": ("two query tiles, 64-key blocks, two S buffers per tile" if half
                         else "two query tiles" if two_q else "one query tile"),
        })
    mod.plan = plan_d
    return mod


# ---------------------------------------------------------------------------
# pre-pass: operand preparation into the workspace
# ---------------------------------------------------------------------------


def _ws_layout(plan, lay):
    """Workspace regions (bytes): hi/lo of K ([BH, S, D]) and V^T ([BH, D, S])
    for f32 (and of Q when Q is not in TMEM); K (only when given transposed)
    and V^T for bf16."""
    n = plan.bh * plan.s * plan.d * plan.e
    off = {}
    cur = 0
    if plan.dtype == "f32":
        names = (["kh", "kl", "vh", "vl"] if lay["q_tmem"] else
                 ["qh", "ql", "kh", "kl", "vh", "vl"])
    else:
        # K only when given transposed; V^T unless P V reads V as stored
        names = (["kh"] if plan.k_trans else []) + (
            [] if getattr(plan, "v_direct", False) else ["vh"])
    for nm in names:
        off[nm] = cur
        cur += n
    return off, cur


def _emit_pre(mod: Module, spec: KernelSpec, plan, lay):
    off, total = _ws_layout(plan, lay)
    f32 = plan.dtype == "f32"
    pre = []
    S, D, BH = plan.s, plan.d, plan.bh
    if f32 and not lay["q_tmem"]:
        mod.kernels.append(_emit_split_copy(spec, plan, plan.q, off["qh"], off["ql"], "_pre_q"))
        pre.append({"entry": f"{spec.entry}_pre_q", "block": 256, "grid_per_sm": 8,
                    "grid_max": max(1, BH * S * D // 4 // 256)})
    if f32:
        if plan.k_trans:
            mod.kernels.append(_emit_transpose(spec, plan, plan.k, D, S, off["kh"],
                                               off["kl"], "_pre_k"))
            pre.append({"entry": f"{spec.entry}_pre_k", "block": 256, "grid_per_sm": 8,
                        "grid_max": BH * (D // 32) * (S // 32)})
        else:
            mod.kernels.append(_emit_split_copy(spec, plan, plan.k, None, off["kl"], "_pre_k"))
            pre.append({"entry": f"{spec.entry}_pre_k", "block": 256, "grid_per_sm": 8,
                        "grid_max": max(1, BH * S * D // 4 // 256)})
        mod.kernels.append(_emit_transpose(spec, plan, plan.v, S, D, off["vh"], off["vl"],
                                           "_pre_v"))
        pre.append({"entry": f"{spec.entry}_pre_v", "block": 256, "grid_per_sm": 8,
                    "grid_max": BH * (S // 32) * (D // 32)})
    else:
        if plan.k_trans:
            mod.kernels.append(_emit_transpose(spec, plan, plan.k, D, S, off["kh"], None,
                                               "_pre_k"))
            pre.append({"entry": f"{spec.entry}_pre_k", "block": 256, "grid_per_sm": 8,
                        "grid_max": BH * (D // 32) * (S // 32)})
        if not plan.v_direct:
            mod.kernels.append(_emit_transpose(spec, plan, plan.v, S, D, off["vh"], None,
                                               "_pre_v"))
            pre.append({"entry": f"{spec.entry}_pre_v", "block": 256, "grid_per_sm": 8,
                        "grid_max": BH * (S // 32) * (D // 32)})
    dt = "f32" if f32 else "bf16"
    e = plan.e
    atom = plan.atom

    def tmap(sym, buf, offset, inner, rows, box_rows):
        return {"sym": sym, "buf": buf, "offset": offset, "dtype": dt,
                "dims": [inner, rows, BH], "strides": [inner * e, inner * rows * e],
                "box": [atom, box_rows, 1], "swizzle": 128}

    tm = []
    if f32:
        if not lay["q_tmem"]:
            tm += [tmap("tmap_qh", "@ws", off["qh"], D, S, BQ),
                   tmap("tmap_ql", "@ws", off["ql"], D, S, BQ)]
        tm += [tmap("tmap_kh", "@ws" if plan.k_trans else plan.k,
                    off["kh"] if plan.k_trans else 0, D, S, plan.bkv),
               tmap("tmap_kl", "@ws", off["kl"], D, S, plan.bkv),
               tmap("tmap_vh", "@ws", off["vh"], S, D, D), tmap("tmap_vl", "@ws", off["vl"], S, D, D)]
    else:
        tm += [tmap("tmap_qh", plan.q, 0, D, S, BQ),
               (tmap("tmap_kh", "@ws", off["kh"], D, S, plan.kv_box) if plan.k_trans else
                tmap("tmap_kh", plan.k, 0, D, S, plan.kv_box)),
               (tmap("tmap_vh", plan.v, 0, D, S, plan.kv_box) if plan.v_direct else
                tmap("tmap_vh", "@ws", off["vh"], S, D, D))]
    return pre, max(total, 16), tm


def _emit_split_copy(spec, plan, buf, off_hi, off_lo, suffix) -> Kernel:
    """x -> (hi, lo) of the same shape (f32); with ``off_hi`` None only lo
    (the hi operand is then read from x itself: a kind::tf32 MMA sees only
    the top 19 bits of each 32-bit value, exactly x & 0xffffe000)."""
    k = Kernel(f"{spec.entry}{suffix}", [(f"p_{n}", ".u64") for n in spec.arg_order])
    X = k.param_ptr(f"p_{buf}")
    ws = k.reg("u64")
    k(f"ld.global.u64 {ws}, [emmy_ws]")
    nvec = plan.bh * plan.s * plan.d // 4
    tid, ntid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ntid.x", "%ctaid.x", "%nctaid.x"))
    i, st = k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {i}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {st}, {ncta}, {ntid}")
    p = k.reg("pred")
    lp, end = k.label("sc"), k.label("scend")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {i}, {nvec}")
    k(f"@{p} bra {end}")
    a = k.addr(X, i, 16)
    x, hi, lo = k.regs("b32", 4), k.regs("b32", 4), k.regs("f32", 4)
    k(f"ld.global.nc.L1::no_allocate.v4.b32 {{{', '.join(x)}}}, [{a}]")
    for e in range(4):
        k(f"and.b32 {hi[e]}, {x[e]}, -8192")
        k(f"sub.rn.f32 {lo[e]}, {x[e]}, {hi[e]}")
    w = k.addr(ws, i, 16)
    if off_hi is not None:
        k(f"st.global.v4.b32 [{w}+{off_hi}], {{{', '.join(hi)}}}")
    k(f"st.global.v4.f32 [{w}+{off_lo}], {{{', '.join(lo)}}}")
    k(f"add.u32 {i}, {i}, {st}")
    k(f"bra.uni {lp}")
    k.place(end)
    return k


def _emit_transpose(spec, plan, buf, rows, cols, off_hi, off_lo, suffix) -> Kernel:
    """Per batch*head: X [rows, cols] -> X^T [cols, rows] in the workspace, in
    32x32 tiles through shared memory; f32 writes hi and lo, bf16 copies."""
    k = Kernel(f"{spec.entry}{suffix}", [(f"p_{n}", ".u64") for n in spec.arg_order])
    f32 = plan.dtype == "f32"
    e = plan.e
    k.shared("\t.shared .align 4 .b32 tr_tile[1056];")
    X = k.param_ptr(f"p_{buf}")
    ws = k.reg("u64")
    k(f"ld.global.u64 {ws}, [emmy_ws]")
    tid, cta, ncta = (k.sreg(s) for s in ("%tid.x", "%ctaid.x", "%nctaid.x"))
    tx, ty = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {tx}, {tid}, 31")
    k(f"shr.u32 {ty}, {tid}, 5")
    tr, tc = rows // 32, cols // 32
    per_bh = tr * tc
    tiles = plan.bh * per_bh
    t = k.reg("u32")
    k(f"mov.u32 {t}, {cta}")
    p = k.reg("pred")
    lp, end = k.label("tp"), k.label("tpend")
    sbase = k.reg("u32")
    k(f"mov.u32 {sbase}, tr_tile")
    k.place(lp)
    k(f"setp.ge.u32 {p}, {t}, {tiles}")
    k(f"@{p} bra {end}")
    bh, rem, ti, tj = (k.reg("u32") for _ in range(4))
    k(f"div.u32 {bh}, {t}, {per_bh}")
    k(f"rem.u32 {rem}, {t}, {per_bh}")
    k(f"div.u32 {ti}, {rem}, {tc}")
    k(f"rem.u32 {tj}, {rem}, {tc}")
    mat = k.reg("u32")
    k(f"mul.lo.u32 {mat}, {bh}, {rows * cols}")
    for j in range(4):
        r, g, sa = k.reg("u32"), k.reg("u32"), k.reg("u32")
        k(f"add.u32 {r}, {ty}, {8 * j}")
        k(f"mad.lo.u32 {g}, {ti}, 32, {r}")
        k(f"mul.lo.u32 {g}, {g}, {cols}")
        k(f"mad.lo.u32 {g}, {tj}, 32, {g}")
        k(f"add.u32 {g}, {g}, {tx}")
        k(f"add.u32 {g}, {g}, {mat}")
        a = k.addr(X, g, e)
        v = k.reg("b32")
        if f32:
            k(f"ld.global.nc.b32 {v}, [{a}]")
        else:
            h = k.reg("b16")
            k(f"ld.global.nc.b16 {h}, [{a}]")
            k(f"cvt.u32.u16 {v}, {h}")
        k(f"mad.lo.u32 {sa}, {r}, 33, {tx}")
        k(f"mad.lo.u32 {sa}, {sa}, 4, {sbase}")
        k(f"st.shared.b32 [{sa}], {v}")
    k("bar.sync 0")
    for j in range(4):
        r, g, sa = k.reg("u32"), k.reg("u32"), k.reg("u32")
        k(f"add.u32 {r}, {ty}, {8 * j}")
        k(f"mad.lo.u32 {sa}, {tx}, 33, {r}")
        k(f"mad.lo.u32 {sa}, {sa}, 4, {sbase}")
        x = k.reg("b32")
        k(f"ld.shared.b32 {x}, [{sa}]")
        # X[ti*32 + tx][tj*32 + r] -> XT[(tj*32 + r) * rows + ti*32 + tx]
        k(f"mad.lo.u32 {g}, {tj}, 32, {r}")
        k(f"mul.lo.u32 {g}, {g}, {rows}")
        k(f"mad.lo.u32 {g}, {ti}, 32, {g}")
        k(f"add.u32 {g}, {g}, {tx}")
        k(f"add.u32 {g}, {g}, {mat}")
        w = k.addr(ws, g, e)
        if f32:
            hi, lo = k.reg("b32"), k.reg("f32")
            k(f"and.b32 {hi}, {x}, -8192")
            k(f"sub.rn.f32 {lo}, {x}, {hi}")
            k(f"st.global.b32 [{w}+{off_hi}], {hi}")
            k(f"st.global.f32 [{w}+{off_lo}], {lo}")
        else:
            h = k.reg("b16")
            k(f"cvt.u16.u32 {h}, {x}")
            k(f"st.global.b16 [{w}+{off_hi}], {h}")
    k("bar.sync 0")
    k(f"add.u32 {t}, {t}, {ncta}")
    k(f"bra.uni {lp}")
    k.place(end)
    return k


# ---------------------------------------------------------------------------
# SIMT path: the IR's per-key statements for each output element
# ---------------------------------------------------------------------------


def _emit_simt(k: Kernel, spec, plan, base, tid, ntid, cta, ncta):
    """out[bh, i, c] with acc0 = sum_d k*q (IR order), x = acc0 * (1/c0), then
    gn = max(m, x); alpha = exp(m - gn); beta = exp(x - gn); l = l*alpha +
    1*beta; o = o*alpha + v*beta; m = max(m, x); out = o * (1/l)."""
    lo = Lowerer(k)
    S, D, BH = plan.s, plan.d, plan.bh
    f32 = plan.dtype == "f32"
    e = plan.e
    Q, K_, V, O = base[plan.q], base[plan.k], base[plan.v], base[plan.out]
    cr = k.reg("f32")
    k(f"ld.global.nc.f32 {cr}, [{base[plan.scale]}]")
    v1 = k.reg("f32")
    k(f"rcp.rn.f32 {v1}, {cr}")
    gid, stride = k.reg("u32"), k.reg("u32")
    k(f"mad.lo.u32 {gid}, {cta}, {ntid}, {tid}")
    k(f"mul.lo.u32 {stride}, {ncta}, {ntid}")
    idx = k.reg("u32")
    k(f"mov.u32 {idx}, {gid}")
    p = k.reg("pred")
    lp, end = k.label("at"), k.label("atend")

    def ld(addr):
        r = k.reg("f32")
        if f32:
            k(f"ld.global.nc.f32 {r}, [{addr}]")
        else:
            h = k.reg("b16")
            k(f"ld.global.nc.b16 {h}, [{addr}]")
            k(f"cvt.f32.bf16 {r}, {h}")
        return r

    k.place(lp)
    k(f"setp.ge.u32 {p}, {idx}, {BH * S * D}")
    k(f"@{p} bra {end}")
    bh, rem, i, c = (k.reg("u32") for _ in range(4))
    k(f"div.u32 {bh}, {idx}, {S * D}")
    k(f"rem.u32 {rem}, {idx}, {S * D}")
    k(f"div.u32 {i}, {rem}, {D}")
    k(f"rem.u32 {c}, {rem}, {D}")
    m, l, o = k.reg("f32"), k.reg("f32"), k.reg("f32")
    k(f"mov.f32 {m}, {f32_hex(-1e30)}")
    k(f"mov.f32 {l}, 0f00000000")
    k(f"mov.f32 {o}, 0f00000000")
    qrow = k.reg("u32")
    k(f"mad.lo.u32 {qrow}, {bh}, {S}, {i}")
    k(f"mul.lo.u32 {qrow}, {qrow}, {D}")
    j = k.reg("u32")
    k(f"mov.u32 {j}, 0")
    jl = k.label("atj")
    k.place(jl)
    acc = k.reg("f32")
    k(f"mov.f32 {acc}, 0f00000000")
    dd = k.reg("u32")
    k(f"mov.u32 {dd}, 0")
    dl = k.label("atd")
    k.place(dl)
    qa, ka = k.reg("u32"), k.reg("u32")
    k(f"add.u32 {qa}, {qrow}, {dd}")
    if plan.k_trans:   # kt[bh, d, j]
        k(f"mad.lo.u32 {ka}, {bh}, {D}, {dd}")
        k(f"mul.lo.u32 {ka}, {ka}, {S}")
        k(f"add.u32 {ka}, {ka}, {j}")
    else:              # k[bh, j, d]
        k(f"mad.lo.u32 {ka}, {bh}, {S}, {j}")
        k(f"mul.lo.u32 {ka}, {ka}, {D}")
        k(f"add.u32 {ka}, {ka}, {dd}")
    qv = ld(k.addr(Q, qa, e))
    kv = ld(k.addr(K_, ka, e))
    pr = k.reg("f32")
    k(f"mul.rn.f32 {pr}, {kv}, {qv}")
    k(f"add.rn.f32 {acc}, {acc}, {pr}")
    k(f"add.u32 {dd}, {dd}, 1")
    k(f"setp.lt.u32 {p}, {dd}, {D}")
    k(f"@{p} bra {dl}")
    x, gn, dg, al, be, t1, t2 = (k.reg("f32") for _ in range(7))
    k(f"mul.rn.f32 {x}, {acc}, {v1}")
    k(f"max.f32 {gn}, {m}, {x}")
    k(f"sub.rn.f32 {dg}, {m}, {gn}")
    k(f"mov.f32 {al}, {lo.exp_f32(dg)}")
    k(f"sub.rn.f32 {dg}, {x}, {gn}")
    k(f"mov.f32 {be}, {lo.exp_f32(dg)}")
    k(f"mul.rn.f32 {t1}, {l}, {al}")
    k(f"mul.rn.f32 {t2}, 0f3F800000, {be}")
    k(f"add.rn.f32 {l}, {t1}, {t2}")
    va = k.reg("u32")
    k(f"mad.lo.u32 {va}, {bh}, {S}, {j}")
    k(f"mad.lo.u32 {va}, {va}, {D}, {c}")
    vv = ld(k.addr(V, va, e))
    k(f"mul.rn.f32 {t1}, {o}, {al}")
    k(f"mul.rn.f32 {t2}, {vv}, {be}")
    k(f"add.rn.f32 {o}, {t1}, {t2}")
    k(f"max.f32 {m}, {m}, {x}")
    k(f"add.u32 {j}, {j}, 1")
    k(f"setp.lt.u32 {p}, {j}, {S}")
    k(f"@{p} bra {jl}")
    r9, res = k.reg("f32"), k.reg("f32")
    k(f"rcp.rn.f32 {r9}, {l}")
    k(f"mul.rn.f32 {res}, {o}, {r9}")
    oa = k.addr(O, idx, e)
    if f32:
        k(f"st.global.f32 [{oa}], {res}")
    else:
        h = k.reg("b16")
        k(f"cvt.rn.bf16.f32 {h}, {res}")
        k(f"st.global.b16 [{oa}], {h}")
    k(f"add.u32 {idx}, {idx}, {stride}")
    k(f"bra.uni {lp}")
    k.place(end)


# ---------------------------------------------------------------------------
# tensor-core path
# ---------------------------------------------------------------------------

# 2^f on [-1/2, 1/2]: degree-3 minimax polynomial (relative error), fitted by
# a Remez exchange in f64 and rounded to f32; evaluated by Horner in f32 its
# maximum relative error is 7.5e-5, below half an ulp of bf16 (2^-9).
EXP2_POLY = (0.9999280571937561, 0.6932609677314758, 0.2426111251115799,
             0.0551716685295105)
# pairs out of every four on the polynomial, measured on B200 for bf16
# [16,32,4096,128] with split O (two passes each): 1 -> 4.09-4.15 ms,
# 2 -> 4.21-4.37, 3 -> 4.42-4.70 (one shared O: 0 -> 4.40-4.43, 1 -> 4.39,
# 2 -> 4.33, 3 -> 4.79-4.84, 4 -> 5.15-5.21)
EXP_POLY_DEFAULT = 1


def _exp_poly_share(default: int = EXP_POLY_DEFAULT) -> int:
    """Element pairs out of every four whose exp2 runs on the FMA pipe
    (polynomial) instead of the MUFU (``ex2.approx``); bf16 P only.
    ``EMMY_ATTN_EXP_POLY`` overrides the kernel's default."""
    v = os.environ.get("EMMY_ATTN_EXP_POLY")
    return max(0, min(4, int(v))) if v else default


def _pair_const(v: float) -> str:
    b = int(f32_hex(v)[2:], 16)
    return f"0x{(b << 32) | b:016X}"


def _exp2_poly_consts(k: Kernel):
    """Packed (x2) registers: the 1.5 * 2^23 shift and the coefficients."""
    regs = []
    for v in (12582912.0,) + EXP2_POLY:
        r = k.reg("b64")
        k(f"mov.b64 {r}, {_pair_const(v)}")
        regs.append(r)
    return regs


def _exp2_poly_pair(k: Kernel, pr, consts):
    """exp2 of the two f32 lanes of ``pr`` (each <= 8) on the FMA pipe:
    x = max(x, -125); x = j + f with j = rint(x) from the 1.5 * 2^23 shift
    (the low bits of the shifted value hold j), 2^f by the polynomial, and
    j added to the exponent field with one integer multiply-add
    (``j << 23`` == ``bits(x + 1.5 * 2^23) * 2^23`` modulo 2^32)."""
    a, b = k.reg("b32"), k.reg("b32")
    k(f"mov.b64 {{{a}, {b}}}, {pr}")
    k(f"max.f32 {a}, {a}, {f32_hex(-125.0)}")
    k(f"max.f32 {b}, {b}, {f32_hex(-125.0)}")
    x, tt, jf, f, q = (k.reg("b64") for _ in range(5))
    k(f"mov.b64 {x}, {{{a}, {b}}}")
    magic, c0, c1, c2, c3 = consts
    k(f"add.rn.f32x2 {tt}, {x}, {magic}")
    k(f"sub.rn.f32x2 {jf}, {tt}, {magic}")
    k(f"sub.rn.f32x2 {f}, {x}, {jf}")
    k(f"fma.rn.f32x2 {q}, {f}, {c3}, {c2}")
    k(f"fma.rn.f32x2 {q}, {q}, {f}, {c1}")
    k(f"fma.rn.f32x2 {q}, {q}, {f}, {c0}")
    t0, t1, q0, q1, r0, r1 = k.regs("b32", 6)
    k(f"mov.b64 {{{t0}, {t1}}}, {tt}")
    k(f"mov.b64 {{{q0}, {q1}}}, {q}")
    k(f"mad.lo.s32 {r0}, {t0}, 8388608, {q0}")
    k(f"mad.lo.s32 {r1}, {t1}, 8388608, {q1}")
    return r0, r1



def _emit_tc(k: Kernel, spec, plan, lay, base, tid, cta, ncta):
    S, D, BH, BKV = plan.s, plan.d, plan.bh, plan.bkv
    f32 = plan.dtype == "f32"
    e, atom, passes = plan.e, plan.atom, plan.passes
    halves = lay["halves"]
    kind = "tf32" if f32 else "f16"
    nkv = S // BKV
    qblocks = S // BQ
    units = BH * qblocks
    kvst = lay["kvst"]
    stage_k = lay[("k", 1, 0)] - lay[("k", 0, 0)] if kvst > 1 else 0

    def k_addr(h, c):
        """Byte offset (in stage 0) of column chunk ``c`` of K half ``h``.  For
        f32 each chunk holds the hi rows then the lo rows, so one MMA with
        N = 2 * BKV reads [K_hi; K_lo] as a single B operand."""
        if f32:
            return lay[("k", 0, 0)] + c * 2 * lay["k_chunk"] + h * lay["k_chunk"]
        return lay[("k", 0, 0)] + c * lay["k_chunk"]
    cx = _Ctx(k)
    for nm in ("q_full", "q_empty", "pv_done", "o_full", "drain", "drain_qk"):
        k.shared(f"\t.shared .align 8 .b64 bar_{nm};")
    for nm, cnt in (("k_full", kvst), ("k_empty", kvst), ("v_full", kvst), ("v_empty", kvst),
                    ("s_full", 2), ("s_free", 2), ("p_full", 2)):
        k.shared(f"\t.shared .align 8 .b64 bar_{nm}[{cnt}];")
    k.shared("\t.shared .align 4 .u32 tmem_slot;")
    k.shared("\t.shared .align 4 .u32 abort_flag;")
    # TMEM columns: two S buffers (the MMA warp fills one while the softmax
    # warps read the other), O, then (f32 with q_tmem) Q hi and Q lo.  An S
    # buffer holds BKV f32 score columns; for f32 also the Q_hi.K_lo partial
    # beside them, later overwritten by P hi and P lo.
    q_tmem = lay["q_tmem"]
    split_o = lay["split_o"]
    s_cols = lay["s_cols"]
    o_col = 2 * s_cols
    q_col = o_col + (2 * D if split_o else D)     # split O: O_A then O_B
    tcols = 1 << (q_col + (2 * D if q_tmem else 0) - 1).bit_length()
    assert tcols <= 512
    warp, lane = k.reg("u32"), k.reg("u32")
    k(f"shr.u32 {warp}, {tid}, 5")
    k(f"and.b32 {lane}, {tid}, 31")
    p, q = k.reg("pred"), k.reg("pred")
    ring = k.reg("u32")
    k(f"mov.u32 {ring}, dsmem")
    k(f"add.u32 {ring}, {ring}, 1023")
    k(f"and.b32 {ring}, {ring}, -1024")
    tm = {}
    for t in _tmap_names(plan, lay):
        r = k.reg("u64")
        k(f"mov.u64 {r}, tmap_{t}")
        k(f"cvta.global.u64 {r}, {r}")
        tm[t] = r

    skip = k.label("noinit")
    k(f"setp.ne.u32 {p}, {tid}, 0")
    k(f"@{p} bra {skip}")
    split = lay["split"]
    # q_full: one TMA arrival, or every softmax thread once its Q row is in TMEM
    # Each barrier a role may wait on after skipping phases is either per
    # S buffer (p_full: the softmax may run a block ahead of the MMA warp's
    # wait) or per unit (o_full: the epilogue's wait for the unit's last
    # P . V), so no waiter is ever two phases behind its barrier.
    for nm, cnt in (("q_full", 128 * split if q_tmem else 1), ("q_empty", 1),
                    ("pv_done", 1), ("o_full", 1), ("drain", 1), ("drain_qk", 1)):
        k(f"mbarrier.init.shared::cta.b64 [bar_{nm}], {cnt}")
    for nm, n, cnt in (("k_full", kvst, 1), ("k_empty", kvst, 1), ("v_full", kvst, 1),
                       ("v_empty", kvst, 1), ("s_full", 2, 1), ("s_free", 2, 1),
                       ("p_full", 2, 128 * split)):
        for i in range(n):
            k(f"mbarrier.init.shared::cta.b64 [bar_{nm}+{8 * i}], {cnt}")
    k("st.shared.u32 [abort_flag], 0")
    for r in tm.values():
        k(f"prefetch.tensormap [{r}]")
    k("fence.mbarrier_init.release.cluster")
    k.place(skip)
    skip2 = k.label("noalloc")
    k(f"setp.ne.u32 {p}, {warp}, {W_PV}")
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
    role_qk, role_pv, role_sm = k.label("rqk"), k.label("rpv"), k.label("rsm")
    w_prod = lay["w_prod"]

    def unit_coords(u):
        bh, qb = k.reg("u32"), k.reg("u32")
        k(f"div.u32 {bh}, {u}, {qblocks}")
        k(f"rem.u32 {qb}, {u}, {qblocks}")
        return bh, qb

    def stage_of(g):
        """(stage index, parity of its full phase) of global key block ``g``:
        g % kvst and (g / kvst) & 1."""
        st, ph = k.reg("u32"), k.reg("u32")
        if kvst == 1:
            k(f"mov.u32 {st}, 0")
            k(f"and.b32 {ph}, {g}, 1")
        else:
            k(f"rem.u32 {st}, {g}, {kvst}")
            k(f"div.u32 {ph}, {g}, {kvst}")
            k(f"and.b32 {ph}, {ph}, 1")
        return st, ph

    def bar_at(name, idx):
        r = k.reg("u32")
        k(f"mov.u32 {r}, bar_{name}")
        k(f"mad.lo.u32 {r}, {idx}, 8, {r}")
        return r

    def flip(ph):
        r = k.reg("u32")
        k(f"xor.b32 {r}, {ph}, 1")
        return r

    # ================= producer =================
    k(f"setp.ne.u32 {p}, {warp}, {w_prod}")
    k(f"@{p} bra {role_qk}")
    # the whole warp runs the loop (converged, so its addresses stay
    # warp-uniform); one elected lane issues the copies
    pe = k.reg("pred")
    k(f"elect.sync _|{pe}, -1")
    uit, g, u = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit}, 0")
    k(f"mov.u32 {g}, 0")
    k(f"mov.u32 {u}, {cta}")
    ul, ue = k.label("p_unit"), k.label("p_unitend")
    k.place(ul)
    k(f"setp.ge.u32 {p}, {u}, {units}")
    k(f"@{p} bra {ue}")
    bh, qb = unit_coords(u)
    qrow = k.reg("u32")
    k(f"mul.lo.u32 {qrow}, {qb}, {BQ}")
    if not q_tmem:
        ph = k.reg("u32")
        k(f"and.b32 {ph}, {uit}, 1")
        k(f"xor.b32 {ph}, {ph}, 1")
        cx.wait("bar_q_empty", ph, abort_l)
        qbytes = lay["q_bytes"] * halves
        k(f"@{pe} mbarrier.arrive.expect_tx.shared::cta.b64 _, [bar_q_full], {qbytes}")
        for h in range(halves):
            for c in range(D // atom):
                dst, cc = k.reg("u32"), k.reg("u32")
                k(f"add.u32 {dst}, {ring}, {lay[('q', h)] + c * lay['q_chunk']}")
                k(f"mov.u32 {cc}, {c * atom}")
                k(f"@{pe} cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
                  f"[{dst}], [{tm['qh' if h == 0 else 'ql']}, {{{cc}, {qrow}, {bh}}}], [bar_q_full]")
    j = k.reg("u32")
    k(f"mov.u32 {j}, 0")
    jl = k.label("p_kv")
    k.place(jl)
    st, phf = stage_of(g)
    phe = flip(phf)
    soff = k.reg("u32")
    k(f"mad.lo.u32 {soff}, {st}, {stage_k}, {ring}")
    krow = k.reg("u32")
    k(f"mul.lo.u32 {krow}, {j}, {BKV}")
    kb, vb = bar_at("k_empty", st), bar_at("v_empty", st)
    kf, vf = bar_at("k_full", st), bar_at("v_full", st)
    cx.wait(kb, phe, abort_l)
    k(f"@{pe} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{kf}], {lay['k_bytes'] * halves}")
    for h in range(halves):
        for c in range(D // atom):
            dst, cc = k.reg("u32"), k.reg("u32")
            k(f"add.u32 {dst}, {soff}, {k_addr(h, c)}")
            k(f"mov.u32 {cc}, {c * atom}")
            k(f"@{pe} cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['kh' if h == 0 else 'kl']}, {{{cc}, {krow}, {bh}}}], [{kf}]")
    cx.wait(vb, phe, abort_l)
    k(f"@{pe} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{vf}], {lay['v_bytes'] * halves}")
    for h in range(halves):
        for c in range(max(1, BKV // atom)):
            dst, cc, z = k.reg("u32"), k.reg("u32"), k.reg("u32")
            k(f"add.u32 {dst}, {soff}, {lay[('v', 0, h)] + c * lay['v_chunk']}")
            k(f"add.u32 {cc}, {krow}, {c * atom}")
            k(f"mov.u32 {z}, 0")
            k(f"@{pe} cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['vh' if h == 0 else 'vl']}, {{{cc}, {z}, {bh}}}], [{vf}]")
    k(f"add.u32 {g}, {g}, 1")
    k(f"add.u32 {j}, {j}, 1")
    k(f"setp.lt.u32 {p}, {j}, {nkv}")
    k(f"@{p} bra {jl}")
    k(f"add.u32 {uit}, {uit}, 1")
    k(f"add.u32 {u}, {u}, {ncta}")
    k(f"bra.uni {ul}")
    k.place(ue)
    k(f"bra.uni {teardown}")

    # ================= MMA issuers =================
    # Warp 0 issues S_g = Q . K_g^T into S buffer g % 2 as soon as K_g is in
    # and the buffer is free; warp 1 issues O (+)= P_g . V_g^T once the softmax
    # warps have written P_g.  Two issuing warps on two SM sub-partitions: the
    # sub-partition that issues MMAs also runs a quarter of the softmax (TMEM
    # lane quarters are tied to sub-partitions), so the issue cost is split.
    # Every ordering between the two goes through a barrier (QK(g) waits
    # s_free, committed when PV(g - 2) completes), none through program order.
    def mma_role(which):
        # converged warp, one elected lane issues (descriptors stay warp-uniform)
        pm = k.reg("pred")
        k(f"elect.sync _|{pm}, -1")
        kmaj = _desc_const(16, 1024, 2)      # K-major, 128-byte swizzle, 8-row groups 1 KB apart
        id_s, id_o = k.reg("u32"), k.reg("u32")
        k(f"mov.u32 {id_s}, {_idesc(kind, BQ, BKV)}")
        id_s2 = k.reg("u32")                 # f32: N = 2 * BKV, B = [K_hi; K_lo]
        k(f"mov.u32 {id_s2}, {_idesc(kind, BQ, 2 * BKV)}")
        k(f"mov.u32 {id_o}, {_idesc(kind, BQ, D)}")
        yes = k.reg("pred")
        k(f"setp.eq.u32 {yes}, 0, 0")
        o_t = k.reg("u32")
        k(f"add.u32 {o_t}, {tmem}, {o_col}")
        pairs = [(0, 0), (0, 1), (1, 0)] if f32 else [(0, 0)]

        # Shared-memory descriptors: one base per K/V stage, built once; an
        # operand's descriptor is its stage base plus (byte offset >> 4) in the
        # 14-bit start-address field (shared addresses stay below 2^18, so the
        # field never carries).
        def mkdesc(addr_reg):
            ad, r = k.reg("u32"), k.reg("u64")
            k(f"shr.u32 {ad}, {addr_reg}, 4")
            k(f"and.b32 {ad}, {ad}, 16383")
            k(f"cvt.u64.u32 {r}, {ad}")
            k(f"or.b64 {r}, {r}, 0x{kmaj:016X}")
            return r

        d_base = mkdesc(ring)

        def stage_desc(st_):
            if kvst == 1:
                return d_base
            t, r = k.reg("u64"), k.reg("u64")
            k(f"mul.wide.u32 {t}, {st_}, {stage_k >> 4}")
            k(f"add.s64 {r}, {d_base}, {t}")
            return r

        def dsc(base_d, off):
            assert off % 16 == 0
            r = k.reg("u64")
            k(f"add.s64 {r}, {base_d}, {off >> 4}")
            return r

        def issue_qk(gr):
            st_, phf_ = stage_of(gr)
            b, phs = k.reg("u32"), k.reg("u32")
            k(f"and.b32 {b}, {gr}, 1")
            k(f"shr.u32 {phs}, {gr}, 1")
            k(f"and.b32 {phs}, {phs}, 1")
            k(f"xor.b32 {phs}, {phs}, 1")
            ds = stage_desc(st_)
            s_t = k.reg("u32")
            k(f"mad.lo.u32 {s_t}, {b}, {s_cols}, {tmem}")
            cx.wait(bar_at("k_full", st_), phf_, abort_l)
            cx.wait(bar_at("s_free", b), phs, abort_l)
            k("tcgen05.fence::after_thread_sync")
            first = True
            # f32: columns [0, BKV) get Q_hi.K_hi + Q_lo.K_hi and [BKV, 2 BKV)
            # get Q_hi.K_lo (summed by the softmax), from 2 MMAs per K-step
            # instead of 3; bf16: one product
            groups = [(0, 0, id_s2), (1, 0, id_s)] if f32 else [(0, 0, id_s)]
            for (ha, hb, idd) in groups:
                for c in range(D // atom):
                    for kk in range(4):
                        if q_tmem:
                            # A (Q) from TMEM: 8 f32 columns per K-step, lo D on
                            a_ = k.reg("u32")
                            k(f"add.u32 {a_}, {tmem}, {q_col + ha * D + c * atom + kk * 8}")
                            a_ = f"[{a_}]"
                        else:
                            a_ = dsc(d_base, lay[("q", ha)] + c * lay["q_chunk"] + kk * 32)
                        b_ = dsc(ds, k_addr(hb, c) + kk * 32)
                        acc = yes
                        if first:
                            acc = k.reg("pred")
                            k(f"setp.ne.u32 {acc}, 0, 0")
                            first = False
                        k(f"@{pm} tcgen05.mma.cta_group::1.kind::{kind} [{s_t}], {a_}, {b_}, {idd}, {acc}")
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('s_full', b)}]")
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('k_empty', st_)}]")

        def issue_pv(gr, jr):
            st_, phf_ = stage_of(gr)
            pbuf, php_ = k.reg("u32"), k.reg("u32")
            k(f"and.b32 {pbuf}, {gr}, 1")
            k(f"shr.u32 {php_}, {gr}, 1")
            k(f"and.b32 {php_}, {php_}, 1")
            ds = stage_desc(st_)
            firstb = k.reg("pred")
            k(f"setp.ne.u32 {firstb}, {jr}, 0")
            cx.wait(bar_at("p_full", pbuf), php_, abort_l)
            cx.wait(bar_at("v_full", st_), phf_, abort_l)
            k("tcgen05.fence::after_thread_sync")
            pb, b2 = k.reg("u32"), k.reg("u32")   # P_g lives in S buffer g % 2
            k(f"and.b32 {b2}, {gr}, 1")
            k(f"mov.u32 {pb}, {b2}")
            k(f"mad.lo.u32 {pb}, {pb}, {s_cols}, {tmem}")
            first = True
            for c in range(max(1, BKV // atom)):
                if split_o:
                    # key chunk c (the half written by softmax threads of half c)
                    # accumulates into O_c, started afresh at the unit's first block
                    first = True
                    o_acc = k.reg("u32")
                    k(f"add.u32 {o_acc}, {o_t}, {c * D}")
                else:
                    o_acc = o_t
                for kk in range(min(4, BKV * e // 32)):
                    for (ha, hb) in pairs:
                        # A (P) from TMEM: a 32-byte K-step is 8 columns (16 packed
                        # bf16 or 8 f32); the f32 lo half sits BKV columns on
                        a_ = k.reg("u32")
                        k(f"add.u32 {a_}, {pb}, {_p_col(c * atom + kk * 32 // e, BKV, split, f32) + ha * BKV}")
                        a_ = f"[{a_}]"
                        b_ = dsc(ds, lay[("v", 0, hb)] + c * lay["v_chunk"] + kk * 32)
                        acc = firstb if first else yes
                        first = False
                        k(f"@{pm} tcgen05.mma.cta_group::1.kind::{kind} [{o_acc}], {a_}, {b_}, {id_o}, {acc}")
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_pv_done]")
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('v_empty', st_)}]")
            # P_g was read from S buffer g % 2: the buffer is free once this is done
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('s_free', b2)}]")
        uit2, g2, u2, j2 = (k.reg("u32") for _ in range(4))
        k(f"mov.u32 {uit2}, 0")
        k(f"mov.u32 {g2}, 0")
        k(f"mov.u32 {u2}, {cta}")
        ml, me, mj = k.label(f"{which}_unit"), k.label(f"{which}_unitend"), k.label(f"{which}_kv")
        k.place(ml)
        k(f"setp.ge.u32 {p}, {u2}, {units}")
        k(f"@{p} bra {me}")
        if which == "qk":
            ph3 = k.reg("u32")
            k(f"and.b32 {ph3}, {uit2}, 1")
            cx.wait("bar_q_full", ph3, abort_l)
        k(f"mov.u32 {j2}, 0")
        k.place(mj)
        if which == "qk":
            issue_qk(g2)
        else:
            issue_pv(g2, j2)
        k(f"add.u32 {g2}, {g2}, 1")
        k(f"add.u32 {j2}, {j2}, 1")
        k(f"setp.lt.u32 {p}, {j2}, {nkv}")
        k(f"@{p} bra {mj}")
        if which == "qk":
            if not q_tmem:
                # the unit's Q tile is free once its last S = Q . K^T is done
                k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
                  f"[bar_q_empty]")
        else:
            # the unit's O is complete once its last P . V is
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[bar_o_full]")
        k(f"add.u32 {uit2}, {uit2}, 1")
        k(f"add.u32 {u2}, {u2}, {ncta}")
        k(f"bra.uni {ml}")
        k.place(me)
        k(f"bra.uni {teardown}")

    k.place(role_qk)
    k(f"setp.ne.u32 {p}, {warp}, {W_QK}")
    k(f"@{p} bra {role_pv}")
    mma_role("qk")
    k.place(role_pv)
    k(f"setp.ne.u32 {p}, {warp}, {W_PV}")
    k(f"@{p} bra {role_sm}")
    mma_role("pv")

    # ================= softmax / correction / epilogue: warps 2-9 =================
    # Two threads per query row: warps 2-5 take the first half of the key
    # block's columns, warps 6-9 the second half.  A warp may only touch TMEM
    # lanes 32 * (warp % 4) .. +31, so both warps of a row pair sit on the
    # same lane quarter.  Split O (bf16): each thread keeps its own running
    # max m_h and sum l_h over its half of the keys and its own accumulator
    # O_h; once per unit the pair swaps (m, l) under a 64-thread named
    # barrier (id 1 + quarter) and each writes half of the output columns of
    #   (O_A 2^(m_A - m) + O_B 2^(m_B - m)) / (l_A 2^(m_A - m) + l_B 2^(m_B - m)).
    # Otherwise the pair swaps partial row maxima every block and shares one
    # O (each thread owning half of its columns); the sums are added once.
    k.place(role_sm)
    if split == 2:
        k.shared("\t.shared .align 16 .f32 xch_max[512];")    # [parity][half][row]
        k.shared(f"\t.shared .align 16 .f32 xch_sum[{512 if split_o else 256}];")
    quad, row, half = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"and.b32 {quad}, {warp}, 3")
    k(f"mad.lo.u32 {row}, {quad}, 32, {lane}")
    k(f"sub.u32 {half}, {warp}, 2")
    k(f"shr.u32 {half}, {half}, 2")
    bar_id = k.reg("u32")
    k(f"add.u32 {bar_id}, {quad}, 1")
    hs, ho = BKV // split, D // split       # columns of S and of O per thread
    lane_off = k.reg("u32")
    k(f"mul.lo.u32 {lane_off}, {quad}, {32 << 16}")
    s_row, o_row = k.reg("u32"), k.reg("u32")
    k(f"add.u32 {s_row}, {tmem}, {lane_off}")
    k(f"mad.lo.u32 {s_row}, {half}, {hs}, {s_row}")
    k(f"add.u32 {o_row}, {tmem}, {lane_off}")
    k(f"add.u32 {o_row}, {o_row}, {o_col}")
    k(f"mad.lo.u32 {o_row}, {half}, {ho}, {o_row}")
    if split_o:
        # the O rescale covers this thread's own accumulator, all D columns
        o_resc, resc_cols = k.reg("u32"), D
        k(f"add.u32 {o_resc}, {tmem}, {lane_off}")
        k(f"add.u32 {o_resc}, {o_resc}, {o_col}")
        k(f"mad.lo.u32 {o_resc}, {half}, {D}, {o_resc}")
    else:
        o_resc, resc_cols = o_row, ho
    if split == 2:
        # exchange slots: mine and my partner's (same row, other half)
        x_me, x_pa = k.reg("u32"), k.reg("u32")
        k(f"mov.u32 {x_me}, xch_max")
        k(f"mad.lo.u32 {x_me}, {row}, 4, {x_me}")
        k(f"xor.b32 {x_pa}, {half}, 1")
        k(f"mad.lo.u32 {x_pa}, {x_pa}, 512, {x_me}")
        k(f"mad.lo.u32 {x_me}, {half}, 512, {x_me}")
    cr = k.reg("f32")
    k(f"ld.global.nc.f32 {cr}, [{base[plan.scale]}]")
    v1, sc2 = k.reg("f32"), k.reg("f32")
    k(f"rcp.rn.f32 {v1}, {cr}")
    k(f"mul.rn.f32 {sc2}, {v1}, {f32_hex(LOG2E)}")   # scores to log2 units
    uit3, g3, u3 = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit3}, 0")
    k(f"mov.u32 {g3}, 0")
    k(f"mov.u32 {u3}, {cta}")
    sl, se = k.label("s_unit"), k.label("s_unitend")
    k.place(sl)
    k(f"setp.ge.u32 {p}, {u3}, {units}")
    k(f"@{p} bra {se}")
    if q_tmem:
        # this thread's half of its Q row -> TF32 hi/lo -> TMEM (the A operand
        # of S = Q . K^T).  The previous unit's S = Q . K^T MMAs are done: this
        # thread consumed the last S block of that unit before its epilogue.
        bhq, qbq = unit_coords(u3)
        qg = k.reg("u32")
        k(f"mad.lo.u32 {qg}, {bhq}, {S}, {row}")
        k(f"mad.lo.u32 {qg}, {qbq}, {BQ}, {qg}")
        k(f"mul.lo.u32 {qg}, {qg}, {D}")
        k(f"mad.lo.u32 {qg}, {half}, {ho}, {qg}")
        qptr = k.addr(base[plan.q], qg, 4)
        q_row_t = k.reg("u32")
        k(f"add.u32 {q_row_t}, {tmem}, {lane_off}")
        k(f"add.u32 {q_row_t}, {q_row_t}, {q_col}")
        k(f"mad.lo.u32 {q_row_t}, {half}, {ho}, {q_row_t}")
        for c0 in range(0, ho, 32):
            cnt = min(32, ho - c0)
            xs = k.regs("b32", cnt)
            for v in range(cnt // 4):
                k(f"ld.global.nc.v4.b32 {{{', '.join(xs[4 * v:4 * v + 4])}}}, "
                  f"[{qptr}+{(c0 + 4 * v) * 4}]")
            qh, ql = k.regs("b32", cnt), k.regs("f32", cnt)
            for t in range(cnt):
                k(f"and.b32 {qh[t]}, {xs[t]}, -8192")
                k(f"sub.rn.f32 {ql[t]}, {xs[t]}, {qh[t]}")
            ta, tb = k.reg("u32"), k.reg("u32")
            k(f"add.u32 {ta}, {q_row_t}, {c0}")
            k(f"add.u32 {tb}, {q_row_t}, {D + c0}")
            k(f"tcgen05.st.sync.aligned.32x32b.x{cnt}.b32 [{ta}], {{{', '.join(qh)}}}")
            k(f"tcgen05.st.sync.aligned.32x32b.x{cnt}.b32 [{tb}], {{{', '.join(ql)}}}")
        k("tcgen05.wait::st.sync.aligned")
        k("tcgen05.fence::before_thread_sync")
        k("mbarrier.arrive.shared::cta.b64 _, [bar_q_full]")
    m_run, l_run = k.reg("f32"), k.reg("f32")
    k(f"mov.f32 {m_run}, {f32_hex(-1e30)}")
    k(f"mov.f32 {l_run}, 0f00000000")
    j3 = k.reg("u32")
    k(f"mov.u32 {j3}, 0")
    sj = k.label("s_kv")
    k.place(sj)
    sb, ph5 = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {sb}, {g3}, 1")
    k(f"shr.u32 {ph5}, {g3}, 1")
    k(f"and.b32 {ph5}, {ph5}, 1")
    cx.wait(bar_at("s_full", sb), ph5, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    # my half of the S row -> registers
    nreg = hs
    sv = k.regs("f32", nreg)
    s_cur = k.reg("u32")
    k(f"mad.lo.u32 {s_cur}, {sb}, {s_cols}, {s_row}")
    for c0 in range(0, nreg, 32):
        cnt = min(32, nreg - c0)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {s_cur}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{cnt}.b32 {{{', '.join(sv[c0:c0 + cnt])}}}, [{tad}]")
    if f32:
        # the Q_hi.K_lo partial sits BKV columns on
        sv2 = k.regs("f32", nreg)
        for c0 in range(0, nreg, 32):
            cnt = min(32, nreg - c0)
            tad = k.reg("u32")
            k(f"add.u32 {tad}, {s_cur}, {BKV + c0}")
            k(f"tcgen05.ld.sync.aligned.32x32b.x{cnt}.b32 {{{', '.join(sv2[c0:c0 + cnt])}}}, [{tad}]")
    k("tcgen05.wait::ld.sync.aligned")
    if f32:
        for t in range(nreg):
            k(f"add.rn.f32 {sv[t]}, {sv[t]}, {sv2[t]}")
    # raw partial max in independent three-input chains; scaling by sc2 > 0
    # is monotone, so max(s) * sc2 == max(s * sc2) exactly
    nch = min(4, nreg)
    mx = k.regs("f32", nch)
    for i in range(nch):
        k(f"mov.f32 {mx[i]}, {sv[i]}")
    rest = sv[nch:]
    for i in range(0, len(rest) - 1, 2):
        c = mx[(i // 2) % nch]
        k(f"max.f32 {c}, {c}, {rest[i]}, {rest[i + 1]}")
    if len(rest) % 2:
        k(f"max.f32 {mx[0]}, {mx[0]}, {rest[-1]}")
    mb = k.reg("f32")
    k(f"mov.f32 {mb}, {mx[0]}")
    for i in range(1, nch):
        k(f"max.f32 {mb}, {mb}, {mx[i]}")
    # swap partial maxima with the partner thread (slots double-buffered by
    # block parity, so a slot is rewritten only after the partner read it)
    if split == 2 and not split_o:
        xo = k.reg("u32")
        k(f"mul.lo.u32 {xo}, {sb}, 1024")
        xa, xb = k.reg("u32"), k.reg("u32")
        k(f"add.u32 {xa}, {x_me}, {xo}")
        k(f"add.u32 {xb}, {x_pa}, {xo}")
        k(f"st.shared.f32 [{xa}], {mb}")
        k(f"barrier.sync {bar_id}, 64")
        mo = k.reg("f32")
        k(f"ld.shared.f32 {mo}, [{xb}]")
        k(f"max.f32 {mb}, {mb}, {mo}")
    k(f"mul.rn.f32 {mb}, {mb}, {sc2}")
    pnot0 = k.reg("pred")
    k(f"setp.ne.u32 {pnot0}, {j3}, 0")
    # conditional rescale of the running max and sum (registers only; the O
    # columns in TMEM are rescaled below, once the previous P . V is done)
    need = k.reg("pred")
    thr = k.reg("f32")
    k(f"add.rn.f32 {thr}, {m_run}, {f32_hex(RESCALE_T)}")
    k(f"setp.gt.f32 {need}, {mb}, {thr}")
    anyn = k.reg("pred")
    k(f"vote.sync.any.pred {anyn}, {need}, -1")
    alpha = k.reg("f32")
    k(f"mov.f32 {alpha}, 0f3F800000")
    norsc = k.label("norescale")
    k(f"@!{anyn} bra {norsc}")
    m_new, dlt = k.reg("f32"), k.reg("f32")
    k(f"max.f32 {m_new}, {m_run}, {mb}")
    k(f"sub.rn.f32 {dlt}, {m_run}, {m_new}")
    k(f"ex2.approx.ftz.f32 {alpha}, {dlt}")
    k(f"mul.rn.f32 {l_run}, {l_run}, {alpha}")
    k(f"mov.f32 {m_run}, {m_new}")
    k.place(norsc)
    # p = exp2(s * sc2 - m) with packed f32x2 FMAs, sums in eight partials
    sc2x2, negm2 = k.reg("b64"), k.reg("b64")
    negm = k.reg("f32")
    k(f"neg.f32 {negm}, {m_run}")
    k(f"mov.b64 {sc2x2}, {{{sc2}, {sc2}}}")
    k(f"mov.b64 {negm2}, {{{negm}, {negm}}}")
    nacc = min(4, nreg // 2)
    acc2 = k.regs("b64", nacc)
    zf = k.reg("f32")
    k(f"mov.f32 {zf}, {f32_hex(0.0)}")
    for i in range(nacc):
        k(f"mov.b64 {acc2[i]}, {{{zf}, {zf}}}")
    poly = 0 if f32 else _exp_poly_share()
    pconsts = _exp2_poly_consts(k) if poly else None
    for t in range(0, nreg, 2):
        pr = k.reg("b64")
        k(f"mov.b64 {pr}, {{{sv[t]}, {sv[t + 1]}}}")
        k(f"fma.rn.f32x2 {pr}, {pr}, {sc2x2}, {negm2}")
        if (t // 2) % 4 < poly:
            sv[t], sv[t + 1] = _exp2_poly_pair(k, pr, pconsts)
            k(f"mov.b64 {pr}, {{{sv[t]}, {sv[t + 1]}}}")
        else:
            k(f"mov.b64 {{{sv[t]}, {sv[t + 1]}}}, {pr}")
            k(f"ex2.approx.ftz.f32 {sv[t]}, {sv[t]}")
            k(f"ex2.approx.ftz.f32 {sv[t + 1]}, {sv[t + 1]}")
            k(f"mov.b64 {pr}, {{{sv[t]}, {sv[t + 1]}}}")
        acc = acc2[(t // 2) % nacc]
        k(f"add.rn.f32x2 {acc}, {acc}, {pr}")
    for i in range(1, nacc):
        k(f"add.rn.f32x2 {acc2[0]}, {acc2[0]}, {acc2[i]}")
    sa, sb_ = k.reg("f32"), k.reg("f32")
    k(f"mov.b64 {{{sa}, {sb_}}}, {acc2[0]}")
    k(f"add.rn.f32 {sa}, {sa}, {sb_}")
    k(f"add.rn.f32 {l_run}, {l_run}, {sa}")
    # P in the MMA operand format: TF32 hi/lo (f32) or packed bf16 pairs
    if f32:
        p_hi, p_lo = k.regs("b32", nreg), k.regs("f32", nreg)
        for t in range(nreg):
            k(f"and.b32 {p_hi[t]}, {sv[t]}, -8192")
            k(f"sub.rn.f32 {p_lo[t]}, {sv[t]}, {p_hi[t]}")
        pieces = [(p_hi, 0), (p_lo, BKV)]
    else:
        pk = k.regs("b32", nreg // 2)
        for t in range(nreg // 2):
            k(f"cvt.rn.bf16x2.f32 {pk[t]}, {sv[2 * t + 1]}, {sv[2 * t]}")
        pieces = [(pk, 0)]
    # P over this thread's own S columns in S buffer g % 2 (the partner may
    # not have loaded its scores yet): f32 hi over the score columns and lo
    # BKV columns on; bf16 packed into the first half of them
    p_cur = k.reg("u32")
    k(f"mad.lo.u32 {p_cur}, {sb}, {s_cols}, {s_row}")
    for regs, off in pieces:
        for c0 in range(0, len(regs), 32):
            cnt = min(32, len(regs) - c0)
            tad = k.reg("u32")
            k(f"add.u32 {tad}, {p_cur}, {off + c0}")
            k(f"tcgen05.st.sync.aligned.32x32b.x{cnt}.b32 [{tad}], "
              f"{{{', '.join(regs[c0:c0 + cnt])}}}")
    k("tcgen05.wait::st.sync.aligned")
    # O is only touched when some row of this warp moved its max; then the
    # previous P . V must be done first
    nor2 = k.label("noorescale")
    k(f"@!{anyn} bra {nor2}")
    k(f"@!{pnot0} bra {nor2}")
    php = k.reg("u32")
    k(f"sub.u32 {php}, {g3}, 1")
    k(f"and.b32 {php}, {php}, 1")
    cx.wait("bar_pv_done", php, abort_l)
    k("tcgen05.fence::after_thread_sync")
    for c0 in range(0, resc_cols, 32):
        cnt = min(32, resc_cols - c0)
        ov = k.regs("f32", cnt)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {o_resc}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{cnt}.b32 {{{', '.join(ov)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        for t in range(cnt):
            k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {alpha}")
        k(f"tcgen05.st.sync.aligned.32x32b.x{cnt}.b32 [{tad}], {{{', '.join(ov)}}}")
    k("tcgen05.wait::st.sync.aligned")
    k.place(nor2)
    k("tcgen05.fence::before_thread_sync")
    k(f"mbarrier.arrive.shared::cta.b64 _, [{bar_at('p_full', sb)}]")
    k(f"add.u32 {g3}, {g3}, 1")
    k(f"add.u32 {j3}, {j3}, 1")
    k(f"setp.lt.u32 {p}, {j3}, {nkv}")
    k(f"@{p} bra {sj}")
    # epilogue: the two partial sums, last P . V done, out = O * (1/l)
    lo_sum = k.reg("f32")
    if split_o:
        # swap (m, l) with the partner (slots double-buffered by unit parity)
        xoff, xq = k.reg("u32"), k.reg("u32")
        k(f"and.b32 {xoff}, {uit3}, 1")
        k(f"mul.lo.u32 {xoff}, {xoff}, 1024")
        k(f"mad.lo.u32 {xoff}, {row}, 4, {xoff}")
        k(f"xor.b32 {xq}, {half}, 1")
        am, al, bm, bl = (k.reg("u32") for _ in range(4))
        k(f"mov.u32 {am}, xch_max")
        k(f"mov.u32 {al}, xch_sum")
        k(f"add.u32 {am}, {am}, {xoff}")
        k(f"add.u32 {al}, {al}, {xoff}")
        k(f"mad.lo.u32 {bm}, {xq}, 512, {am}")
        k(f"mad.lo.u32 {bl}, {xq}, 512, {al}")
        k(f"mad.lo.u32 {am}, {half}, 512, {am}")
        k(f"mad.lo.u32 {al}, {half}, 512, {al}")
        k(f"st.shared.f32 [{am}], {m_run}")
        k(f"st.shared.f32 [{al}], {l_run}")
        k(f"barrier.sync {bar_id}, 64")
        mo, lo2 = k.reg("f32"), k.reg("f32")
        k(f"ld.shared.f32 {mo}, [{bm}]")
        k(f"ld.shared.f32 {lo2}, [{bl}]")
        # half A's numbers first on both threads, so both compute the same
        is1 = k.reg("pred")
        k(f"setp.ne.u32 {is1}, {half}, 0")
        m0, m1, l0, l1 = (k.reg("f32") for _ in range(4))
        k(f"selp.f32 {m0}, {mo}, {m_run}, {is1}")
        k(f"selp.f32 {m1}, {m_run}, {mo}, {is1}")
        k(f"selp.f32 {l0}, {lo2}, {l_run}, {is1}")
        k(f"selp.f32 {l1}, {l_run}, {lo2}, {is1}")
        mm, a0, a1 = k.reg("f32"), k.reg("f32"), k.reg("f32")
        k(f"max.f32 {mm}, {m0}, {m1}")
        k(f"sub.rn.f32 {a0}, {m0}, {mm}")
        k(f"sub.rn.f32 {a1}, {m1}, {mm}")
        k(f"ex2.approx.ftz.f32 {a0}, {a0}")
        k(f"ex2.approx.ftz.f32 {a1}, {a1}")
        k(f"mul.rn.f32 {lo_sum}, {l0}, {a0}")
        k(f"fma.rn.f32 {lo_sum}, {l1}, {a1}, {lo_sum}")
    elif split == 2:
        xs, xp = k.reg("u32"), k.reg("u32")
        k(f"mov.u32 {xs}, xch_sum")
        k(f"mad.lo.u32 {xs}, {row}, 4, {xs}")
        k(f"xor.b32 {xp}, {half}, 1")
        k(f"mad.lo.u32 {xp}, {xp}, 512, {xs}")
        k(f"mad.lo.u32 {xs}, {half}, 512, {xs}")
        k(f"st.shared.f32 [{xs}], {l_run}")
        k(f"barrier.sync {bar_id}, 64")
        k(f"ld.shared.f32 {lo_sum}, [{xp}]")
        # both threads add the same two numbers (commutative), so agree on l
        k(f"add.rn.f32 {lo_sum}, {l_run}, {lo_sum}")
    else:
        k(f"mov.f32 {lo_sum}, {l_run}")
    phl = k.reg("u32")
    k(f"and.b32 {phl}, {uit3}, 1")
    cx.wait("bar_o_full", phl, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    rl = k.reg("f32")
    k(f"rcp.rn.f32 {rl}, {lo_sum}")
    if split_o:
        w0, w1 = k.reg("f32"), k.reg("f32")
        k(f"mul.rn.f32 {w0}, {a0}, {rl}")
        k(f"mul.rn.f32 {w1}, {a1}, {rl}")
    bh3, qb3 = unit_coords(u3)
    grow = k.reg("u32")
    k(f"mad.lo.u32 {grow}, {bh3}, {S}, {row}")
    k(f"mad.lo.u32 {grow}, {qb3}, {BQ}, {grow}")
    k(f"mul.lo.u32 {grow}, {grow}, {D}")
    k(f"mad.lo.u32 {grow}, {half}, {ho}, {grow}")
    optr = k.addr(base[plan.out], grow, e)
    for c0 in range(0, ho, 32):
        cnt = min(32, ho - c0)
        ov = k.regs("f32", cnt)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {o_row}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{cnt}.b32 {{{', '.join(ov)}}}, [{tad}]")
        if split_o:
            ob = k.regs("f32", cnt)
            tb = k.reg("u32")
            k(f"add.u32 {tb}, {tad}, {D}")
            k(f"tcgen05.ld.sync.aligned.32x32b.x{cnt}.b32 {{{', '.join(ob)}}}, [{tb}]")
        k("tcgen05.wait::ld.sync.aligned")
        for t in range(cnt):
            if split_o:
                k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {w0}")
                k(f"fma.rn.f32 {ov[t]}, {ob[t]}, {w1}, {ov[t]}")
            else:
                k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {rl}")
        if f32:
            for v in range(cnt // 4):
                k(f"st.global.v4.f32 [{optr}+{(c0 + 4 * v) * 4}], {{{', '.join(ov[4 * v:4 * v + 4])}}}")
        else:
            pk = k.regs("b32", cnt // 2)
            for t in range(cnt // 2):
                k(f"cvt.rn.bf16x2.f32 {pk[t]}, {ov[2 * t + 1]}, {ov[2 * t]}")
            for v in range(cnt // 8):
                k(f"st.global.v4.b32 [{optr}+{(c0 + 8 * v) * 2}], {{{', '.join(pk[4 * v:4 * v + 4])}}}")
    k("tcgen05.fence::before_thread_sync")
    k(f"add.u32 {uit3}, {uit3}, 1")
    k(f"add.u32 {u3}, {u3}, {ncta}")
    k(f"bra.uni {sl}")
    k.place(se)
    k(f"bra.uni {teardown}")

    # ================= abort and teardown =================
    k.place(abort_l)
    k("st.volatile.shared.u32 [abort_flag], 1")
    k.place(teardown)
    k("barrier.sync 0")
    ab = k.reg("u32")
    k(f"ld.volatile.shared.u32 {ab}, [abort_flag]")
    drained = k.label("drained")
    k(f"setp.eq.u32 {p}, {ab}, 0")
    k(f"@{p} bra {drained}")
    k(f"setp.ne.u32 {q}, {tid}, 0")
    k(f"@{q} bra {drained}")
    t0, t1 = k.reg("u64"), k.reg("u64")
    lw = k.label("drain")
    k(f"mov.u64 {t0}, %globaltimer")
    k.place(lw)
    k(f"mov.u64 {t1}, %globaltimer")
    k(f"sub.u64 {t1}, {t1}, {t0}")
    k(f"setp.lt.u64 {p}, {t1}, 50000000")
    k(f"@{p} bra {lw}")
    k.place(drained)
    # each issuing lane (lane 0 of warps 0 and 1, the elect.sync leaders)
    # waits, bounded, for its own MMAs to complete before TMEM is freed
    for w_iss, dbar in ((W_QK, "bar_drain_qk"), (W_PV, "bar_drain")):
        k(f"setp.ne.u32 {q}, {tid}, {w_iss * 32}")
        nd = k.label("nodrain")
        k(f"@{q} bra {nd}")
        k(f"tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [{dbar}]")
        pp2 = k.reg("pred")
        t2, t3 = k.reg("u64"), k.reg("u64")
        lw2, ld2 = k.label("mdrain"), k.label("mdraindone")
        k(f"mov.u64 {t2}, %globaltimer")
        k.place(lw2)
        k(f"mbarrier.try_wait.parity.shared::cta.b64 {pp2}, [{dbar}], 0")
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
    k(f"setp.ne.u32 {p}, {warp}, {W_PV}")
    k(f"@{p} bra {fin}")
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, {tcols}")
    k.place(fin)
