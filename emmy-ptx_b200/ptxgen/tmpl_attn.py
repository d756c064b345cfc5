"""Fused online-softmax attention on tcgen05 (a01/a02 family, and [B,H,S,D]).

IR family: ``out[.., i, c] = sum_j softmax_j(q_i . k_j * (1/c0)) v[.., j, c]``
with the online-softmax update per key (``a02``: Loop over keys, inner Loop
over the head dimension, coupled max/sum Accums, final multiply by the
reciprocal of the sum).  K is given either transposed (``kt [D, S]``, the
shipped problems) or as ``k [.., S, D]``.

B200 kernel (one persistent CTA per SM, 192 threads; a unit is one
batch*head and 128 query rows):

* warp 0 -- TMA: the unit's Q tile once, then per key block the K block and
  the V^T block (all K-major, 128-byte swizzle);
* warp 1 -- allocates TMEM (S block + O, f32) and issues
  ``S = Q . K^T`` then ``O += P . V^T`` with ``tcgen05.mma`` (kind::tf32 in
  three hi/lo passes for f32 data; kind::f16 on bf16 data);
* warps 2-5 -- one thread per query row: ``tcgen05.ld`` of its S row, row max,
  ``p = exp(s/c0 - m)``, running sum, P written to shared memory as the A
  operand of the next MMA (hi/lo TF32 or bf16), rescale of its O row in TMEM
  only when the row max grew by more than 8 (``m`` is otherwise kept, so
  ``p <= e^8``; the result is the same sum, only rounded differently), and at
  the end ``O / l`` to global memory.

A pre-pass writes the hi/lo TF32 halves of Q and K (f32 only) and V^T (and K
from K^T when the IR gives K transposed) into a launcher-owned workspace.
Every wait is bounded by ``%globaltimer`` and reports through ``emmy_err``.

Any other launch -- meta.json's geometry, or shapes the tensor-core path
does not tile (S not a multiple of 128) -- takes a SIMT path that evaluates
each output element with the IR's own per-key statements.
"""

from __future__ import annotations

import math

from . import ir
from .analysis import NoMatch, flat_affine, numel
from .lower import Lowerer, Val
from .model import KernelSpec, dtype_info
from .ptx import Kernel, Module, f32_hex
from .tmpl_mma import ERR_WAIT_TIMEOUT, PLAN_MAGIC, _Ctx, _desc_const

LOG2E = 1.4426950408889634
THREADS = 192
W_PROD, W_MMA = 0, 1
BQ = 128
RESCALE_T = 8.0


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


def _layout(plan):
    """Shared-memory regions (bytes) of one unit: Q (resident), K block, V^T
    block and P, each ``passes`` deep (hi, lo) for f32."""
    e, atom, bkv, d = plan.e, plan.atom, plan.bkv, plan.d
    halves = 2 if plan.dtype == "f32" else 1
    q_chunk = BQ * 128                 # one 128-byte-wide column chunk of 128 rows
    q_bytes = (d // atom) * q_chunk
    k_chunk = bkv * 128
    k_bytes = (d // atom) * k_chunk
    v_chunk = d * 128                  # V^T: d rows, bkv keys wide
    v_bytes = max(1, bkv // atom) * v_chunk
    p_chunk = BQ * 128
    p_bytes = max(1, bkv // atom) * p_chunk
    lay = {}
    off = 0
    for name, size in (("q", q_bytes), ("k", k_bytes), ("v", v_bytes), ("p", p_bytes)):
        for h in range(halves):
            lay[(name, h)] = off
            off += size
    lay["total"] = off
    lay.update(q_bytes=q_bytes, k_bytes=k_bytes, v_bytes=v_bytes, p_bytes=p_bytes,
               q_chunk=q_chunk, k_chunk=k_chunk, v_chunk=v_chunk, p_chunk=p_chunk,
               halves=halves)
    return lay


def emit_attention(spec: KernelSpec, plan: AttnPlan) -> Module:
    params = [(f"p_{n}", ".u64") for n in spec.arg_order]
    k = Kernel(spec.entry, params)
    mod = Module(comment=f"emmy-b200 tcgen05 attention template for {spec.entry}")
    mod.add_global(".visible .global .align 4 .u32 emmy_err;")
    mod.add_global(".visible .global .align 4 .u32 emmy_plan;")
    mod.add_global(".visible .global .align 8 .u64 emmy_ws;")
    tnames = ["qh", "ql", "kh", "kl", "vh", "vl"] if plan.dtype == "f32" else ["qh", "kh", "vh"]
    for t in tnames:
        mod.add_global(f".visible .global .align 64 .b8 tmap_{t}[128];")
    base = {n: k.param_ptr(f"p_{n}") for n in spec.arg_order}
    tid, ntid = k.sreg("%tid.x"), k.sreg("%ntid.x")
    cta, ncta = k.sreg("%ctaid.x"), k.sreg("%nctaid.x")
    p = k.reg("pred")
    simt = k.label("simt")
    lay = _layout(plan)
    dyn = lay["total"] + 1024
    if plan.tc and dyn <= 232448 - 1024:
        mod.add_global(".extern .shared .align 1024 .b8 dsmem[];")
        flag, dsz = k.reg("u32"), k.reg("u32")
        k(f"ld.global.u32 {flag}, [emmy_plan]")
        k(f"setp.ne.u32 {p}, {flag}, {PLAN_MAGIC}")
        k(f"@{p} bra {simt}")
        k(f"setp.ne.u32 {p}, {ntid}, {THREADS}")
        k(f"@{p} bra {simt}")
        k(f"mov.u32 {dsz}, %dynamic_smem_size")
        k(f"setp.lt.u32 {p}, {dsz}, {dyn}")
        k(f"@{p} bra {simt}")
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
        pre, ws_bytes, tm = _emit_pre(mod, spec, plan)
        plan_d.update({
            "block": THREADS, "grid_per_sm": 1, "grid_max": BH * (S // BQ), "smem": dyn,
            "workspace": {"sym": "emmy_ws", "bytes": ws_bytes}, "pre": pre, "tmaps": tm,
            "flags": [{"sym": "emmy_plan", "value": PLAN_MAGIC}],
            "tile": [BQ, plan.bkv, D], "passes": plan.passes,
        })
    mod.plan = plan_d
    return mod


# ---------------------------------------------------------------------------
# pre-pass: operand preparation into the workspace
# ---------------------------------------------------------------------------


def _ws_layout(plan):
    """Workspace regions (bytes): hi/lo of Q, K ([BH, S, D]) and V^T ([BH, D, S])
    for f32; K (only when given transposed) and V^T for bf16."""
    n = plan.bh * plan.s * plan.d * plan.e
    off = {}
    cur = 0
    names = ["qh", "ql", "kh", "kl", "vh", "vl"] if plan.dtype == "f32" else ["kh", "vh"]
    for nm in names:
        off[nm] = cur
        cur += n
    return off, cur


def _emit_pre(mod: Module, spec: KernelSpec, plan):
    off, total = _ws_layout(plan)
    f32 = plan.dtype == "f32"
    pre = []
    S, D, BH = plan.s, plan.d, plan.bh
    if f32:
        mod.kernels.append(_emit_split_copy(spec, plan, plan.q, off["qh"], off["ql"], "_pre_q"))
        pre.append({"entry": f"{spec.entry}_pre_q", "block": 256, "grid_per_sm": 8,
                    "grid_max": max(1, BH * S * D // 4 // 256)})
        if plan.k_trans:
            mod.kernels.append(_emit_transpose(spec, plan, plan.k, D, S, off["kh"],
                                               off["kl"], "_pre_k"))
            pre.append({"entry": f"{spec.entry}_pre_k", "block": 256, "grid_per_sm": 8,
                        "grid_max": BH * (D // 32) * (S // 32)})
        else:
            mod.kernels.append(_emit_split_copy(spec, plan, plan.k, off["kh"], off["kl"],
                                                "_pre_k"))
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
        mod.kernels.append(_emit_transpose(spec, plan, plan.v, S, D, off["vh"], None, "_pre_v"))
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
        tm += [tmap("tmap_qh", "@ws", off["qh"], D, S, BQ), tmap("tmap_ql", "@ws", off["ql"], D, S, BQ),
               tmap("tmap_kh", "@ws", off["kh"], D, S, plan.bkv),
               tmap("tmap_kl", "@ws", off["kl"], D, S, plan.bkv),
               tmap("tmap_vh", "@ws", off["vh"], S, D, D), tmap("tmap_vl", "@ws", off["vl"], S, D, D)]
    else:
        tm += [tmap("tmap_qh", plan.q, 0, D, S, BQ),
               (tmap("tmap_kh", "@ws", off["kh"], D, S, plan.bkv) if plan.k_trans else
                tmap("tmap_kh", plan.k, 0, D, S, plan.bkv)),
               tmap("tmap_vh", "@ws", off["vh"], S, D, D)]
    return pre, max(total, 16), tm


def _emit_split_copy(spec, plan, buf, off_hi, off_lo, suffix) -> Kernel:
    """x -> (hi, lo) of the same shape (f32)."""
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


def _emit_tc(k: Kernel, spec, plan, lay, base, tid, cta, ncta):
    S, D, BH, BKV = plan.s, plan.d, plan.bh, plan.bkv
    f32 = plan.dtype == "f32"
    e, atom, passes = plan.e, plan.atom, plan.passes
    halves = lay["halves"]
    kind = "tf32" if f32 else "f16"
    nkv = S // BKV
    qblocks = S // BQ
    units = BH * qblocks
    cx = _Ctx(k)
    for nm in ("q_full", "q_empty", "kv_full", "kv_empty", "s_full", "p_full", "pv_done",
               "drain"):
        k.shared(f"\t.shared .align 8 .b64 bar_{nm};")
    k.shared("\t.shared .align 4 .u32 tmem_slot;")
    k.shared("\t.shared .align 4 .u32 abort_flag;")
    s_cols = max(32, BKV)
    tcols = 1 << (s_cols + D - 1).bit_length()
    warp, lane = k.reg("u32"), k.reg("u32")
    k(f"shr.u32 {warp}, {tid}, 5")
    k(f"and.b32 {lane}, {tid}, 31")
    p, q = k.reg("pred"), k.reg("pred")
    ring = k.reg("u32")
    k(f"mov.u32 {ring}, dsmem")
    k(f"add.u32 {ring}, {ring}, 1023")
    k(f"and.b32 {ring}, {ring}, -1024")
    tnames = ["qh", "ql", "kh", "kl", "vh", "vl"] if f32 else ["qh", "kh", "vh"]
    tm = {}
    for t in tnames:
        r = k.reg("u64")
        k(f"mov.u64 {r}, tmap_{t}")
        k(f"cvta.global.u64 {r}, {r}")
        tm[t] = r

    skip = k.label("noinit")
    k(f"setp.ne.u32 {p}, {tid}, 0")
    k(f"@{p} bra {skip}")
    for nm, cnt in (("q_full", 1), ("q_empty", 1), ("kv_full", 1), ("kv_empty", 1),
                    ("s_full", 1), ("p_full", 128), ("pv_done", 1), ("drain", 1)):
        k(f"mbarrier.init.shared::cta.b64 [bar_{nm}], {cnt}")
    k("st.shared.u32 [abort_flag], 0")
    for r in tm.values():
        k(f"prefetch.tensormap [{r}]")
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
    role_mma, role_sm = k.label("rmma"), k.label("rsm")

    def smem(name, h, extra=0):
        r = k.reg("u32")
        k(f"add.u32 {r}, {ring}, {lay[(name, h)] + extra}")
        return r

    def unit_coords(u):
        bh, qb = k.reg("u32"), k.reg("u32")
        k(f"div.u32 {bh}, {u}, {qblocks}")
        k(f"rem.u32 {qb}, {u}, {qblocks}")
        return bh, qb

    # ================= producer =================
    k(f"setp.ne.u32 {p}, {warp}, {W_PROD}")
    k(f"@{p} bra {role_mma}")
    k(f"setp.ne.u32 {p}, {lane}, 0")
    k(f"@{p} bra {teardown}")
    uit, kvit, u = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit}, 0")
    k(f"mov.u32 {kvit}, 0")
    k(f"mov.u32 {u}, {cta}")
    ul, ue = k.label("p_unit"), k.label("p_unitend")
    k.place(ul)
    k(f"setp.ge.u32 {p}, {u}, {units}")
    k(f"@{p} bra {ue}")
    bh, qb = unit_coords(u)
    qrow = k.reg("u32")
    k(f"mul.lo.u32 {qrow}, {qb}, {BQ}")
    ph = k.reg("u32")
    k(f"and.b32 {ph}, {uit}, 1")
    k(f"xor.b32 {ph}, {ph}, 1")
    cx.wait("bar_q_empty", ph, abort_l)
    qbytes = lay["q_bytes"] * halves
    k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [bar_q_full], {qbytes}")
    for h in range(halves):
        for c in range(D // atom):
            dst, cc = smem("q", h, c * lay["q_chunk"]), k.reg("u32")
            k(f"mov.u32 {cc}, {c * atom}")
            k(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['qh' if h == 0 else 'ql']}, {{{cc}, {qrow}, {bh}}}], [bar_q_full]")
    j = k.reg("u32")
    k(f"mov.u32 {j}, 0")
    jl = k.label("p_kv")
    k.place(jl)
    ph2 = k.reg("u32")
    k(f"and.b32 {ph2}, {kvit}, 1")
    k(f"xor.b32 {ph2}, {ph2}, 1")
    cx.wait("bar_kv_empty", ph2, abort_l)
    kvbytes = (lay["k_bytes"] + lay["v_bytes"]) * halves
    k(f"mbarrier.arrive.expect_tx.shared::cta.b64 _, [bar_kv_full], {kvbytes}")
    krow = k.reg("u32")
    k(f"mul.lo.u32 {krow}, {j}, {BKV}")
    for h in range(halves):
        for c in range(D // atom):
            dst, cc = smem("k", h, c * lay["k_chunk"]), k.reg("u32")
            k(f"mov.u32 {cc}, {c * atom}")
            k(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['kh' if h == 0 else 'kl']}, {{{cc}, {krow}, {bh}}}], [bar_kv_full]")
        for c in range(max(1, BKV // atom)):
            dst, cc = smem("v", h, c * lay["v_chunk"]), k.reg("u32")
            k(f"add.u32 {cc}, {krow}, {c * atom}")
            z = k.reg("u32")
            k(f"mov.u32 {z}, 0")
            k(f"cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['vh' if h == 0 else 'vl']}, {{{cc}, {z}, {bh}}}], [bar_kv_full]")
    k(f"add.u32 {kvit}, {kvit}, 1")
    k(f"add.u32 {j}, {j}, 1")
    k(f"setp.lt.u32 {p}, {j}, {nkv}")
    k(f"@{p} bra {jl}")
    k(f"add.u32 {uit}, {uit}, 1")
    k(f"add.u32 {u}, {u}, {ncta}")
    k(f"bra.uni {ul}")
    k.place(ue)
    k(f"bra.uni {teardown}")

    # ================= MMA issuer =================
    k.place(role_mma)
    k(f"setp.ne.u32 {p}, {warp}, {W_MMA}")
    k(f"@{p} bra {role_sm}")
    k(f"setp.ne.u32 {p}, {lane}, 0")
    k(f"@{p} bra {teardown}")
    kmaj = _desc_const(16, 1024, 2)      # K-major, 128-byte swizzle, 8-row groups 1 KB apart
    id_s, id_o = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {id_s}, {_idesc(kind, BQ, BKV)}")
    k(f"mov.u32 {id_o}, {_idesc(kind, BQ, D)}")
    yes = k.reg("pred")
    k(f"setp.eq.u32 {yes}, 0, 0")
    s_t, o_t = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {s_t}, {tmem}")
    k(f"add.u32 {o_t}, {tmem}, {s_cols}")
    uit2, kvit2, u2 = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit2}, 0")
    k(f"mov.u32 {kvit2}, 0")
    k(f"mov.u32 {u2}, {cta}")
    ml, me = k.label("m_unit"), k.label("m_unitend")
    k.place(ml)
    k(f"setp.ge.u32 {p}, {u2}, {units}")
    k(f"@{p} bra {me}")
    ph3 = k.reg("u32")
    k(f"and.b32 {ph3}, {uit2}, 1")
    cx.wait("bar_q_full", ph3, abort_l)
    j2 = k.reg("u32")
    k(f"mov.u32 {j2}, 0")
    mj = k.label("m_kv")
    k.place(mj)
    ph4 = k.reg("u32")
    k(f"and.b32 {ph4}, {kvit2}, 1")
    cx.wait("bar_kv_full", ph4, abort_l)
    k("tcgen05.fence::after_thread_sync")

    def desc(addr_reg, off):
        ad, r = k.reg("u32"), k.reg("u64")
        k(f"add.u32 {ad}, {addr_reg}, {off}")
        k(f"shr.u32 {ad}, {ad}, 4")
        k(f"and.b32 {ad}, {ad}, 16383")
        k(f"cvt.u64.u32 {r}, {ad}")
        k(f"or.b64 {r}, {r}, 0x{kmaj:016X}")
        return r

    pairs = [(0, 0), (0, 1), (1, 0)] if f32 else [(0, 0)]
    # S = Q . K^T over D, in atom-wide chunks of 4 MMA K-steps
    first = True
    for c in range(D // atom):
        for kk in range(4):
            for (ha, hb) in pairs:
                a = desc(ring, lay[("q", ha)] + c * lay["q_chunk"] + kk * 32)
                b = desc(ring, lay[("k", hb)] + c * lay["k_chunk"] + kk * 32)
                acc = yes
                if first:
                    acc = k.reg("pred")
                    k(f"setp.ne.u32 {acc}, 0, 0")
                    first = False
                k(f"tcgen05.mma.cta_group::1.kind::{kind} [{s_t}], {a}, {b}, {id_s}, {acc}")
    k("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_s_full]")
    # O (+)= P . V^T over the key block
    cx.wait("bar_p_full", ph4, abort_l)
    k("tcgen05.fence::after_thread_sync")
    firstb = k.reg("pred")
    k(f"setp.ne.u32 {firstb}, {j2}, 0")
    first = True
    for c in range(max(1, BKV // atom)):
        for kk in range(min(4, BKV * e // 32)):
            for (ha, hb) in pairs:
                a = desc(ring, lay[("p", ha)] + c * lay["p_chunk"] + kk * 32)
                b = desc(ring, lay[("v", hb)] + c * lay["v_chunk"] + kk * 32)
                acc = firstb if first else yes
                first = False
                k(f"tcgen05.mma.cta_group::1.kind::{kind} [{o_t}], {a}, {b}, {id_o}, {acc}")
    k("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_pv_done]")
    k("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_kv_empty]")
    k(f"add.u32 {kvit2}, {kvit2}, 1")
    k(f"add.u32 {j2}, {j2}, 1")
    k(f"setp.lt.u32 {p}, {j2}, {nkv}")
    k(f"@{p} bra {mj}")
    k("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [bar_q_empty]")
    k(f"add.u32 {uit2}, {uit2}, 1")
    k(f"add.u32 {u2}, {u2}, {ncta}")
    k(f"bra.uni {ml}")
    k.place(me)
    k(f"bra.uni {teardown}")

    # ================= softmax / correction / epilogue: warps 2-5 =================
    k.place(role_sm)
    quad, row = k.reg("u32"), k.reg("u32")
    k(f"and.b32 {quad}, {warp}, 3")
    k(f"mad.lo.u32 {row}, {quad}, 32, {lane}")
    lane_off = k.reg("u32")
    k(f"mul.lo.u32 {lane_off}, {quad}, {32 << 16}")
    s_row, o_row = k.reg("u32"), k.reg("u32")
    k(f"add.u32 {s_row}, {tmem}, {lane_off}")
    k(f"add.u32 {o_row}, {s_row}, {s_cols}")
    cr = k.reg("f32")
    k(f"ld.global.nc.f32 {cr}, [{base[plan.scale]}]")
    v1, sc2 = k.reg("f32"), k.reg("f32")
    k(f"rcp.rn.f32 {v1}, {cr}")
    k(f"mul.rn.f32 {sc2}, {v1}, {f32_hex(LOG2E)}")   # scores to log2 units
    # smem P row address pieces: chunk base + (row/8)*1024 + (row%8)*128; swizzle by row%8
    r8, rlo, prow = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"shr.u32 {r8}, {row}, 3")
    k(f"and.b32 {rlo}, {row}, 7")
    k(f"mad.lo.u32 {prow}, {r8}, 1024, {ring}")
    k(f"mad.lo.u32 {prow}, {rlo}, 128, {prow}")
    uit3, kvit3, u3 = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit3}, 0")
    k(f"mov.u32 {kvit3}, 0")
    k(f"mov.u32 {u3}, {cta}")
    sl, se = k.label("s_unit"), k.label("s_unitend")
    k.place(sl)
    k(f"setp.ge.u32 {p}, {u3}, {units}")
    k(f"@{p} bra {se}")
    m_run, l_run = k.reg("f32"), k.reg("f32")
    k(f"mov.f32 {m_run}, {f32_hex(-1e30)}")
    k(f"mov.f32 {l_run}, 0f00000000")
    j3 = k.reg("u32")
    k(f"mov.u32 {j3}, 0")
    sj = k.label("s_kv")
    k.place(sj)
    ph5 = k.reg("u32")
    k(f"and.b32 {ph5}, {kvit3}, 1")
    cx.wait("bar_s_full", ph5, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    # S row -> registers (log2-scaled), row max
    nreg = BKV
    sv = k.regs("f32", nreg)
    for c0 in range(0, BKV, 32):
        cnt = min(32, BKV - c0)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {s_row}, {c0}")
        shape = f"32x32b.x{cnt}"
        k(f"tcgen05.ld.sync.aligned.{shape}.b32 {{{', '.join(sv[c0:c0 + cnt])}}}, [{tad}]")
    k("tcgen05.wait::ld.sync.aligned")
    mb = k.reg("f32")
    k(f"mul.rn.f32 {sv[0]}, {sv[0]}, {sc2}")
    k(f"mov.f32 {mb}, {sv[0]}")
    for t in range(1, nreg):
        k(f"mul.rn.f32 {sv[t]}, {sv[t]}, {sc2}")
        k(f"max.f32 {mb}, {mb}, {sv[t]}")
    # previous P . V done before P is overwritten or O rescaled
    pnot0 = k.reg("pred")
    k(f"setp.ne.u32 {pnot0}, {j3}, 0")
    wprev = k.label("nowaitpv")
    k(f"@!{pnot0} bra {wprev}")
    php = k.reg("u32")
    k(f"sub.u32 {php}, {kvit3}, 1")
    k(f"and.b32 {php}, {php}, 1")
    cx.wait("bar_pv_done", php, abort_l)
    k.place(wprev)
    # conditional rescale, warp-uniform
    need = k.reg("pred")
    thr = k.reg("f32")
    k(f"add.rn.f32 {thr}, {m_run}, {f32_hex(RESCALE_T)}")
    k(f"setp.gt.f32 {need}, {mb}, {thr}")
    anyn = k.reg("pred")
    k(f"vote.sync.any.pred {anyn}, {need}, -1")
    norsc = k.label("norescale")
    k(f"@!{anyn} bra {norsc}")
    m_new, alpha, dlt = k.reg("f32"), k.reg("f32"), k.reg("f32")
    k(f"max.f32 {m_new}, {m_run}, {mb}")
    k(f"sub.rn.f32 {dlt}, {m_run}, {m_new}")
    k(f"ex2.approx.ftz.f32 {alpha}, {dlt}")
    k(f"mul.rn.f32 {l_run}, {l_run}, {alpha}")
    k(f"mov.f32 {m_run}, {m_new}")
    # O row *= alpha (only after the first block has written O)
    k(f"@!{pnot0} bra {norsc}")
    k("tcgen05.fence::after_thread_sync")
    for c0 in range(0, D, 32):
        ov = k.regs("f32", 32)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {o_row}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        for t in range(32):
            k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {alpha}")
        k(f"tcgen05.st.sync.aligned.32x32b.x32.b32 [{tad}], {{{', '.join(ov)}}}")
    k("tcgen05.wait::st.sync.aligned")
    k.place(norsc)
    # P = exp2(s - m), row sum, P -> smem (K-major, 128-byte swizzle)
    for t in range(nreg):
        k(f"sub.rn.f32 {sv[t]}, {sv[t]}, {m_run}")
        k(f"ex2.approx.ftz.f32 {sv[t]}, {sv[t]}")
        k(f"add.rn.f32 {l_run}, {l_run}, {sv[t]}")
    per16 = 16 // e                       # elements per 16-byte unit
    for c in range(max(1, BKV // atom)):
        for uidx in range(min(8, BKV * e // 16)):
            vals = sv[c * atom + uidx * per16: c * atom + (uidx + 1) * per16]
            sw, ad = k.reg("u32"), k.reg("u32")
            k(f"xor.b32 {sw}, {rlo}, {uidx}")
            k(f"mad.lo.u32 {ad}, {sw}, 16, {prow}")
            if f32:
                hi, lo_ = k.regs("b32", 4), k.regs("f32", 4)
                for t in range(4):
                    k(f"and.b32 {hi[t]}, {vals[t]}, -8192")
                    k(f"sub.rn.f32 {lo_[t]}, {vals[t]}, {hi[t]}")
                k(f"st.shared.v4.b32 [{ad}+{lay[('p', 0)] + c * lay['p_chunk']}], "
                  f"{{{', '.join(hi)}}}")
                k(f"st.shared.v4.f32 [{ad}+{lay[('p', 1)] + c * lay['p_chunk']}], "
                  f"{{{', '.join(lo_)}}}")
            else:
                pk = k.regs("b32", 4)
                for t in range(4):
                    k(f"cvt.rn.bf16x2.f32 {pk[t]}, {vals[2 * t + 1]}, {vals[2 * t]}")
                k(f"st.shared.v4.b32 [{ad}+{lay[('p', 0)] + c * lay['p_chunk']}], "
                  f"{{{', '.join(pk)}}}")
    k("fence.proxy.async.shared::cta")
    k("tcgen05.fence::before_thread_sync")
    k("mbarrier.arrive.shared::cta.b64 _, [bar_p_full]")
    k(f"add.u32 {kvit3}, {kvit3}, 1")
    k(f"add.u32 {j3}, {j3}, 1")
    k(f"setp.lt.u32 {p}, {j3}, {nkv}")
    k(f"@{p} bra {sj}")
    # epilogue: last P . V done, out = O * (1/l)
    phl = k.reg("u32")
    k(f"sub.u32 {phl}, {kvit3}, 1")
    k(f"and.b32 {phl}, {phl}, 1")
    cx.wait("bar_pv_done", phl, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    rl = k.reg("f32")
    k(f"rcp.rn.f32 {rl}, {l_run}")
    bh3, qb3 = unit_coords(u3)
    grow = k.reg("u32")
    k(f"mad.lo.u32 {grow}, {bh3}, {S}, {row}")
    k(f"mad.lo.u32 {grow}, {qb3}, {BQ}, {grow}")
    k(f"mul.lo.u32 {grow}, {grow}, {D}")
    optr = k.addr(base[plan.out], grow, e)
    for c0 in range(0, D, 32):
        ov = k.regs("f32", 32)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {o_row}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        for t in range(32):
            k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {rl}")
        if f32:
            for v in range(8):
                k(f"st.global.v4.f32 [{optr}+{(c0 + 4 * v) * 4}], {{{', '.join(ov[4 * v:4 * v + 4])}}}")
        else:
            pk = k.regs("b32", 16)
            for t in range(16):
                k(f"cvt.rn.bf16x2.f32 {pk[t]}, {ov[2 * t + 1]}, {ov[2 * t]}")
            for v in range(4):
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
