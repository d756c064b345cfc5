"""bf16 attention with two query tiles per unit (tcgen05 + TMEM + TMA).

The [B,H,S,D] online-softmax attention of ``tmpl_attn`` for bf16 data with
D = 128, scheduled so that the tensor pipe works on one query tile while
the softmax of the other runs.  A unit is one batch*head and 256 query rows:
tile A (rows 0-127) and tile B (rows 128-255).  Per 128-key block g:

    S_A = Q_A K_g^T   S_B = Q_B K_g^T     (into S_A, S_B in TMEM)
    softmax A -> P_A over S_A             softmax B -> P_B over S_B
    O_A += P_A V_g    O_B += P_B V_g      (P from TMEM, V from smem)

TMEM holds S_A, S_B, O_A, O_B: 4 x 128 columns, all 512.  The MMA thread
issues QK_A(g), QK_B(g), then per block PV_A(g), QK_A(g+1), PV_B(g),
QK_B(g+1): while softmax A works on block g+1 the pipe computes tile B's
products and the other way round, so each tile's chain (S, softmax, P V)
has two blocks' worth of MMA time to hide in.  Both tiles read each K and
V block once: half the K/V traffic per query row of the one-tile kernel.

CTA: 320 threads, one per SM (192 KB of shared memory):
* warp 0 -- allocates TMEM; issues every MMA (converged loop, one elected
  lane), commits to the barriers;
* warp 1 -- TMA: the unit's Q_A and Q_B (64 KB), then per key block K_g and
  V_g (32 KB each; V as stored, an MN-major operand, or V^T from the
  pre-pass with ``EMMY_ATTN_V_DIRECT=0``) into two stages;
* warps 2-5 -- softmax and epilogue of tile A, one thread per query row
  (TMEM lane quarter warp % 4); warps 6-9 -- the same for tile B.  Per
  block: ``tcgen05.ld`` of the row's 128 scores, row max, ``p = exp2(s *
  log2e / c0 - m)`` (one pair in four on the FMA-pipe polynomial), running
  sum, P as packed bf16 over the first 64 score columns, and a rescale of
  O_X in TMEM only when a row's max grew by more than 8 (log2 units); at
  the end ``O_X / l`` to global memory as bf16.

Barriers (the protocol is modelled on the CPU in
``tests/test_attn2q_protocol.py``): ``q_full``/``q_empty`` per unit;
``k_full``/``k_empty``, ``v_full``/``v_empty`` per stage; per tile X
``s_full_X`` (S_X written), ``p_full_X`` (128 arrivals: P_X written),
``pv_done_X`` (O_X += P_X V done: S_X may be overwritten, O_X is stable).
Every wait is bounded by ``%globaltimer`` (``emmy_err`` 0x201 on expiry;
the kernel then drains its MMAs, frees TMEM and returns).

``tmpl_attn``'s pre-pass feeds it K from K^T when the IR gives K
transposed (and V^T with ``EMMY_ATTN_V_DIRECT=0``); any launch
that does not match the plan takes ``tmpl_attn``'s SIMT path.
"""

from __future__ import annotations

import os

from .ptx import Kernel, f32_hex
from .tmpl_attn import (LOG2E, RESCALE_T, _exp2_poly_consts, _exp2_poly_pair, _exp_poly_share,
                        _idesc)
from .tmpl_mma import ERR_WAIT_TIMEOUT, _Ctx, _desc_const

BQ, BKV, D = 128, 128, 128
THREADS = 320
W_MMA, W_TMA = 0, 1
CHUNK = 128 * 128              # one 128-byte-wide column chunk of 128 rows (bytes)
Q_BYTES = 2 * CHUNK            # one 128 x 128 bf16 tile
KV_BYTES = 2 * CHUNK
STAGES = 2
OFF_Q = (0, Q_BYTES)                                   # Q_A, Q_B
OFF_K = tuple(2 * Q_BYTES + st * 2 * KV_BYTES for st in range(STAGES))
OFF_V = tuple(o + KV_BYTES for o in OFF_K)
SMEM_DYN = 2 * Q_BYTES + STAGES * 2 * KV_BYTES + 1024
S_COL = (0, BKV)                                       # S_A, S_B
O_COL = (2 * BKV, 2 * BKV + D)                         # O_A, O_B


def v_direct() -> bool:
    """P V reads V as stored ([keys][D], D contiguous) as an MN-major B
    operand (allowed for 16-bit types), so no pre-pass writes V^T;
    ``EMMY_ATTN_V_DIRECT=0`` restores the transposing pre-pass.  Read when a
    kernel is compiled."""
    return os.environ.get("EMMY_ATTN_V_DIRECT", "1") not in ("0", "")


def eligible(plan) -> bool:
    """bf16, D = 128, whole 256-row units: the two-tile kernel applies."""
    if os.environ.get("EMMY_ATTN_2Q", "1") in ("0", ""):
        return False
    return (plan.tc and plan.dtype == "bf16" and plan.d == D and plan.bkv == BKV
            and plan.s % (2 * BQ) == 0 and plan.atom == 64)


def emit_tc2q(k: Kernel, spec, plan, base, tid, cta, ncta):
    VD = v_direct()
    S, BH = plan.s, plan.bh
    nkv = S // BKV
    qblocks = S // (2 * BQ)
    units = BH * qblocks
    cx = _Ctx(k)
    for nm in ("q_full", "q_empty", "drain"):
        k.shared(f"\t.shared .align 8 .b64 bar_{nm};")
    for nm, cnt in (("k_full", STAGES), ("k_empty", STAGES), ("v_full", STAGES),
                    ("v_empty", STAGES), ("s_full", 2), ("p_full", 2), ("pv_done", 2)):
        k.shared(f"\t.shared .align 8 .b64 bar_{nm}[{cnt}];")
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
    tm = {}
    for t in ("qh", "kh", "vh"):
        r = k.reg("u64")
        k(f"mov.u64 {r}, tmap_{t}")
        k(f"cvta.global.u64 {r}, {r}")
        tm[t] = r

    # ---- set-up: barriers (thread 0), TMEM (warp 0) ----
    skip = k.label("noinit")
    k(f"setp.ne.u32 {p}, {tid}, 0")
    k(f"@{p} bra {skip}")
    for nm in ("q_full", "q_empty", "drain"):
        k(f"mbarrier.init.shared::cta.b64 [bar_{nm}], 1")
    for nm, n, cnt in (("k_full", STAGES, 1), ("k_empty", STAGES, 1), ("v_full", STAGES, 1),
                       ("v_empty", STAGES, 1), ("s_full", 2, 1), ("p_full", 2, 128),
                       ("pv_done", 2, 1)):
        for i in range(n):
            k(f"mbarrier.init.shared::cta.b64 [bar_{nm}+{8 * i}], {cnt}")
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
    k(f"tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [{slot}], 512")
    k("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned")
    k.place(skip2)
    k("tcgen05.fence::before_thread_sync")
    k("barrier.sync 0")
    k("tcgen05.fence::after_thread_sync")
    tmem = k.reg("u32")
    k(f"ld.shared.u32 {tmem}, [tmem_slot]")
    teardown, abort_l = k.label("teardown"), k.label("abort")
    role_tma, role_sm = k.label("rtma"), k.label("rsm")

    def bar_at(name, idx):
        r = k.reg("u32")
        k(f"mov.u32 {r}, bar_{name}")
        if isinstance(idx, int):
            k(f"add.u32 {r}, {r}, {8 * idx}")
        else:
            k(f"mad.lo.u32 {r}, {idx}, 8, {r}")
        return r

    def stage_of(g):
        """(stage, parity of its full phase) of global key block g."""
        st, ph = k.reg("u32"), k.reg("u32")
        k(f"and.b32 {st}, {g}, 1")
        k(f"shr.u32 {ph}, {g}, 1")
        k(f"and.b32 {ph}, {ph}, 1")
        return st, ph

    def flip(ph):
        r = k.reg("u32")
        k(f"xor.b32 {r}, {ph}, 1")
        return r

    def unit_coords(u):
        bh, qb = k.reg("u32"), k.reg("u32")
        k(f"div.u32 {bh}, {u}, {qblocks}")
        k(f"rem.u32 {qb}, {u}, {qblocks}")
        return bh, qb

    # ================= MMA issuer: warp 0 =================
    k(f"setp.ne.u32 {p}, {warp}, {W_MMA}")
    k(f"@{p} bra {role_tma}")
    pm = k.reg("pred")
    k(f"elect.sync _|{pm}, -1")
    kmaj = _desc_const(16, 1024, 2)        # K-major, 128-byte swizzle, 8-row groups 1 KB apart
    id_s, id_o = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {id_s}, {_idesc('f16', BQ, BKV)}")
    # V as stored is MN-major for P V: instruction-descriptor bit 16
    k(f"mov.u32 {id_o}, {_idesc('f16', BQ, D) | ((1 << 16) if VD else 0)}")
    yes = k.reg("pred")
    k(f"setp.eq.u32 {yes}, 0, 0")

    def mkdesc(addr_reg):
        ad, r = k.reg("u32"), k.reg("u64")
        k(f"shr.u32 {ad}, {addr_reg}, 4")
        k(f"and.b32 {ad}, {ad}, 16383")
        k(f"cvt.u64.u32 {r}, {ad}")
        k(f"or.b64 {r}, {r}, 0x{kmaj:016X}")
        return r

    d_base = mkdesc(ring)
    # MN-major, 128-byte swizzle: along D 64 elements per 128-byte row, the
    # next 64 (the second D chunk) 16 KB on (leading offset); along the keys
    # 8 rows of 128 bytes, the next 8 rows 1 KB on (stride offset)
    mnmaj = _desc_const(CHUNK, 1024, 2)
    ad0, d_base_mn = k.reg("u32"), k.reg("u64")
    k(f"shr.u32 {ad0}, {ring}, 4")
    k(f"and.b32 {ad0}, {ad0}, 16383")
    k(f"cvt.u64.u32 {d_base_mn}, {ad0}")
    k(f"or.b64 {d_base_mn}, {d_base_mn}, 0x{mnmaj:016X}")

    def dsc(base_d, off):
        assert off % 16 == 0
        r = k.reg("u64")
        k(f"add.s64 {r}, {base_d}, {off >> 4}")
        return r

    def stage_desc(st_, offs, base_d=None):
        # the stage's operand base: offs[0] for stage 0, offs[1] for stage 1
        r, t = k.reg("u64"), k.reg("u64")
        k(f"mul.wide.u32 {t}, {st_}, {(offs[1] - offs[0]) >> 4}")
        k(f"add.s64 {r}, {base_d or d_base}, {t}")
        return dsc(r, offs[0]) if offs[0] else r

    def issue_qk(x, gg, commit_k, commit_q=None):
        """S_x = Q_x K_gg^T (8 MMAs of K = 16); commits s_full_x, and for
        tile B the K stage (both tiles have read it)."""
        st_, phf = stage_of(gg)
        cx.wait(bar_at("k_full", st_), phf, abort_l)
        # S_x still holds P_x of block gg-1 until that P_x V is done
        notfirst, php = k.reg("pred"), k.reg("u32")
        k(f"setp.ne.u32 {notfirst}, {gg}, 0")
        skipw = k.label("qk_nowait")
        k(f"@!{notfirst} bra {skipw}")
        k(f"sub.u32 {php}, {gg}, 1")
        k(f"and.b32 {php}, {php}, 1")
        cx.wait(bar_at("pv_done", x), php, abort_l)
        k.place(skipw)
        k("tcgen05.fence::after_thread_sync")
        kd = stage_desc(st_, OFF_K)
        s_t = k.reg("u32")
        k(f"add.u32 {s_t}, {tmem}, {S_COL[x]}")
        first = True
        for c in range(2):
            for kk in range(4):
                a_ = dsc(d_base, OFF_Q[x] + c * CHUNK + kk * 32)
                b_ = dsc(kd, c * CHUNK + kk * 32)
                acc = yes
                if first:
                    acc = k.reg("pred")
                    k(f"setp.ne.u32 {acc}, 0, 0")
                    first = False
                k(f"@{pm} tcgen05.mma.cta_group::1.kind::f16 [{s_t}], {a_}, {b_}, {id_s}, {acc}")
        k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
          f"[{bar_at('s_full', x)}]")
        if commit_k:
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('k_empty', st_)}]")
        if commit_q is not None:
            # the unit's Q tiles are free once its last S = Q K^T is done
            k(f"@{commit_q} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[bar_q_empty]")

    def issue_pv(x, gg, jj, commit_v):
        """O_x (+)= P_x V_gg (8 MMAs of K = 16 keys, P from TMEM)."""
        st_, phf = stage_of(gg)
        pph = k.reg("u32")
        k(f"and.b32 {pph}, {gg}, 1")
        cx.wait(bar_at("p_full", x), pph, abort_l)
        cx.wait(bar_at("v_full", st_), phf, abort_l)
        k("tcgen05.fence::after_thread_sync")
        vd = stage_desc(st_, OFF_V, d_base_mn if VD else None)
        o_t = k.reg("u32")
        k(f"add.u32 {o_t}, {tmem}, {O_COL[x]}")
        firstb = k.reg("pred")
        k(f"setp.ne.u32 {firstb}, {jj}, 0")
        first = True
        for c in range(2):
            for kk in range(4):
                a_ = k.reg("u32")
                # keys c*64 + kk*16 .. +15: packed two per column from S_x's first
                k(f"add.u32 {a_}, {tmem}, {S_COL[x] + c * 32 + kk * 8}")
                # keys c*64 + kk*16 .. +15: V [keys][D] rows (MN-major) or
                # V^T [D][keys] columns (K-major)
                b_ = dsc(vd, (c * 4 + kk) * 2048 if VD else c * CHUNK + kk * 32)
                acc = firstb if first else yes
                first = False
                k(f"@{pm} tcgen05.mma.cta_group::1.kind::f16 [{o_t}], [{a_}], {b_}, {id_o}, {acc}")
        k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
          f"[{bar_at('pv_done', x)}]")
        if commit_v:
            k(f"@{pm} tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 "
              f"[{bar_at('v_empty', st_)}]")

    uit, g, u, j = (k.reg("u32") for _ in range(4))
    k(f"mov.u32 {uit}, 0")
    k(f"mov.u32 {g}, 0")
    k(f"mov.u32 {u}, {cta}")
    ml, me, mj = k.label("m_unit"), k.label("m_unitend"), k.label("m_kv")
    k.place(ml)
    k(f"setp.ge.u32 {p}, {u}, {units}")
    k(f"@{p} bra {me}")
    phq = k.reg("u32")
    k(f"and.b32 {phq}, {uit}, 1")
    cx.wait("bar_q_full", phq, abort_l)
    one_blk = k.reg("pred")
    k(f"setp.eq.u32 {one_blk}, 0, {0 if nkv == 1 else 1}")
    issue_qk(0, g, False)
    qlast = k.reg("pred")
    k(f"and.pred {qlast}, {pm}, {one_blk}")
    issue_qk(1, g, True, qlast)
    k(f"mov.u32 {j}, 0")
    k.place(mj)
    gn = k.reg("u32")
    k(f"add.u32 {gn}, {g}, 1")
    more, last2 = k.reg("pred"), k.reg("pred")
    k(f"setp.lt.u32 {more}, {j}, {nkv - 1}")          # a next block exists
    k(f"setp.eq.u32 {last2}, {j}, {nkv - 2}")          # the next block is the unit's last
    issue_pv(0, g, j, False)
    nqa = k.label("m_noqa")
    k(f"@!{more} bra {nqa}")
    issue_qk(0, gn, False)
    k.place(nqa)
    issue_pv(1, g, j, True)
    nqb = k.label("m_noqb")
    k(f"@!{more} bra {nqb}")
    ql2 = k.reg("pred")
    k(f"and.pred {ql2}, {pm}, {last2}")
    issue_qk(1, gn, True, ql2)
    k.place(nqb)
    k(f"mov.u32 {g}, {gn}")
    k(f"add.u32 {j}, {j}, 1")
    k(f"setp.lt.u32 {p}, {j}, {nkv}")
    k(f"@{p} bra {mj}")
    k(f"add.u32 {uit}, {uit}, 1")
    k(f"add.u32 {u}, {u}, {ncta}")
    k(f"bra.uni {ml}")
    k.place(me)
    k(f"bra.uni {teardown}")

    # ================= TMA producer: warp 1 =================
    k.place(role_tma)
    k(f"setp.ne.u32 {p}, {warp}, {W_TMA}")
    k(f"@{p} bra {role_sm}")
    pe = k.reg("pred")
    k(f"elect.sync _|{pe}, -1")
    uit1, g1, u1 = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {uit1}, 0")
    k(f"mov.u32 {g1}, 0")
    k(f"mov.u32 {u1}, {cta}")
    pl, pend = k.label("p_unit"), k.label("p_unitend")
    k.place(pl)
    k(f"setp.ge.u32 {p}, {u1}, {units}")
    k(f"@{p} bra {pend}")
    bh, qb = unit_coords(u1)
    qrow = k.reg("u32")
    k(f"mul.lo.u32 {qrow}, {qb}, {2 * BQ}")
    phe = k.reg("u32")
    k(f"and.b32 {phe}, {uit1}, 1")
    k(f"xor.b32 {phe}, {phe}, 1")
    cx.wait("bar_q_empty", phe, abort_l)
    k(f"@{pe} mbarrier.arrive.expect_tx.shared::cta.b64 _, [bar_q_full], {2 * Q_BYTES}")
    for x in range(2):
        rr = k.reg("u32")
        k(f"add.u32 {rr}, {qrow}, {x * BQ}")
        for c in range(2):
            dst, cc = k.reg("u32"), k.reg("u32")
            k(f"add.u32 {dst}, {ring}, {OFF_Q[x] + c * CHUNK}")
            k(f"mov.u32 {cc}, {c * 64}")
            k(f"@{pe} cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm['qh']}, {{{cc}, {rr}, {bh}}}], [bar_q_full]")
    j1 = k.reg("u32")
    k(f"mov.u32 {j1}, 0")
    pj = k.label("p_kv")
    k.place(pj)
    st, phf = stage_of(g1)
    phe2 = flip(phf)
    krow = k.reg("u32")
    k(f"mul.lo.u32 {krow}, {j1}, {BKV}")
    for nm, offs, tmn in (("k", OFF_K, "kh"), ("v", OFF_V, "vh")):
        cx.wait(bar_at(f"{nm}_empty", st), phe2, abort_l)
        fb = bar_at(f"{nm}_full", st)
        k(f"@{pe} mbarrier.arrive.expect_tx.shared::cta.b64 _, [{fb}], {KV_BYTES}")
        sbase = k.reg("u32")
        k(f"mad.lo.u32 {sbase}, {st}, {offs[1] - offs[0]}, {ring}")
        for c in range(2):
            dst, c0, c1 = k.reg("u32"), k.reg("u32"), k.reg("u32")
            k(f"add.u32 {dst}, {sbase}, {offs[0] + c * CHUNK}")
            if nm == "k" or VD:
                # K or V [keys, D]: D chunk c, key rows krow .. +127
                k(f"mov.u32 {c0}, {c * 64}")
                k(f"mov.u32 {c1}, {krow}")
            else:
                # V^T [D, keys]: key chunk c, D rows 0 .. 127
                k(f"add.u32 {c0}, {krow}, {c * 64}")
                k(f"mov.u32 {c1}, 0")
            k(f"@{pe} cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
              f"[{dst}], [{tm[tmn]}, {{{c0}, {c1}, {bh}}}], [{fb}]")
    k(f"add.u32 {g1}, {g1}, 1")
    k(f"add.u32 {j1}, {j1}, 1")
    k(f"setp.lt.u32 {p}, {j1}, {nkv}")
    k(f"@{p} bra {pj}")
    k(f"add.u32 {uit1}, {uit1}, 1")
    k(f"add.u32 {u1}, {u1}, {ncta}")
    k(f"bra.uni {pl}")
    k.place(pend)
    k(f"bra.uni {teardown}")

    # ================= softmax + epilogue: warps 2-5 (tile A), 6-9 (tile B) ==========
    k.place(role_sm)
    quad, row, xt = k.reg("u32"), k.reg("u32"), k.reg("u32")
    k(f"and.b32 {quad}, {warp}, 3")
    k(f"mad.lo.u32 {row}, {quad}, 32, {lane}")
    k(f"sub.u32 {xt}, {warp}, 2")
    k(f"shr.u32 {xt}, {xt}, 2")                       # 0: tile A, 1: tile B
    lane_off = k.reg("u32")
    k(f"mul.lo.u32 {lane_off}, {quad}, {32 << 16}")
    s_row, o_row = k.reg("u32"), k.reg("u32")
    k(f"add.u32 {s_row}, {tmem}, {lane_off}")
    k(f"mad.lo.u32 {s_row}, {xt}, {BKV}, {s_row}")    # S_A at 0, S_B at 128
    k(f"add.u32 {o_row}, {tmem}, {lane_off}")
    k(f"add.u32 {o_row}, {o_row}, {O_COL[0]}")
    k(f"mad.lo.u32 {o_row}, {xt}, {D}, {o_row}")      # O_A at 256, O_B at 384
    sfull, pfull, pvd = bar_at("s_full", xt), bar_at("p_full", xt), bar_at("pv_done", xt)
    cr = k.reg("f32")
    k(f"ld.global.nc.f32 {cr}, [{base[plan.scale]}]")
    v1, sc2 = k.reg("f32"), k.reg("f32")
    k(f"rcp.rn.f32 {v1}, {cr}")
    k(f"mul.rn.f32 {sc2}, {v1}, {f32_hex(LOG2E)}")   # scores to log2 units
    poly = _exp_poly_share()
    pconsts = _exp2_poly_consts(k) if poly else None
    g3, u3 = k.reg("u32"), k.reg("u32")
    k(f"mov.u32 {g3}, 0")
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
    k(f"and.b32 {ph5}, {g3}, 1")
    cx.wait(sfull, ph5, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    # pass 1: the row max, 64 scores at a time (a thread keeps at most 64
    # scores live: with 10 warps, 3 share a sub-partition's 16K registers)
    HALF = BKV // 2
    mx = k.regs("f32", 4)
    for h in range(2):
        sv = k.regs("f32", HALF)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {s_row}, {h * HALF}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{HALF}.b32 {{{', '.join(sv)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        rest = sv
        if h == 0:
            for i in range(4):
                k(f"mov.f32 {mx[i]}, {sv[i]}")
            rest = sv[4:]
        for i in range(0, len(rest) - 1, 2):
            c = mx[(i // 2) % 4]
            k(f"max.f32 {c}, {c}, {rest[i]}, {rest[i + 1]}")
    mb = k.reg("f32")
    k(f"max.f32 {mb}, {mx[0]}, {mx[1]}, {mx[2]}")
    k(f"max.f32 {mb}, {mb}, {mx[3]}")
    # the scale sc2 > 0 is monotone: max(s) * sc2 == max(s * sc2) exactly
    k(f"mul.rn.f32 {mb}, {mb}, {sc2}")
    pnot0 = k.reg("pred")
    k(f"setp.ne.u32 {pnot0}, {j3}, 0")
    need, thr = k.reg("pred"), k.reg("f32")
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
    # p = exp2(s * sc2 - m): packed f32x2 FMAs, sums in four partials, P as
    # packed bf16 pairs
    sc2x2, negm2, negm = k.reg("b64"), k.reg("b64"), k.reg("f32")
    k(f"neg.f32 {negm}, {m_run}")
    k(f"mov.b64 {sc2x2}, {{{sc2}, {sc2}}}")
    k(f"mov.b64 {negm2}, {{{negm}, {negm}}}")
    acc2 = k.regs("b64", 4)
    zf = k.reg("f32")
    k(f"mov.f32 {zf}, {f32_hex(0.0)}")
    for i in range(4):
        k(f"mov.b64 {acc2[i]}, {{{zf}, {zf}}}")
    # pass 2, per half: reload the scores, exponentials, P as packed bf16
    # over the first 64 score columns (keys 2c, 2c+1 in column c: half 0
    # writes columns 0-31, whose scores it has just read, half 1 columns
    # 32-63, whose scores half 0 read)
    for h in range(2):
        sv = k.regs("f32", HALF)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {s_row}, {h * HALF}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x{HALF}.b32 {{{', '.join(sv)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        pk = k.regs("b32", HALF // 2)
        for t in range(0, HALF, 2):
            pr = k.reg("b64")
            k(f"mov.b64 {pr}, {{{sv[t]}, {sv[t + 1]}}}")
            k(f"fma.rn.f32x2 {pr}, {pr}, {sc2x2}, {negm2}")
            if (t // 2) % 4 < poly:
                ea, eb = _exp2_poly_pair(k, pr, pconsts)
            else:
                ea, eb = k.reg("f32"), k.reg("f32")
                k(f"mov.b64 {{{ea}, {eb}}}, {pr}")
                k(f"ex2.approx.ftz.f32 {ea}, {ea}")
                k(f"ex2.approx.ftz.f32 {eb}, {eb}")
            k(f"mov.b64 {pr}, {{{ea}, {eb}}}")
            acc = acc2[(t // 2) % 4]
            k(f"add.rn.f32x2 {acc}, {acc}, {pr}")
            k(f"cvt.rn.bf16x2.f32 {pk[t // 2]}, {eb}, {ea}")
        tad2 = k.reg("u32")
        k(f"add.u32 {tad2}, {s_row}, {h * HALF // 2}")
        k(f"tcgen05.st.sync.aligned.32x32b.x{HALF // 2}.b32 [{tad2}], {{{', '.join(pk)}}}")
        # the next half's reload must not see these stores land on its scores:
        # half 1 reads columns 64-127, half 0 wrote 0-31 -- disjoint
    for i in range(1, 4):
        k(f"add.rn.f32x2 {acc2[0]}, {acc2[0]}, {acc2[i]}")
    sa, sb_ = k.reg("f32"), k.reg("f32")
    k(f"mov.b64 {{{sa}, {sb_}}}, {acc2[0]}")
    k(f"add.rn.f32 {sa}, {sa}, {sb_}")
    k(f"add.rn.f32 {l_run}, {l_run}, {sa}")
    k("tcgen05.wait::st.sync.aligned")
    # O_X is touched only when some row of this warp moved its max; the
    # previous P_X V must be done first
    nor2 = k.label("noorescale")
    k(f"@!{anyn} bra {nor2}")
    k(f"@!{pnot0} bra {nor2}")
    php = k.reg("u32")
    k(f"sub.u32 {php}, {g3}, 1")
    k(f"and.b32 {php}, {php}, 1")
    cx.wait(pvd, php, abort_l)
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
    k.place(nor2)
    k("tcgen05.fence::before_thread_sync")
    k(f"mbarrier.arrive.shared::cta.b64 _, [{pfull}]")
    k(f"add.u32 {g3}, {g3}, 1")
    k(f"add.u32 {j3}, {j3}, 1")
    k(f"setp.lt.u32 {p}, {j3}, {nkv}")
    k(f"@{p} bra {sj}")
    # epilogue: the unit's last P_X V done, out = O_X / l as bf16
    phl = k.reg("u32")
    k(f"sub.u32 {phl}, {g3}, 1")
    k(f"and.b32 {phl}, {phl}, 1")
    cx.wait(pvd, phl, abort_l)
    k("bar.warp.sync -1")
    k("tcgen05.fence::after_thread_sync")
    rl = k.reg("f32")
    k(f"rcp.rn.f32 {rl}, {l_run}")
    bh3, qb3 = unit_coords(u3)
    grow = k.reg("u32")
    k(f"mad.lo.u32 {grow}, {bh3}, {S}, {row}")
    k(f"mad.lo.u32 {grow}, {qb3}, {2 * BQ}, {grow}")
    k(f"mad.lo.u32 {grow}, {xt}, {BQ}, {grow}")
    k(f"mul.lo.u32 {grow}, {grow}, {D}")
    optr = k.addr(base[plan.out], grow, 2)
    for c0 in range(0, D, 32):
        ov = k.regs("f32", 32)
        tad = k.reg("u32")
        k(f"add.u32 {tad}, {o_row}, {c0}")
        k(f"tcgen05.ld.sync.aligned.32x32b.x32.b32 {{{', '.join(ov)}}}, [{tad}]")
        k("tcgen05.wait::ld.sync.aligned")
        for t in range(32):
            k(f"mul.rn.f32 {ov[t]}, {ov[t]}, {rl}")
        po = k.regs("b32", 16)
        for t in range(16):
            k(f"cvt.rn.bf16x2.f32 {po[t]}, {ov[2 * t + 1]}, {ov[2 * t]}")
        for v in range(4):
            k(f"st.global.v4.b32 [{optr}+{(c0 + 8 * v) * 2}], {{{', '.join(po[4 * v:4 * v + 4])}}}")
    k("tcgen05.fence::before_thread_sync")
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
    # after an abort, let the TMA copies in flight land (bounded: 50 ms)
    t0, t1 = k.reg("u64"), k.reg("u64")
    lw = k.label("drain")
    k(f"mov.u64 {t0}, %globaltimer")
    k.place(lw)
    k(f"mov.u64 {t1}, %globaltimer")
    k(f"sub.u64 {t1}, {t1}, {t0}")
    k(f"setp.lt.u64 {p}, {t1}, 50000000")
    k(f"@{p} bra {lw}")
    k.place(drained)
    # the issuing lane (lane 0 of warp 0, the elect.sync leader): every MMA
    # it issued has completed before TMEM is freed (bounded)
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
    k(f"tcgen05.dealloc.cta_group::1.sync.aligned.b32 {tmem}, 512")
    k.place(fin)
