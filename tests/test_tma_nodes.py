"""The bulk-async transport nodes on the CPU: IR round trip, the oracle's
box copy against numpy (zero fill, every swizzle, rank-2 and rank-3 views),
its error cases, and the CUDA lowering's compile-time checks and assembly.

The reference lists these nodes (``TASK.md:121-127``) but neither interprets
nor lowers them, so there is no reference output to pin: the oracle states
the meaning and the GPU tests hold the CUDA lowering to it bit for bit."""

import shutil
import subprocess

import numpy as np
import pytest

from oracle.interp import interpret
from ptxgen import ir, irgen
from ptxgen.emit import compile_kernel
from ptxgen.generic import emit_generic
from ptxgen.lower import LowerError
from ptxgen.loader import load_kernel_data
from ptxgen.runtime import parse_plan

from tests.tma_cases import BOX_CASES, box_case, box_inputs, box_reference, unarrived_wait


def test_repr_round_trip():
    nodes = [ir.TmaDescriptor(name="d", src_buf="x0", src_shape=(8, 16), box_extents=(4, 8),
                              swizzle="B32", dtype="f32"),
             ir.TmaLoad(smem="t", smem_index=irgen.L(0), desc="d",
                        coords=(irgen.V("r"), irgen.L(0)), mbar="bar", mbar_slot=irgen.L(1)),
             ir.MbarrierInit(mbar="bar", count=irgen.L(1), slot=None),
             ir.MbarrierArriveExpectTx(mbar="bar", bytes_=irgen.L(128), slot=irgen.L(0)),
             ir.MbarrierArrive(mbar="bar", slot=None),
             ir.MbarrierWait(mbar="bar", phase=irgen.V("k"), slot=irgen.L(0)),
             ir.SetMaxNReg(count=96, direction="dec")]
    for n in nodes:
        assert ir.parse_stmt(repr(n)) == n


@pytest.mark.parametrize("view3", [False, True])
@pytest.mark.parametrize("case", BOX_CASES, ids=lambda c: f"{c[0]}-{c[1]}-{c[8]}-{c[9]}")
def test_oracle_box_copy(case, view3):
    if view3 and (case[2] % 2 or case[4] % 2 or case[8] % 2):
        pytest.skip("rank-3 view needs even rows, box rows and row offset")
    spec = box_case(case, view3=view3)
    x = box_inputs(spec)
    out = interpret(spec, {"x0": x["x0"].copy()})["out"]
    assert np.array_equal(out, box_reference(case, x["x0"]))


def test_oracle_swizzle_moves_chunks():
    """Under B128 the box's 16-byte chunks really move in shared memory: an
    IR that reads the box back without undoing the swizzle gets a
    permutation of it, not the box."""
    from oracle.interp import tma_swizzle_perm
    perm = tma_swizzle_perm((8, 32), 4, "B128")
    assert sorted(perm) == list(range(256)) and not np.array_equal(perm, np.arange(256))
    assert list(perm[32:36]) == [36, 37, 38, 39]          # row 1, chunk 0 -> chunk 1
    assert tma_swizzle_perm((8, 32), 4, "NONE") is None


def test_oracle_rejects_misaligned_inner_coordinate():
    case = ("f32", "NONE", 32, 32, 8, 8, 2, 2, 0, 2)      # 2 floats = 8 bytes
    spec = box_case(case)
    with pytest.raises(ValueError, match="16-byte"):
        interpret(spec, box_inputs(spec))


@pytest.mark.parametrize("kw, msg", [
    (dict(bc=6), "multiples of 16 bytes"),                # 24-byte box row
    (dict(bc=16, swizzle="B32"), "32-byte box row"),      # 64-byte row under B32
    (dict(br=300, nbr=1), "1..256"),
])
def test_lowering_rejects_bad_descriptors(kw, msg):
    a = dict(rows=32, cols=32, br=8, bc=8, nbr=2, nbc=2, dtype="f32", swizzle="NONE")
    a.update(kw)
    if a["br"] > a["rows"]:
        a["rows"] = a["br"]
    gm = irgen.tma_box_copy(**a)
    spec = load_kernel_data(gm[0], gm[1], "bad")
    with pytest.raises(LowerError, match=msg):
        emit_generic(spec)


def test_tma_kernels_take_the_generic_path():
    for spec in (box_case(BOX_CASES[0]),
                 load_kernel_data(*irgen.matmul_tma(64, 96, 48), "mt")):
        plan = parse_plan(compile_kernel(spec))
        assert plan["kind"] == "generic"


def test_setmaxnreg_lowers_to_nothing():
    ptx = compile_kernel(box_case(BOX_CASES[0], maxnreg=64))
    assert "setmaxnreg" not in ptx
    assert "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes" in ptx
    assert "mbarrier.try_wait.parity" in ptx


def test_matmul_tma_oracle():
    spec = load_kernel_data(*irgen.matmul_tma(64, 96, 48), "mt")
    rng = np.random.default_rng(3)
    a = rng.standard_normal((64, 48)).astype(np.float32)
    b = rng.standard_normal((48, 96)).astype(np.float32)
    c = interpret(spec, {"x0": a, "x1": b})["matmul"]
    ref = np.zeros((64, 96), np.float32)
    for kk in range(48):                                   # K order, f32 per op
        ref = (ref + (b[kk][None, :] * a[:, kk][:, None]).astype(np.float32)).astype(np.float32)
    assert np.array_equal(c, ref)


def test_unarrived_wait_is_a_no_op_in_the_oracle():
    spec = unarrived_wait()
    x = np.arange(64, dtype=np.float32)
    assert np.array_equal(interpret(spec, {"x0": x})["out"], x)


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
def test_tma_kernels_assemble(tmp_path):
    specs = [box_case(c, name=f"tb{i}") for i, c in enumerate(BOX_CASES)]
    specs += [box_case(BOX_CASES[6], view3=True, name="tb3d"),
              load_kernel_data(*irgen.matmul_tma(64, 96, 48), "mt"), unarrived_wait()]
    for i, spec in enumerate(specs):
        f = tmp_path / f"k{i}.ptx"
        f.write_text(compile_kernel(spec))
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(f)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


# -- warp-level tensor-core fragments ------------------------------------------

def _mma_inputs(m, n, k, dt, seed=0):
    from oracle.interp import storage_dtype
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((m, k)).astype(storage_dtype(dt)),
            rng.standard_normal((k, n)).astype(storage_dtype(dt)))


def _mma_steps_reference(a, b, guard=None):
    """C summed one K step of 16 at a time: exact products of the step plus
    the running C, rounded once to f32 per step."""
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    c = np.zeros((a.shape[0], b.shape[1]), np.float32)
    for k0 in range(0, a.shape[1], 16):
        c = (a64[:, k0:k0 + 16] @ b64[k0:k0 + 16] + c).astype(np.float32)
    if guard:
        c[guard[0]:] = 0
        c[:, guard[1]:] = 0
    return c


def test_mma_layout_covers_each_cell_once():
    from oracle.interp import mma_layout
    for role, shape in (("a", (16, 16)), ("b", (16, 8)), ("c", (16, 8))):
        r, c = mma_layout(role)
        cells = set(zip(r.ravel().tolist(), c.ravel().tolist()))
        assert len(cells) == r.size == shape[0] * shape[1]


@pytest.mark.parametrize("dt", ["bf16", "f16"])
def test_oracle_matmul_mma(dt):
    spec = load_kernel_data(*irgen.matmul_mma(128, 64, 96, dt), "mm")
    a, b = _mma_inputs(128, 64, 96, dt)
    got = interpret(spec, {"x0": a, "x1": b})["matmul"]
    assert np.array_equal(got, _mma_steps_reference(a, b))


def test_oracle_matmul_mma_guards():
    spec = load_kernel_data(*irgen.matmul_mma(128, 64, 32, "bf16", m_valid=100, n_valid=50),
                            "mmg")
    a, b = _mma_inputs(128, 64, 32, "bf16", 1)
    got = interpret(spec, {"x0": a, "x1": b})["matmul"]
    assert np.array_equal(got, _mma_steps_reference(a, b, (100, 50)))


def test_fragment_nodes_round_trip():
    nodes = [ir.RegFragment(name="fa", role="a", shape="m16n8k16", dtype="bf16", count=1,
                            nregs=4),
             ir.LdmatrixLoad(frag="fb", src_buffer="s", src_index=(irgen.L(0), irgen.L(8)),
                             role="b", b_trans=True, fragment_index=irgen.L(1)),
             ir.MmaSyncPtx(c_frag="fc[1]", a_frag="fa", b_frag="fb[1]"),
             ir.RegStore(dst_buffer="o", dst_index=(irgen.V("r"), irgen.L(0)), frag="fc",
                         fragment_index=irgen.L(1), m_guard=irgen.L(100))]
    for n in nodes:
        assert ir.parse_stmt(repr(n)) == n


def test_fragment_options_not_lowered_are_refused():
    gm = irgen.matmul_mma(64, 32, 16)
    spec = load_kernel_data(gm[0], gm[1], "mmopt")
    body = list(spec.op.body[0].body)
    for i, st in enumerate(body):
        if isinstance(st, ir.RegStore):
            st.epilogue = "relu"
            break
    spec.op.body[0].body = tuple(body)
    with pytest.raises(LowerError, match="epilogue"):
        emit_generic(spec)


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
def test_fragment_kernels_assemble(tmp_path):
    for i, gm in enumerate((irgen.matmul_mma(128, 64, 64, "bf16"),
                            irgen.matmul_mma(64, 96, 32, "f16", m_valid=50, n_valid=70))):
        f = tmp_path / f"m{i}.ptx"
        ptx = compile_kernel(load_kernel_data(gm[0], gm[1], f"m{i}"))
        assert "ldmatrix.sync.aligned.m8n8.x4.shared.b16" in ptx
        assert "ldmatrix.sync.aligned.m8n8.x2.trans.shared.b16" in ptx
        assert "mma.sync.aligned.m16n8k16.row.col.f32" in ptx
        f.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(f)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


# -- warpgroup products ------------------------------------------------------------

def _wgmma_inputs(m, n, k, dt, seed=0):
    from oracle.interp import storage_dtype
    rng = np.random.default_rng(seed)
    return (rng.standard_normal((m, k)).astype(storage_dtype(dt)),
            rng.standard_normal((n, k)).astype(storage_dtype(dt)))


def _wgmma_reference(a, bt):
    """One rounding to f32 per k16 product, in K order."""
    a64, b64 = a.astype(np.float64), bt.astype(np.float64)
    c = np.zeros((a.shape[0], bt.shape[0]), np.float32)
    for k0 in range(0, a.shape[1], 16):
        c = (a64[:, k0:k0 + 16] @ b64[:, k0:k0 + 16].T + c).astype(np.float32)
    return c


def test_wgmma_c_layout_covers_the_tile_once():
    from oracle.interp import wgmma_c_layout
    for n in (8, 64, 256):
        r, c = wgmma_c_layout(n)
        cells = set(zip(r.ravel().tolist(), c.ravel().tolist()))
        assert len(cells) == r.size == 64 * n


@pytest.mark.parametrize("args", [(128, 64, 128, "bf16", 64, 1), (128, 128, 64, "f16", 128, 2),
                                  (64, 256, 192, "bf16", 256, 1)])
def test_oracle_matmul_wgmma(args):
    m, n, k, dt, bn, g = args
    spec = load_kernel_data(*irgen.matmul_wgmma(m, n, k, dt, bn, g), "wg")
    a, bt = _wgmma_inputs(m, n, k, dt)
    got = interpret(spec, {"x0": a, "x1": bt})["matmul"]
    assert np.array_equal(got, _wgmma_reference(a, bt))


def test_wgmma_nodes_round_trip():
    nodes = [ir.WgmmaDescriptor(name="da", smem="s", smem_index=irgen.L(16), swizzle="B128",
                                lbo_bytes=16, sbo_bytes=1024),
             ir.WgmmaMma(c_frags="fc", b_desc="db", shape="m64n64k16", ab_dtype="bf16",
                         a_desc="da", scale_d=irgen.L(1)),
             ir.WgmmaFence(), ir.WgmmaCommit(), ir.WgmmaWait(group=0)]
    for n in nodes:
        assert ir.parse_stmt(repr(n)) == n


def test_wgmma_lowering_refuses_uncommitted_loops():
    """Products issued in a loop iteration must be committed and waited for
    in it: the accumulators move between registers and TMEM there."""
    gm = irgen.matmul_wgmma(64, 64, 128)
    spec = load_kernel_data(gm[0], gm[1], "wgbad")
    tl = spec.op.body[0]
    body = list(tl.body)
    loop_i = next(i for i, s_ in enumerate(body) if isinstance(s_, ir.StridedLoop))
    lp = body[loop_i]
    lp.body = tuple(s_ for s_ in lp.body if not isinstance(s_, (ir.WgmmaCommit, ir.WgmmaWait)))
    with pytest.raises(LowerError, match="loop iteration"):
        emit_generic(spec)


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
def test_wgmma_kernels_assemble(tmp_path):
    for i, gm in enumerate((irgen.matmul_wgmma(128, 64, 128, "bf16", 64, 1),
                            irgen.matmul_wgmma(128, 128, 64, "f16", 128, 2),
                            irgen.matmul_wgmma(64, 256, 64, "bf16", 256, 1))):
        ptx = compile_kernel(load_kernel_data(gm[0], gm[1], f"w{i}"))
        for op in ("tcgen05.alloc", "tcgen05.mma.cta_group::1.kind::f16", "tcgen05.commit",
                   "tcgen05.st.sync.aligned.16x256b", "tcgen05.ld.sync.aligned.16x256b",
                   "tcgen05.dealloc"):
            assert op in ptx
        f = tmp_path / f"w{i}.ptx"
        f.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(f)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


# -- fragment arithmetic: apply, row reduce, repack ---------------------------------

def _attn_inputs(bh, s, d, dt, seed=0):
    from oracle.interp import storage_dtype
    rng = np.random.default_rng(seed)
    return {x: rng.standard_normal((bh, s, d)).astype(storage_dtype(dt)) for x in "qkv"}


def _attn_f64(x):
    q, k, v = (x[n].astype(np.float64) for n in "qkv")
    sc = q @ k.transpose(0, 2, 1) / np.sqrt(q.shape[-1])
    p = np.exp(sc - sc.max(-1, keepdims=True))
    return (p / p.sum(-1, keepdims=True)) @ v


@pytest.mark.parametrize("args", [(2, 128, 64, "bf16"), (1, 192, 32, "f16"),
                                  (1, 64, 128, "bf16")])
def test_oracle_attention_mma(args):
    """The fragment attention in the oracle against float64 softmax
    attention: P is rounded to the 16-bit type before P V, so the bound is a
    few 16-bit ulps of the output scale."""
    bh, s, d, dt = args
    spec = load_kernel_data(*irgen.attention_mma(bh, s, d, dt), "am")
    x = _attn_inputs(bh, s, d, dt)
    got = interpret(spec, {n: a.copy() for n, a in x.items()})["out"]
    ref = _attn_f64(x)
    assert np.abs(got - ref).max() <= 8e-3 * np.abs(ref).max()


def test_fragment_arith_round_trip():
    nodes = [ir.FragmentApply(out="fs[2]", op="subtract", args=(("a", "b"),), kinds=("row",)),
             ir.FragmentRowReduce(top="t", bot="b", frags=("fs[0]", "fs[1]"), op="maximum"),
             ir.FragmentRepack(frag="fp[1]", srcs=("fs[2]", "fs[3]"), ab_dtype="bf16")]
    for n in nodes:
        assert ir.parse_stmt(repr(n)) == n


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
def test_attention_mma_assembles(tmp_path):
    for i, args in enumerate(((2, 128, 64, "bf16"), (1, 64, 128, "f16"))):
        ptx = compile_kernel(load_kernel_data(*irgen.attention_mma(*args), f"am{i}"))
        assert "shfl.sync.bfly.b32" in ptx and "cvt.rn." in ptx
        f = tmp_path / f"a{i}.ptx"
        f.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(f)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr[-2000:]


def test_generic_plan_requests_the_whole_dynamic_pool():
    """Shared memory above 48 KB goes to a dynamic pool; the plan asks for
    all of it even when meta.json's smem_bytes is 0, and the kernel checks
    the size it was given before any shared access."""
    spec = load_kernel_data(*irgen.attention_mma(1, 64, 128, "bf16"), "amsm")
    assert spec.smem_bytes == 0
    ptx = compile_kernel(spec)
    assert parse_plan(ptx)["smem"] >= 3 * 64 * 128 * 2
    assert ptx.index("%dynamic_smem_size") < ptx.index("emmy_dyn_smem;")


# -- carried state ------------------------------------------------------------------

def carry_scan_reference(x):
    rows, cols = x.shape
    ref = np.zeros((rows, cols + 5), np.float32)
    half = np.float32(0.5)
    for r in range(rows):
        for rep in range(2):
            st0, st1, cnt = np.float32(1), np.float32(1), np.float32(0)
            for c in range(cols):
                ref[r, c] = st1
                n1 = np.float32(np.float32(st0 * half) + np.float32(st1 * x[r, c]))
                st0, st1 = st1, n1
                if x[r, c] > 0:
                    cnt = np.float32(cnt + 1)
            ref[r, cols + 3 + rep] = st1
        ref[r, cols:cols + 3] = [st0, st1, cnt]
    return ref


def test_oracle_carry_scan():
    """Reads within a step see the previous state (st[0] <- st[1] and st[1]
    <- f(st[0], st[1]) use the old values), a cell set under a condition
    keeps its value elsewhere, the carrying loop seeds its cells each time
    it starts, and Pre after the loop reads the final state; the block's
    tail lanes (200 rows, 128 threads) change nothing."""
    spec = load_kernel_data(*irgen.carry_scan(200, 37), "cs")
    x = np.random.default_rng(0).standard_normal((200, 37)).astype(np.float32)
    assert np.array_equal(interpret(spec, {"x": x})["y"], carry_scan_reference(x))


def test_carry_nodes_round_trip_and_assemble(tmp_path):
    for n in (ir.Pre(name="p", carrier="st", index=(irgen.L(1),)),
              ir.Carry(name="st", value="v", index=(irgen.L(1),), seed=1.0, dtype="f32")):
        assert ir.parse_stmt(repr(n)) == n
    if shutil.which("ptxas") is None:
        return
    f = tmp_path / "cs.ptx"
    f.write_text(compile_kernel(load_kernel_data(*irgen.carry_scan(200, 37), "cs")))
    r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(f)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]


def test_carry_seeding_is_outside_the_step():
    """The carrying loop's seeding comes before its head label, not inside
    every step."""
    ptx = compile_kernel(load_kernel_data(*irgen.carry_scan(64, 5), "cs"))
    lines = [ln.strip() for ln in ptx.splitlines()]
    heads = [i for i, ln in enumerate(lines) if ln.startswith("$L_lp_")]
    inner = heads[1]
    seeds = [i for i, ln in enumerate(lines) if ln.startswith("@") and "0f3F800000" in ln]
    assert seeds and all(i < inner for i in seeds)


def test_oracle_f16_accumulators_and_promote():
    """f16 c cells take each k16 product rounded once to f16; every third K
    step FragmentPromote adds them into the f32 cells and clears them."""
    spec = load_kernel_data(*irgen.matmul_mma(128, 64, 160, "f16", promote_every=3), "mp")
    a, b = _mma_inputs(128, 64, 160, "f16", 3)
    got = interpret(spec, {"x0": a, "x1": b})["matmul"]
    a64, b64 = a.astype(np.float64), b.astype(np.float64)
    fc = np.zeros((128, 64), np.float32)
    fh = np.zeros((128, 64), np.float32)
    for i, k0 in enumerate(range(0, 160, 16)):
        fh = (a64[:, k0:k0 + 16] @ b64[k0:k0 + 16] + fh).astype(np.float16).astype(np.float32)
        if i % 3 == 2:
            fc, fh = (fc + fh).astype(np.float32), np.zeros_like(fh)
    assert np.array_equal(got, (fc + fh).astype(np.float32))
    assert ir.parse_stmt(repr(ir.FragmentPromote(dst="fc[1]", src="fh[1]"))) == \
        ir.FragmentPromote(dst="fc[1]", src="fh[1]")


@pytest.mark.parametrize("case, view3", __import__("tests.tma_cases", fromlist=["x"])
                         .random_box_cases(40, seed=1))
def test_oracle_random_box_copies(case, view3):
    spec = box_case(case, view3=view3, name="rb")
    x = box_inputs(spec, seed=2)
    got = interpret(spec, {"x0": x["x0"].copy()})["out"]
    assert np.array_equal(got, box_reference(case, x["x0"]))
