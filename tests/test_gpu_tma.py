"""GPU parity for the bulk-async transport nodes lowered by the generic path.

Every box copy runs as real ``cp.async.bulk`` copies completing on the IR's
mbarrier and must equal the oracle bit for bit (zero fill, swizzles, f32 /
bf16 / f16 / f64, rank-2 and rank-3 views); the m02-style matmul fed by box
copies must equal the oracle's K-order f32 sums bit for bit.  The kernel's
own checks turn a misaligned box into ``emmy_err`` 0x305 without issuing the
copy, and a wait nothing completes gives up after its limit with 0x304; the
context stays usable after both."""

import numpy as np
import pytest

from oracle.interp import interpret
from ptxgen import irgen
from ptxgen.loader import load_kernel_data

from tests.tma_cases import BOX_CASES, box_case, box_inputs, box_reference, unarrived_wait

pytestmark = pytest.mark.gpu


def _run(spec, inputs):
    from ptxgen.runtime import run_kernel
    return run_kernel(spec, {k: v.copy() for k, v in inputs.items()})


@pytest.mark.parametrize("case", BOX_CASES, ids=lambda c: f"{c[0]}-{c[1]}-{c[8]}-{c[9]}")
def test_box_copy_bitexact(case):
    spec = box_case(case)
    x = box_inputs(spec, seed=5)
    want = interpret(spec, {"x0": x["x0"].copy()})["out"]
    got = _run(spec, x)["out"]
    assert np.array_equal(got.view(np.uint8), want.view(np.uint8))
    assert np.array_equal(got, box_reference(case, x["x0"]))


@pytest.mark.parametrize("idx", [1, 6, 3])
def test_box_copy_rank3_view(idx):
    case = BOX_CASES[idx]
    if case[2] % 2 or case[4] % 2 or case[8] % 2:
        case = case[:8] + (case[8] + 1,) + case[9:]
    spec = box_case(case, view3=True, name="tb3")
    x = box_inputs(spec, seed=6)
    got = _run(spec, x)["out"]
    assert np.array_equal(got, box_reference(case, x["x0"]))


def test_box_copy_with_setmaxnreg_node():
    spec = box_case(BOX_CASES[5], maxnreg=64, name="tbreg")
    x = box_inputs(spec, seed=7)
    assert np.array_equal(_run(spec, x)["out"], box_reference(BOX_CASES[5], x["x0"]))


@pytest.mark.parametrize("mnk", [(64, 96, 48), (128, 128, 256), (256, 64, 1024)])
def test_matmul_tma_bitexact(mnk):
    m, n, k = mnk
    spec = load_kernel_data(*irgen.matmul_tma(m, n, k), f"mt{m}")
    rng = np.random.default_rng(m + n + k)
    a = rng.standard_normal((m, k)).astype(np.float32)
    b = rng.standard_normal((k, n)).astype(np.float32)
    want = interpret(spec, {"x0": a.copy(), "x1": b.copy()})["matmul"]
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    assert np.array_equal(got, want)


def test_matmul_tma_repeated_launches():
    """The mbarrier is initialised by every launch and its phases counted
    from 0 again: three launches on the same buffers give the same C."""
    from ptxgen.runtime import PreparedKernel
    spec = load_kernel_data(*irgen.matmul_tma(128, 64, 512), "mtr")
    rng = np.random.default_rng(8)
    a = rng.standard_normal((128, 512)).astype(np.float32)
    b = rng.standard_normal((512, 64)).astype(np.float32)
    want = interpret(spec, {"x0": a.copy(), "x1": b.copy()})["matmul"]
    pk = PreparedKernel(spec)
    try:
        pk.upload({"x0": a, "x1": b})
        for _ in range(3):
            pk.launch()
            pk.check_errors()
            assert np.array_equal(pk.download()["matmul"], want)
    finally:
        pk.close()


def test_misaligned_box_is_reported_and_skipped():
    """Inner coordinate 2 floats (8 bytes) off the 16-byte grid: the kernel's
    check skips the copy, completes its bytes on the mbarrier (no wait is
    left hanging) and reports 0x305; a correct kernel then runs."""
    from ptxgen.runtime import EmmyError
    case = ("f32", "NONE", 32, 32, 8, 8, 2, 2, 0, 2)
    spec = box_case(case, name="tbbad")
    with pytest.raises(EmmyError, match="0x305"):
        _run(spec, box_inputs(spec))
    good = box_case(BOX_CASES[0], name="tbgood")
    x = box_inputs(good)
    assert np.array_equal(_run(good, x)["out"], box_reference(BOX_CASES[0], x["x0"]))


def test_unarrived_wait_gives_up_and_reports():
    """Nothing arrives on the mbarrier: each lane's wait ends after its 2 s
    limit with 0x304 and the kernel finishes (out = x); the context stays
    usable."""
    from ptxgen.runtime import EmmyError, PreparedKernel
    spec = unarrived_wait()
    x = np.arange(64, dtype=np.float32)
    pk = PreparedKernel(spec)
    try:
        pk.upload({"x0": x})
        pk.launch()
        with pytest.raises(EmmyError, match="0x304"):
            pk.check_errors()
        assert np.array_equal(pk.download()["out"], x)
    finally:
        pk.close()
    good = box_case(BOX_CASES[1], name="tbafter")
    xi = box_inputs(good)
    assert np.array_equal(_run(good, xi)["out"], box_reference(BOX_CASES[1], xi["x0"]))


def _mma_case(m, n, k, dt, seed, **kw):
    from oracle.interp import storage_dtype
    spec = load_kernel_data(*irgen.matmul_mma(m, n, k, dt, **kw), f"mma{m}{n}{k}{dt}")
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(storage_dtype(dt))
    b = rng.standard_normal((k, n)).astype(storage_dtype(dt))
    return spec, a, b


@pytest.mark.parametrize("dt", ["bf16", "f16"])
@pytest.mark.parametrize("mnk", [(64, 32, 16), (128, 64, 96), (256, 128, 512)])
def test_matmul_mma_fragments(mnk, dt):
    """``ldmatrix`` + ``mma.sync`` in the PTX fragment layouts against the
    oracle: any layout slip moves whole products (errors of order one); the
    tensor core's own accumulation stays within 2^-17 of sum |a||b| per
    element."""
    m, n, k = mnk
    spec, a, b = _mma_case(m, n, k, dt, m + k)
    want = interpret(spec, {"x0": a.copy(), "x1": b.copy()})["matmul"]
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    assert np.all(np.abs(got - want) <= 2.0 ** -17 * scale + 1e-30)


def test_matmul_mma_store_guards():
    spec, a, b = _mma_case(128, 64, 64, "bf16", 9, m_valid=100, n_valid=50)
    want = interpret(spec, {"x0": a.copy(), "x1": b.copy()})["matmul"]
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    assert np.all(got[100:] == 0) and np.all(got[:, 50:] == 0)
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    assert np.all(np.abs(got - want) <= 2.0 ** -17 * scale + 1e-30)


def _wgmma_case(m, n, k, dt, bn, groups, seed):
    from oracle.interp import storage_dtype
    spec = load_kernel_data(*irgen.matmul_wgmma(m, n, k, dt, bn, groups),
                            f"wg{m}{n}{k}{dt}{bn}{groups}")
    rng = np.random.default_rng(seed)
    a = rng.standard_normal((m, k)).astype(storage_dtype(dt))
    bt = rng.standard_normal((n, k)).astype(storage_dtype(dt))
    return spec, a, bt


@pytest.mark.parametrize("args", [(128, 64, 128, "bf16", 64, 1), (256, 128, 256, "f16", 128, 2),
                                  (64, 512, 192, "bf16", 256, 1), (128, 64, 64, "bf16", 32, 1)])
def test_matmul_wgmma_on_tcgen05(args):
    """Warpgroup products lowered to tcgen05 (M = 64, accumulators in TMEM,
    16x256b moves to and from the fragment registers) against the oracle,
    within 2^-17 of sum |a||b| per element."""
    m, n, k, dt, bn, g = args
    spec, a, bt = _wgmma_case(m, n, k, dt, bn, g, m + n + k)
    want = interpret(spec, {"x0": a.copy(), "x1": bt.copy()})["matmul"]
    got = _run(spec, {"x0": a, "x1": bt})["matmul"]
    scale = np.abs(a.astype(np.float64)) @ np.abs(bt.astype(np.float64)).T
    assert np.all(np.abs(got - want) <= 2.0 ** -17 * scale + 1e-30)


@pytest.mark.parametrize("args", [(2, 128, 64, "bf16"), (1, 192, 32, "f16"),
                                  (4, 256, 128, "bf16")])
def test_attention_in_fragments(args):
    """Flash attention written with FragmentRowReduce / FragmentApply /
    FragmentRepack over mma.sync cells: against the oracle within 2e-3 of
    the output scale (exp and the tensor core's sums round their own way,
    which can move a P value by one 16-bit step), and against float64."""
    from oracle.interp import storage_dtype
    bh, s, d, dt = args
    spec = load_kernel_data(*irgen.attention_mma(bh, s, d, dt), f"am{bh}{s}{d}{dt}")
    rng = np.random.default_rng(bh + s + d)
    x = {n: rng.standard_normal((bh, s, d)).astype(storage_dtype(dt)) for n in "qkv"}
    want = interpret(spec, {n: a.copy() for n, a in x.items()})["out"]
    got = _run(spec, x)["out"]
    scale = np.abs(want).max()
    assert np.abs(got - want).max() <= 2e-3 * scale
    q, k, v = (x[n].astype(np.float64) for n in "qkv")
    sc = q @ k.transpose(0, 2, 1) / np.sqrt(d)
    p = np.exp(sc - sc.max(-1, keepdims=True))
    ref = (p / p.sum(-1, keepdims=True)) @ v
    assert np.abs(got - ref).max() <= 8e-3 * np.abs(ref).max()


def test_short_dynamic_smem_is_reported_not_faulted():
    """The d = 128 fragment attention lays out 49,160 bytes of shared memory
    (a dynamic pool); meta.json's launch asks for none.  The plan launch
    requests the whole pool, and a launch with less makes every thread
    report 0x308 and return before touching shared memory."""
    from ptxgen.runtime import EmmyError, parse_plan, run_kernel
    from ptxgen.emit import compile_kernel
    from oracle.interp import storage_dtype
    spec = load_kernel_data(*irgen.attention_mma(1, 64, 128, "bf16"), "amsm")
    assert parse_plan(compile_kernel(spec))["smem"] >= 49160
    rng = np.random.default_rng(0)
    x = {n: rng.standard_normal((1, 64, 128)).astype(storage_dtype("bf16")) for n in "qkv"}
    with pytest.raises(EmmyError, match="0x308"):
        run_kernel(spec, {n: a.copy() for n, a in x.items()}, geometry="meta")
    want = interpret(spec, {n: a.copy() for n, a in x.items()})["out"]
    got = _run(spec, x)["out"]
    assert np.abs(got - want).max() <= 2e-3 * np.abs(want).max()


@pytest.mark.parametrize("shape", [(200, 37), (1000, 130)])
def test_carry_scan_bitexact(shape):
    """Carried state (Pre / Carry) in registers: a two-cell recurrence, a
    conditional counter and a carrying loop run twice, bit for bit against
    the oracle."""
    rows, cols = shape
    spec = load_kernel_data(*irgen.carry_scan(rows, cols), f"cs{rows}")
    x = np.random.default_rng(rows).standard_normal((rows, cols)).astype(np.float32)
    want = interpret(spec, {"x": x.copy()})["y"]
    assert np.array_equal(_run(spec, {"x": x})["y"], want)


@pytest.mark.parametrize("every", [1, 3])
def test_matmul_mma_f16_accumulators(every):
    """mma.sync with f16 accumulators, promoted into f32 cells every
    ``every`` K steps (FragmentPromote): against the oracle within 2^-9 of
    sum |a||b| per element (the tensor core rounds its f16 sums its own
    way; a layout slip would be off by whole products)."""
    m, n, k = 128, 64, 160
    spec = load_kernel_data(*irgen.matmul_mma(m, n, k, "f16", promote_every=every),
                            f"mp{every}")
    rng = np.random.default_rng(every)
    a = rng.standard_normal((m, k)).astype(np.float16)
    b = rng.standard_normal((k, n)).astype(np.float16)
    want = interpret(spec, {"x0": a.copy(), "x1": b.copy()})["matmul"]
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    assert np.all(np.abs(got - want) <= 2.0 ** -9 * scale)


def test_random_box_copies_bitexact():
    """40 seeded box copies (every dtype and swizzle, view and box sizes,
    origins off every edge, rank-3 views) bit for bit against the oracle."""
    from tests.tma_cases import random_box_cases
    for i, (case, view3) in enumerate(random_box_cases(40, seed=1)):
        spec = box_case(case, view3=view3, name=f"rb{i}")
        x = box_inputs(spec, seed=2)
        want = interpret(spec, {"x0": x["x0"].copy()})["out"]
        got = _run(spec, x)["out"]
        assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), (i, case, view3)
