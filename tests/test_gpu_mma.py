"""GPU parity for the tcgen05 3xTF32 matmul template (m01/m02 family).

* plan launch (tcgen05 + TMA path) against the oracle and ``expected.npz``;
* meta.json launch (the SIMT path every other launch takes): bit for bit
  with the oracle for m01, whose IR sums K in order with one rounding per op;
* generated shapes and the BASELINE shapes against float64 numpy with the
  bounds of ``tests/contraction.py``: |got - ref| <= 2^-15 * sum_k |a_ik|
  |b_kj| per element and max|err| <= 1e-4 * max|ref| per block of 16 rows
  (the ``north_star`` 1e-4 relative), which a one-pass TF32 product fails
  (``tests/test_contraction_bounds.py``).
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.interp import interpret, make_inputs
from ptxgen import irgen
from ptxgen.loader import load_kernel, load_kernel_data

from tests.contraction import matmul_check

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden" / "problems"


def _run(spec, inputs, geometry="plan"):
    from ptxgen.runtime import run_kernel
    return run_kernel(spec, {k: v.copy() for k, v in inputs.items()}, geometry=geometry)


def _bound_ok(got, a, b, rows=None):
    ok, elem, block = matmul_check(got, a, b, rows)
    return ok, (elem, block)


@pytest.mark.parametrize("prob", ["m01_matmul_512", "m02_matmul_rect"])
def test_problem_plan(prob):
    pdir = GOLDEN / prob
    meta = json.loads((pdir / "meta.json").read_text())
    spec = load_kernel(next(pdir.glob("*.ir.json")))
    inputs = make_inputs(spec)
    got = _run(spec, inputs)["matmul"]
    ok, rel = _bound_ok(got, inputs["x0"], inputs["x1"])
    assert ok, rel
    exp = np.load(pdir / "expected.npz")["matmul"]
    assert np.allclose(got, exp, rtol=meta["rtol"], atol=meta["atol"])


def test_m01_meta_geometry_bitexact():
    spec = load_kernel(next((GOLDEN / "m01_matmul_512").glob("*.ir.json")))
    inputs = make_inputs(spec)
    want = interpret(spec, {k: v.copy() for k, v in inputs.items()})["matmul"]
    got = _run(spec, inputs, geometry="meta")["matmul"]
    assert np.array_equal(got, want)


def test_m02_meta_geometry():
    spec = load_kernel(next((GOLDEN / "m02_matmul_rect").glob("*.ir.json")))
    inputs = make_inputs(spec)
    want = interpret(spec, {k: v.copy() for k, v in inputs.items()})["matmul"]
    got = _run(spec, inputs, geometry="meta")["matmul"]
    assert np.allclose(got, want, rtol=1e-5, atol=1e-5)


@pytest.mark.parametrize("m,n,k", [(256, 512, 256), (384, 192, 512), (128, 64, 1024)])
def test_matmul_generated(m, n, k):
    spec = load_kernel_data(*irgen.matmul(m, n, k), "mm")
    rng = np.random.default_rng(m + n + k)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    ok, rel = _bound_ok(got, a, b)
    assert ok, rel


def test_splitk_generated():
    spec = load_kernel_data(*irgen.matmul_splitk(256, 256, 1024, slice_k=128), "sk")
    rng = np.random.default_rng(9)
    a = rng.standard_normal((256, 1024)).astype(np.float32)
    b = rng.standard_normal((1024, 256)).astype(np.float32)
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    ok, rel = _bound_ok(got, a, b)
    assert ok, rel


@pytest.mark.parametrize("mnk", [(4736, 2048, 512), (256, 256, 1024)])
def test_splitk_repeated_launches(mnk):
    """Split-K IR adds into a C cleared before every launch.  With the slices
    grouped into one CTA per tile (4736x2048x512: 296 tiles, two full waves
    on 148 SMs) the kernel stores C in full and the launcher skips the
    clearing (plan ``overwrites``); with slices spread over CTAs
    (256x256x1024) it clears C and the kernel reduce-adds.  Three launches
    on the same buffers must each give A.B, not a sum."""
    from ptxgen.runtime import PreparedKernel
    m, n, k = mnk
    spec = load_kernel_data(*irgen.matmul_splitk(m, n, k, slice_k=128), "skr")
    rng = np.random.default_rng(4)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    pk = PreparedKernel(spec)
    try:
        assert ("overwrites" in pk.plan) == (m == 4736)
        pk.upload({"x0": a, "x1": b})
        for _ in range(3):
            pk.launch()
        pk.check_errors()
        got = pk.download()["matmul"]
    finally:
        pk.close()
    rows = np.random.default_rng(5).choice(m, min(m, 64), replace=False)
    ok, rel = _bound_ok(got, a, b, rows)
    assert ok, rel


def test_sliced_k_repeated_launches(monkeypatch):
    """Non-atomic IR whose K is cut into slices of at most 1024 (the opt-in
    for a smaller tensor-core accumulation error): the launcher clears C
    before every launch (plan ``zero``) and the slices reduce-add into it;
    three launches must each give A.B, and the error is the lower one."""
    from ptxgen.runtime import PreparedKernel
    monkeypatch.setenv("EMMY_MATMUL_MAX_SLICE_K", "1024")
    m, n, k = 512, 1024, 8192
    spec = load_kernel_data(*irgen.matmul(m, n, k), "mmslice")
    rng = np.random.default_rng(6)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    pk = PreparedKernel(spec)
    try:
        assert pk.plan["split_k"] > 1 and pk.plan.get("zero") == ["matmul"]
        pk.upload({"x0": a, "x1": b})
        for _ in range(3):
            pk.launch()
        pk.check_errors()
        got = pk.download()["matmul"]
    finally:
        pk.close()
    ok, rel = _bound_ok(got, a, b)
    assert ok and rel[1] <= 2e-5, rel


@pytest.mark.parametrize("shape", ["square", "splitk8"])
def test_baseline_shapes_sampled(shape):
    if shape == "square":
        m = n = k = 8192
        spec = load_kernel_data(*irgen.matmul(m, n, k), "sq")
    else:
        m, n, k = 16384, 4096, 1024
        spec = load_kernel_data(*irgen.matmul_splitk(m, n, k, slice_k=128), "sk8")
    rng = np.random.default_rng(1)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    rows = np.random.default_rng(2).choice(m, 64, replace=False)
    ok, rel = _bound_ok(got, a, b, rows)
    assert ok, rel


@pytest.mark.parametrize("m,n,k,bn,forced", [(1024, 4160, 256, 256, None),
                                             (512, 2496, 512, 256, None),
                                             (1024, 8192, 256, 224, "224"),
                                             (2048, 4096, 256, 160, "160")])
def test_ragged_n_edge(m, n, k, bn, forced, monkeypatch):
    """Tile widths that leave a ragged N edge (4160 = 16 x 256 + 64, 2496 =
    9 x 256 + 192; forced widths 224 and 160 at 8192 and 4096): the edge
    tile's B rows past N load as zeros and its C columns past N are not
    stored."""
    from ptxgen.runtime import PreparedKernel
    if forced:
        monkeypatch.setenv("EMMY_MATMUL_BN", forced)
    else:
        monkeypatch.delenv("EMMY_MATMUL_BN", raising=False)
    spec = load_kernel_data(*irgen.matmul(m, n, k), f"rag{n}{bn}")
    rng = np.random.default_rng(m + n + bn)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    pk = PreparedKernel(spec)
    try:
        assert pk.plan["tile"][1] == bn and n % bn
        pk.upload({"x0": a, "x1": b})
        pk.launch()
        pk.check_errors()
        got = pk.download()["matmul"]
    finally:
        pk.close()
    rows = np.random.default_rng(7).choice(m, 64, replace=False)
    ok, rel = _bound_ok(got, a, b, rows)
    assert ok, rel
    # every column of the last (ragged) tile, all rows of one row block
    ref = a[:128].astype(np.float64) @ b[:, (n // bn) * bn:].astype(np.float64)
    assert np.abs(got[:128, (n // bn) * bn:] - ref).max() <= 1e-4 * np.abs(ref).max()


def test_ragged_n_edge_sliced(monkeypatch):
    """The same ragged edge with K slices reduce-added into a cleared C (the
    opt-in slicing): the overhanging chunks are not reduce-added either."""
    monkeypatch.delenv("EMMY_MATMUL_BN", raising=False)
    monkeypatch.setenv("EMMY_MATMUL_MAX_SLICE_K", "256")
    m, n, k = 1024, 4160, 512
    spec = load_kernel_data(*irgen.matmul(m, n, k), "ragsl")
    rng = np.random.default_rng(8)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    rows = np.random.default_rng(9).choice(m, 64, replace=False)
    ok, rel = _bound_ok(got, a, b, rows)
    assert ok, rel


def test_ragged_n_edge_infinite_operand(monkeypatch):
    """An infinite A element at a ragged shape: its row's outputs are
    recomputed in f32 (+-inf by the sign of B's element, NaN where that is
    0), and the overhanging chunks of the edge tile, whose zero-filled B
    makes inf * 0 = NaN there, are skipped rather than recomputed from B
    columns past N."""
    monkeypatch.delenv("EMMY_MATMUL_BN", raising=False)
    m, n, k = 1024, 4160, 256
    spec = load_kernel_data(*irgen.matmul(m, n, k), "raginf")
    rng = np.random.default_rng(10)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    b[17, 5] = 0.0
    a[900, 17] = np.inf
    got = _run(spec, {"x0": a, "x1": b})["matmul"]
    want = np.where(b[17] > 0, np.inf, np.where(b[17] < 0, -np.inf, np.nan)).astype(np.float32)
    assert np.array_equal(got[900], want, equal_nan=True)
    others = np.delete(np.arange(m), 900)[:: 97]
    ok, rel = _bound_ok(got, a, b, others)
    assert ok, rel


def test_bind_reads_another_kernels_buffer():
    """``PreparedKernel.bind``: a matmul whose A argument is bound to another
    kernel's A buffer reads that buffer -- its tensor maps follow -- and
    closing both kernels frees each buffer once."""
    from ptxgen.runtime import PreparedKernel
    m, n, k = 256, 512, 256
    spec = load_kernel_data(*irgen.matmul(m, n, k), "bind")
    rng = np.random.default_rng(11)
    a1, a2 = ((rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32) for _ in range(2))
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    p1, p2 = PreparedKernel(spec), PreparedKernel(spec)
    try:
        p1.upload({"x0": a1, "x1": b})
        p2.upload({"x0": a2, "x1": b})
        own = p2.bind("x0", p1.bufs["x0"])
        p2.launch()
        p2.check_errors()
        ok, rel = _bound_ok(p2.download()["matmul"], a1, b)
        assert ok, rel
        p2.bind("x0", own)
        p2.launch()
        p2.check_errors()
        ok, rel = _bound_ok(p2.download()["matmul"], a2, b)
        assert ok, rel
    finally:
        p2.close()
        p1.close()
