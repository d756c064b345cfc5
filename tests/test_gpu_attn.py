"""GPU parity for the fused attention template (a01/a02 family, [B,H,S,D]).

* shipped problems against the oracle and ``expected.npz`` under the plan
  launch (tensor cores where the shape tiles, a02) and meta.json's launch
  (the SIMT path that follows the IR per key);
* generated [B, H, S, D] shapes, f32 (3xTF32: per query row max|err| <=
  1e-4 of the row's max|ref|, ``tests/contraction.py``, which a one-pass
  TF32 kernel fails) and bf16 (bf16 output, |err| <= 2e-2 of the scale),
  against float64 numpy;
* the BASELINE shape [16, 32, 4096, 128] on sampled (batch, head) pairs.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.interp import interpret, make_inputs
from ptxgen import irgen
from ptxgen.loader import load_kernel, load_kernel_data

from tests.contraction import attention_check

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden" / "problems"


def _close(out, ref, dtype):
    """f32: the per-row 3xTF32 bound; bf16: 2e-2 of the output scale."""
    if dtype == "f32":
        return attention_check(out, ref)
    worst = float(np.abs(out - ref).max() / np.abs(ref).max())
    return worst <= 2e-2, worst


def _run(spec, inputs, geometry="plan"):
    from ptxgen.runtime import run_kernel
    return run_kernel(spec, {k: v.copy() for k, v in inputs.items()}, geometry=geometry)


def _ref(q, k, v):
    q, k, v = (x.astype(np.float64) for x in (q, k, v))
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return p @ v


@pytest.mark.parametrize("geometry", ["plan", "meta"])
@pytest.mark.parametrize("prob", ["a01_attention", "a02_attention_128"])
def test_problem(prob, geometry):
    pdir = GOLDEN / prob
    meta = json.loads((pdir / "meta.json").read_text())
    spec = load_kernel(next(pdir.glob("*.ir.json")))
    inputs = make_inputs(spec)
    want = interpret(spec, {k: v.copy() for k, v in inputs.items()})["matmul_1"]
    got = _run(spec, inputs, geometry)["matmul_1"]
    assert np.allclose(got, want, rtol=1e-4, atol=1e-5), float(np.abs(got - want).max())
    exp = np.load(pdir / "expected.npz")["matmul_1"]
    assert np.allclose(got, exp, rtol=meta["rtol"], atol=meta["atol"])


def _bhsd(b, h, s, d, dtype, seed=0):
    rng = np.random.default_rng(seed)
    if dtype == "bf16":
        from ml_dtypes import bfloat16
        mk = lambda: rng.standard_normal((b, h, s, d)).astype(bfloat16)  # noqa: E731
    else:
        mk = lambda: rng.standard_normal((b, h, s, d)).astype(np.float32)  # noqa: E731
    return mk(), mk(), mk()


@pytest.mark.parametrize("dtype,shape", [("f32", (2, 2, 256, 64)), ("f32", (1, 3, 384, 128)),
                                         ("f32", (1, 2, 256, 32)),
                                         ("bf16", (2, 2, 256, 128)), ("bf16", (1, 2, 512, 64)),
                                         ("bf16", (1, 2, 256, 256)), ("bf16", (1, 2, 384, 128)),
                                         ("bf16", (2, 1, 256, 32)), ("bf16", (1, 3, 128, 128))])
def test_generated(dtype, shape):
    b, h, s, d = shape
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, dtype), "att")
    q, k, v = _bhsd(b, h, s, d, dtype)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"].astype(np.float64)
    ok, worst = _close(out, _ref(q, k, v), dtype)
    assert ok, worst


SCHEDULES = {"half": ({}, "two query tiles, 64-key blocks, two S buffers per tile"),
             "two_q": ({"EMMY_ATTN_HALF": "0"}, "two query tiles"),
             "one_q": ({"EMMY_ATTN_HALF": "0", "EMMY_ATTN_2Q": "0"}, "one query tile")}


@pytest.mark.parametrize("sched", list(SCHEDULES))
@pytest.mark.parametrize("shape", [(1, 2, 256, 128), (2, 3, 512, 128), (1, 1, 1024, 128),
                                   (8, 16, 512, 128)])
def test_bf16_d128_schedules(shape, sched, monkeypatch):
    """bf16 with D = 128 and S a multiple of 256 runs the two-tile kernel on
    64-key blocks (``tmpl_attn2h``); ``EMMY_ATTN_HALF=0`` selects the
    two-tile kernel on 128-key blocks (``tmpl_attn2q``), and with
    ``EMMY_ATTN_2Q=0`` too the one-tile kernel.  All three at the same
    shapes, two launches each; the last shape has 256 units, so most CTAs
    run two (the hand-over of Q and O between a CTA's units)."""
    env, want = SCHEDULES[sched]
    for key, val in env.items():
        monkeypatch.setenv(key, val)
    b, h, s, d = shape
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, "bf16"), f"att{sched}")
    q, k, v = _bhsd(b, h, s, d, "bf16", seed=21)
    from ptxgen.runtime import PreparedKernel
    pk = PreparedKernel(spec)
    try:
        assert pk.plan["schedule"] == want
        pk.upload({"q": q, "k": k, "v": v})
        for _ in range(2):
            pk.launch()
        pk.check_errors()
        out = pk.download()["out"].astype(np.float64)
    finally:
        pk.close()
    ok, worst = _close(out, _ref(q, k, v), "bf16")
    assert ok, worst


@pytest.mark.parametrize("sched", ["half", "two_q"])
def test_bf16_two_tile_rescale_path(sched, monkeypatch):
    """Keys scaled up along the sequence: every row's max keeps growing, so
    the two-tile kernels rescale O in TMEM block after block."""
    for key, val in SCHEDULES[sched][0].items():
        monkeypatch.setenv(key, val)
    b, h, s, d = 1, 2, 2048, 128
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, "bf16"), f"att2r{sched}")
    q, k, v = _bhsd(b, h, s, d, "bf16", seed=23)
    grow = (1.0 + 8.0 * np.arange(s) / s)[None, None, :, None]
    k = (k.astype(np.float64) * grow).astype(k.dtype)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"].astype(np.float64)
    ok, worst = _close(out, _ref(q, k, v), "bf16")
    assert ok, worst


@pytest.mark.parametrize("geometry", ["plan", "meta"])
@pytest.mark.parametrize("shape", [(96, 64), (128, 32), (256, 128), (512, 64)])
def test_tiled_generated(shape, geometry):
    """a01's schedule (4 x 2 outputs per thread) at other shapes: against the
    oracle where it is quick, and against float64 numpy everywhere."""
    s, d = shape
    spec = load_kernel_data(*irgen.attention_tiled(s, d), "attt")
    inputs = make_inputs(spec)
    got = _run(spec, inputs, geometry)["matmul_1"]
    if s * d <= 128 * 64:
        want = interpret(spec, {k: v.copy() for k, v in inputs.items()})["matmul_1"]
        assert np.allclose(got, want, rtol=1e-4, atol=1e-5), float(np.abs(got - want).max())
    ref = _ref(inputs["q"], np.swapaxes(inputs["kt"], 0, 1), inputs["v"])
    ok, worst = attention_check(got, ref)
    assert ok, worst


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_rescale_path(dtype):
    """Keys scaled by 1 + 6 j / S: each row's max keeps growing over the key
    blocks, so O in TMEM is rescaled (max grown by more than 8 in log2
    units) several times per row."""
    b, h, s, d = 1, 2, 1024, 128
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, dtype), "attr")
    q, k, v = _bhsd(b, h, s, d, dtype, seed=5)
    grow = (1.0 + 6.0 * np.arange(s) / s)[None, None, :, None]
    k = (k.astype(np.float64) * grow).astype(k.dtype)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"].astype(np.float64)
    ok, worst = _close(out, _ref(q, k, v), dtype)
    assert ok, worst


def test_bf16_shared_o(monkeypatch):
    """The bf16 form with one shared O and a per-block max exchange between
    a row's two threads (split O off) stays correct."""
    monkeypatch.setenv("EMMY_ATTN_SPLIT_O", "0")
    b, h, s, d = 2, 2, 512, 128
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, "bf16"), "atto")
    q, k, v = _bhsd(b, h, s, d, "bf16", seed=9)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"].astype(np.float64)
    ref = _ref(q, k, v)
    assert np.abs(out - ref).max() <= 2e-2 * np.abs(ref).max()


@pytest.mark.parametrize("share", [0, 1, 4])
def test_bf16_polynomial_exp2(share, monkeypatch):
    """bf16 P with none, one pair in four, or all of exp2 on the FMA-pipe
    polynomial (the kernels' defaults differ: the one-tile and 128-key
    two-tile kernels use one pair in four, the 64-key kernel none)."""
    monkeypatch.setenv("EMMY_ATTN_EXP_POLY", str(share))
    b, h, s, d = 2, 2, 512, 128
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, "bf16"), "attp")
    q, k, v = _bhsd(b, h, s, d, "bf16", seed=11)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"].astype(np.float64)
    ref = _ref(q, k, v)
    assert np.abs(out - ref).max() <= 2e-2 * np.abs(ref).max()


@pytest.mark.parametrize("dtype", ["f32", "bf16"])
def test_baseline_shape_sampled(dtype):
    b, h, s, d = 16, 32, 4096, 128
    spec = load_kernel_data(*irgen.attention_bhsd(b, h, s, d, dtype), "attbig")
    q, k, v = _bhsd(b, h, s, d, dtype, seed=3)
    out = _run(spec, {"q": q, "k": k, "v": v})["out"]
    for (bi, hi) in ((0, 0), (7, 19), (15, 31)):
        rows = np.arange(0, s, 97)
        qq = q[bi, hi, rows]
        ref = _ref(qq, k[bi, hi], v[bi, hi])
        got = out[bi, hi, rows].astype(np.float64)
        ok, worst = _close(got, ref, dtype)
        assert ok, (bi, hi, worst)
