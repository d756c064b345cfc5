"""Whole problems on the B200 through the local runner (``run_problem``):
every shipped problem passes its own ``expected.npz`` check under both the
plan and the meta geometry, the CLI prints PASS lines, and the two-kernel
``center`` problem chains its intermediate on the device."""

import os
import subprocess
import sys
from pathlib import Path

import numpy as np
import pytest

from ptxgen.problem import check, run_problem
from tests.test_problem import write_center, write_zero_chain

pytestmark = pytest.mark.gpu

ROOT = Path(__file__).resolve().parent.parent
GOLDEN = ROOT / "tests" / "golden" / "problems"
PROBS = sorted(p.name for p in GOLDEN.iterdir() if (p / "meta.json").exists())


@pytest.mark.parametrize("geometry", ["plan", "meta"])
@pytest.mark.parametrize("prob", PROBS)
def test_shipped_problem_passes(prob, geometry):
    outs = run_problem(GOLDEN / prob, geometry=geometry, return_all=True)
    res = check(outs, GOLDEN / prob)
    assert res and all(ok for _, ok, _ in res), res


def test_cli_prints_pass():
    r = subprocess.run([sys.executable, "-m", "ptxgen.problem", str(GOLDEN / "r03_mean")],
                       capture_output=True, text=True,
                       env={**os.environ, "PYTHONPATH": str(ROOT / "emmy-ptx_b200")})
    assert r.returncode == 0, r.stderr
    assert r.stdout.startswith("PASS")


@pytest.mark.parametrize("n", [4096, 1 << 24])
def test_center_chains_on_device(n, tmp_path):
    if n <= 4096:
        write_center(tmp_path, n)
        outs = run_problem(tmp_path)
        res = check(outs, tmp_path)
        assert res and all(ok for _, ok, _ in res), res
    else:
        from ptxgen import irgen
        graphs, meta = irgen.center(n, threads=1024)
        irgen.write_problem(tmp_path, graphs, meta)
        outs = run_problem(tmp_path, return_all=True)
        x = np.random.default_rng(0).standard_normal(n).astype(np.float32)
        m = x.astype(np.float64).mean()
        assert abs(float(outs["mean"][0]) - m) <= 1e-5 * np.abs(x).mean()
        np.testing.assert_allclose(outs["y"], x - np.float32(outs["mean"][0]), rtol=0, atol=0)


def test_zero_chain_runs_on_device(tmp_path):
    """The delegated zero-init: the whole chain against the oracle's, then
    the first kernel alone on an accumulator left dirty, which its
    ZeroPrologue must clear, and three chains in a row on the same buffers
    (no clearing in between), each giving the single-run result."""
    from ptxgen.emit import compile_kernel
    from ptxgen.problem import seeded_inputs
    from ptxgen.runtime import Device, PreparedKernel
    specs, produced = write_zero_chain(tmp_path)
    res = check(run_problem(tmp_path), tmp_path)
    assert res and all(ok for _, ok, _ in res), res
    dev = Device.get(0)
    pk1 = PreparedKernel(specs[0], ptx=compile_kernel(specs[0]), dev=dev)
    pk2 = PreparedKernel(specs[1], ptx=compile_kernel(specs[1]), dev=dev)
    try:
        pk1.upload(seeded_inputs(specs[0]))
        dev.htod(pk1.bufs["acc"], np.full(37, 7.0, np.float32))
        pk1.launch()
        pk1.check_errors()
        first = pk1.download()
        assert np.all(first["acc"] == 0)
        x = np.random.default_rng(0).standard_normal(5000).astype(np.float32)
        assert np.array_equal(first["y"], (x * np.float32(0.75)).astype(np.float32))
        dev.dtod(pk2.bufs["y"], pk1.bufs["y"], 5000 * 4)
        for _ in range(3):
            pk1.launch()
            dev.dtod(pk2.bufs["acc"], pk1.bufs["acc"], 37 * 4)
            pk2.launch()
            pk2.check_errors()
            got = pk2.download()["acc"]
            assert np.allclose(got, produced["acc"], rtol=1e-5, atol=1e-5)
            dev.dtod(pk1.bufs["acc"], pk2.bufs["acc"], 37 * 4)   # leave it dirty again
    finally:
        pk1.close()
        pk2.close()
