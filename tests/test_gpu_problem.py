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
from tests.test_problem import write_center

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
