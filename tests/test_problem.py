"""Problem directories with several kernels (``submit.py:80-159``): the
generated two-kernel ``center`` problem loads, both kernels compile to PTX
ptxas accepts, the runner's seeded inputs are the oracle's, and the oracle
run chained kernel by kernel matches f64."""

import json
import shutil
import subprocess
import sys

import numpy as np
import pytest

from oracle.interp import interpret, make_inputs
from ptxgen import irgen
from ptxgen.emit import compile_kernel
from ptxgen.problem import load_problem, seeded_inputs


def _oracle_chain(specs):
    produced = {}
    for s in specs:
        produced.update(interpret(s, make_inputs(s, produced)))
    return produced


def write_center(pdir, n):
    """The center problem plus its expected.npz from the chained oracle."""
    graphs, meta = irgen.center(n)
    irgen.write_problem(pdir, graphs, meta)
    _, specs = load_problem(pdir)
    produced = _oracle_chain(specs)
    np.savez(pdir / "expected.npz", y=produced["y"])
    return specs, produced


def test_center_problem_loads_and_chains(tmp_path):
    specs, produced = write_center(tmp_path, 4096)
    assert [s.entry for s in specs] == ["k_mean_ffcca3", "k_sub_pointwise"]
    assert specs[1].args["mean"].intermediate and specs[0].args["mean"].output
    meta = json.loads((tmp_path / "meta.json").read_text())
    assert [k["final"] for k in meta["kernels"]] == [False, True]
    x = np.random.default_rng(0).standard_normal(4096)
    np.testing.assert_allclose(produced["y"], x - x.mean(), rtol=0, atol=1e-6)


def test_center_kernels_compile(tmp_path):
    specs, _ = write_center(tmp_path, 4096)
    if shutil.which("ptxas") is None:
        pytest.skip("ptxas not on PATH")
    for s in specs:
        ptx = tmp_path / f"{s.entry}.ptx"
        ptx.write_text(compile_kernel(s))
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(ptx)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr


def test_seeded_inputs_match_the_runner_semantics(tmp_path):
    specs, _ = write_center(tmp_path, 1000)
    for s in specs:
        ours = seeded_inputs(s)
        ref = make_inputs(s, {"mean": np.zeros(1, np.float32)})
        assert set(ours) == {n for n in s.arg_order
                             if s.args[n].seed is not None and not s.args[n].intermediate
                             and not s.args[n].output}
        for n, arr in ours.items():
            np.testing.assert_array_equal(arr, ref[n])


def test_missing_producer_is_one_line_error(tmp_path):
    graphs, meta = irgen.center(1024)
    meta["kernels"] = meta["kernels"][1:]          # the consumer alone
    irgen.write_problem(tmp_path, {k: g for k, g in graphs.items() if k == "k_sub_pointwise"},
                        meta)
    r = subprocess.run([sys.executable, "-m", "ptxgen.problem", str(tmp_path)],
                       capture_output=True, text=True,
                       env={**__import__("os").environ,
                            "PYTHONPATH": str(__import__("pathlib").Path(__file__).resolve()
                                              .parent.parent / "emmy-ptx_b200")})
    assert r.returncode == 1 and r.stdout == ""
    assert len(r.stderr.strip().splitlines()) == 1


def write_zero_chain(pdir, n=5000, m=37):
    """The zero-chain problem plus its expected.npz from the chained oracle."""
    graphs, meta = irgen.zero_chain(n, m)
    irgen.write_problem(pdir, graphs, meta)
    _, specs = load_problem(pdir)
    produced = _oracle_chain(specs)
    np.savez(pdir / "expected.npz", acc=produced["acc"])
    return specs, produced


def test_zero_chain_loads_and_chains(tmp_path):
    """ZeroPrologue in the first kernel, zero_delegated and atomic writes in
    the second, y and acc chained as intermediates."""
    specs, produced = write_zero_chain(tmp_path)
    assert [s.entry for s in specs] == ["k_scale_zero", "k_accum_into"]
    assert type(specs[0].op.body[0]).__name__ == "ZeroPrologue"
    assert tuple(specs[1].op.zero_delegated) == ("acc",) and not specs[1].zero_outputs
    assert specs[1].args["acc"].intermediate and specs[1].args["acc"].output
    x = np.random.default_rng(0).standard_normal(5000).astype(np.float32)
    want = np.zeros(37)
    np.add.at(want, np.arange(5000) % 37, (x * np.float32(0.75)).astype(np.float64))
    np.testing.assert_allclose(produced["acc"], want, rtol=1e-5, atol=1e-5)
    if shutil.which("ptxas") is None:
        return
    for s in specs:
        ptx = tmp_path / f"{s.entry}.ptx"
        ptx.write_text(compile_kernel(s))
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(ptx)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
