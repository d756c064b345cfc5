"""Random statement mixes (``tests/fuzz_soup.py``) on the CPU: the cases are
deterministic, exercise Cond/Select/Loop, compile on every path to PTX that
ptxas accepts for sm_100a, and the oracle gives finite results."""

import re
import shutil
import subprocess

import numpy as np
import pytest

from oracle.interp import interpret
from ptxgen import ir
from ptxgen.emit import compile_kernel
from tests import fuzz_soup


def test_cases_are_deterministic():
    a, b = fuzz_soup.case(5), fuzz_soup.case(5)
    assert a.graph == b.graph
    for k in a.inputs:
        assert np.array_equal(a.inputs[k], b.inputs[k])


def test_mixes_cover_the_statement_kinds():
    seen = set()
    for seed in range(32):
        seen |= {type(s).__name__ for s in ir.walk(fuzz_soup.case(seed).spec.op.body)}
    assert {"Cond", "Select", "Loop", "Accum", "Let", "Load", "Assign", "Write"} <= seen


@pytest.mark.parametrize("seed", range(16))
def test_case_compiles_and_oracle_is_finite(seed, tmp_path):
    c = fuzz_soup.case(seed)
    out = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})
    assert np.all(np.isfinite(out["out"]))
    for kw in ({}, {"generic": True, "checked": True}):
        ptx = compile_kernel(c.spec, **kw)
        assert re.search(r'"template": "(\w+)"', ptx).group(1) == "generic"
        if shutil.which("ptxas") is None:
            continue
        p = tmp_path / "k.ptx"
        p.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(p)],
                           capture_output=True, text=True)
        assert r.returncode == 0, (c.name, kw, r.stderr)


def test_bit_exact_comparison_catches_a_planted_error():
    """A one-ulp change planted in the oracle's answer (on the CPU) fails the
    comparison the GPU test applies."""
    c = fuzz_soup.case(3)
    want = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})["out"]
    bad = want.copy()
    bad[0] = np.nextafter(bad[0], np.float32(np.inf))
    assert not np.array_equal(bad, want)
