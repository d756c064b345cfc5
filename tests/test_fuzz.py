"""The differential fuzzer's cases (``tests/fuzz_ir.py``) are deterministic,
pick the expected template, and compile -- template path and range-checked
generic path -- to PTX that ptxas accepts for sm_100a."""

import re
import shutil
import subprocess

import numpy as np
import pytest

from ptxgen.emit import compile_kernel
from tests import fuzz_ir

EXPECT = {"pointwise": "pointwise", "reduce_full": "reduce_full", "rows": "rows",
          "matmul": "matmul", "splitk": "matmul", "attention": "attention"}


def test_cases_are_deterministic():
    a, b = fuzz_ir.case(7), fuzz_ir.case(7)
    assert a.name == b.name and a.spec.arg_order == b.spec.arg_order
    for k in a.inputs:
        assert np.array_equal(a.inputs[k], b.inputs[k])


@pytest.mark.parametrize("seed", range(24))
def test_case_compiles(seed, tmp_path):
    c = fuzz_ir.case(seed)
    for checked in (False, True):
        ptx = compile_kernel(c.spec, checked=checked)
        tmpl = re.search(r'"template": "(\w+)"', ptx).group(1)
        assert tmpl == ("generic" if checked else EXPECT[c.family]), (c.name, tmpl)
        if shutil.which("ptxas") is None:
            continue
        p = tmp_path / "k.ptx"
        p.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(p)],
                           capture_output=True, text=True)
        assert r.returncode == 0, (c.name, r.stderr)


def test_compare_catches_a_planted_error():
    """A mistake planted in the oracle's answer (on the CPU) is caught."""
    from oracle.interp import interpret
    c = fuzz_ir.case(0)
    want = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})
    bad = {k: v.copy() for k, v in want.items()}
    name = next(iter(bad))
    bad[name].reshape(-1)[0] += 1.0
    with pytest.raises(AssertionError):
        fuzz_ir.compare(c, bad, want)
    fuzz_ir.compare(c, want, want)
