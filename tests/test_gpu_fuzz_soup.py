"""Random statement mixes through the generic lowering on B200, plain and
range-checked, against the oracle: bit for bit (every op in the mixes is
exactly rounded).  128 seeded cases (``tests/fuzz_soup.py``); a quarter of
them also under meta.json's launch geometry."""

import numpy as np
import pytest

from oracle.interp import interpret
from ptxgen.emit import compile_kernel
from tests import fuzz_soup

pytestmark = pytest.mark.gpu
N_CASES = 128


@pytest.mark.parametrize("seed", range(N_CASES))
def test_soup_case(seed):
    from ptxgen.runtime import run_kernel
    c = fuzz_soup.case(seed)
    want = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})["out"]
    variants = [({}, "plan"), ({"checked": True}, "plan")]
    if seed % 4 == 0:
        variants.append(({}, "meta"))
    for kw, geometry in variants:
        got = run_kernel(c.spec, {k: v.copy() for k, v in c.inputs.items()},
                         ptx=compile_kernel(c.spec, **kw), geometry=geometry)["out"]
        diff = np.flatnonzero(got != want)
        assert diff.size == 0, (c.name, kw, geometry, int(diff.size), int(diff[0]),
                                float(got[diff[0]]), float(want[diff[0]]))
