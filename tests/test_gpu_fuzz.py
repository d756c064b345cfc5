"""Differential fuzzing on the B200: every case of ``tests/fuzz_ir.py`` runs
through its template (the plan's launch) and through the range-checked
generic lowering (meta.json's launch), and both must match the oracle within
the family's bound; a checked run that touched memory outside a buffer fails
with the buffer and index."""

import pytest

from oracle.interp import interpret
from ptxgen.emit import compile_kernel
from ptxgen.runtime import run_kernel
from tests import fuzz_ir

pytestmark = pytest.mark.gpu
N_CASES = 192


@pytest.mark.parametrize("seed", range(N_CASES))
def test_fuzz_case(seed):
    c = fuzz_ir.case(seed)
    want = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})
    for checked, geometry in ((False, "plan"), (True, "meta")):
        got = run_kernel(c.spec, {k: v.copy() for k, v in c.inputs.items()},
                         geometry=geometry, ptx=compile_kernel(c.spec, checked=checked))
        fuzz_ir.compare(c, got, want)
