"""GPU parity of the generic statement-by-statement lowering, plain and
range-checked.

Every shipped problem and every generated golden kernel is compiled with the
templates switched off and run under meta.json's own launch, then compared
with the CPU oracle: bit for bit for pointwise kernels, to 1e-5 for the rest
(exp-based ops, and the order of split-K atomic adds, differ from the
reference; f16 results may also move by one ulp).  The checked variant must give the same results and report no
violation on these in-bounds kernels."""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.interp import interpret, make_inputs
from ptxgen.emit import compile_kernel
from ptxgen.loader import load_kernel, load_kernel_data

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
PROBS = sorted(p.name for p in (GOLDEN / "problems").iterdir() if (p / "meta.json").exists())
GEN = [c for c in json.loads((GOLDEN / "cases.json").read_text()) if "meta" in c]
EXACT = ("p0", "gen_add", "gen_relu", "gen_colsum", "gen_sum_f16acc", "soup_", "gen_scalar")


def _check(spec, inputs, exact, checked=False):
    from ptxgen.runtime import run_kernel
    want = interpret(spec, {k: v.copy() for k, v in inputs.items()})
    got = run_kernel(spec, {k: v.copy() for k, v in inputs.items()},
                     ptx=compile_kernel(spec, generic=True, checked=checked))
    for name, ref in want.items():
        if exact:
            assert np.array_equal(got[name], ref), name
        else:
            # f16 results: the f32 sum order may move the rounding by one ulp
            r = np.asarray(ref)
            tol = 1e-5 * (1.0 + np.abs(r.astype(np.float64)))
            if r.dtype == np.float16:
                tol = tol + np.spacing(np.abs(r)).astype(np.float64)
            err = np.abs(np.asarray(got[name]).astype(np.float64) - r.astype(np.float64))
            assert np.all(err <= tol), (name, float(err.max()))


@pytest.mark.parametrize("checked", [False, True], ids=["plain", "checked"])
@pytest.mark.parametrize("prob", PROBS)
def test_problem_generic(prob, checked):
    spec = load_kernel(next((GOLDEN / "problems" / prob).glob("*.ir.json")))
    _check(spec, make_inputs(spec), prob.startswith("p0"), checked)


@pytest.mark.parametrize("checked", [False, True], ids=["plain", "checked"])
@pytest.mark.parametrize("case", GEN, ids=[c["case"] for c in GEN])
def test_generated_generic(case, checked):
    spec = load_kernel_data(json.loads((GOLDEN / case["ir"]).read_text()),
                            json.loads((GOLDEN / case["meta"]).read_text()), case["case"])
    from tests.golden.make_golden import rebuild_inputs
    _check(spec, rebuild_inputs(spec, case["seed_offset"], case["dist"]),
           case["case"].startswith(EXACT), checked)
