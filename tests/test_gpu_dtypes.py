"""GPU parity of the f16 and f64 data paths against the reference
interpreter's own recorded outputs (``tests/golden/ref_interp``).

Each generated f16/f64 golden kernel runs through its template and through
the generic lowering.  The reference's semantics being checked
(``ptxgen/interp.py:105-141``, ``:238-250``, ``:706-721``): f64 binary
arithmetic stays f64, unary ops evaluate in f32, an ``Assign``/``Accum``
rounds its result to its dtype, f16 values compute in f32 and round once to
f16 on every coercion.  Pointwise kernels and the sequential column sums
must match bit for bit; the cross-thread sums differ from the reference only
in the order of their f32 additions, so they are held to that order's bound
(1e-5 of the sum of magnitudes) plus one ulp of the stored f16 result."""

from pathlib import Path

import numpy as np
import pytest

from ptxgen.emit import compile_kernel
from tests.golden.make_golden import rebuild_inputs
from tests.test_dtypes import CASES, spec_of

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
# the f16-accumulated sum keeps the IR's thread mapping and combine tree
# (templates decline it), so it too must match bit for bit
EXACT = ("gen_add", "gen_relu_mul", "gen_colsum", "gen_sum_f16acc")


def _bound(case, spec, inputs, ref):
    x = np.abs(inputs["x"].astype(np.float64))
    total = x.sum() if ref.size == 1 else x.sum(axis=-1).reshape(ref.shape)
    if case["case"].startswith("gen_mean"):
        total = total / x.size
    ulp = np.spacing(np.abs(ref).astype(ref.dtype)).astype(np.float64)
    return 1e-5 * total + ulp


@pytest.mark.parametrize("generic", [False, True], ids=["template", "generic"])
@pytest.mark.parametrize("case", CASES, ids=[c["case"] for c in CASES])
def test_dtype_case_matches_reference(case, generic):
    from ptxgen.runtime import run_kernel
    spec = spec_of(case)
    inputs = rebuild_inputs(spec, case["seed_offset"], case["dist"])
    got = run_kernel(spec, {k: v.copy() for k, v in inputs.items()},
                     ptx=compile_kernel(spec, generic=generic))
    ref = np.load(GOLDEN / "ref_interp" / f"{case['case']}.npz")
    for name in ref.files:
        r, g = ref[name], np.asarray(got[name])
        assert g.dtype == r.dtype and g.shape == r.shape, (name, g.dtype, r.dtype)
        if case["case"].startswith(EXACT):
            assert np.array_equal(g, r, equal_nan=True), (
                name, int(np.sum(g != r)), float(np.abs(g.astype(np.float64) - r).max()))
        else:
            err = np.abs(g.astype(np.float64) - r.astype(np.float64))
            assert np.all(err <= _bound(case, spec, inputs, r)), (name, float(err.max()))
