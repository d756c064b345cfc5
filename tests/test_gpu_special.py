"""Special-value parity on B200: every recorded IR (shipped problems,
generated kernels, statement mixes -- the 63 of ``special_digests.json``)
run through its template with NaN, +-inf, -0.0, f32 subnormals, +-3e38, 0
and 1 mixed into its inputs (``make_golden.special_inputs``), and again
with a sparser mix without +-3e38 (variant ``nonfinite``), compared with
the oracle, whose outputs on exactly these inputs are pinned to the
reference interpreter's by digest (``tests/test_oracle.py``).

The reference's f32 semantics (``ptxgen/interp.py:196-217``): ``+ - * /``
rounded once in IEEE f32, ``maximum``/``minimum`` dropping a NaN operand.

* Kernels whose arithmetic is exactly rounded, or whose order of
  operations equals the IR's, must match bit for bit (NaN = NaN).
* Kernels that sum in another order (full and row reductions, the fused
  rows, the 3xTF32 contraction, split-K, attention) or approximate ``exp``
  must give the same NaN and +-inf positions (and signs), and finite
  values within the family's bound -- the bound the family's other GPU
  tests use.  The one exception is a sum whose order decides overflow:
  where the terms' absolute values add up past the f32 range (the same IR
  run on ``|inputs|`` overflows), IEEE f32 gives +inf, -inf, NaN or a
  finite value depending on the order, and the reference's order is an
  artifact of its interpreter.  Such outputs are not compared; the
  ``nonfinite`` variant has none, so there every output is checked.
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.interp import interpret
from tests.golden.make_golden import _case_spec, special_inputs

pytestmark = pytest.mark.gpu
GOLDEN = Path(__file__).parent / "golden"
RECORDS = [dict(d, variant=v) for v, f in (("all", "special_digests.json"),
                                           ("nonfinite", "special_nonfinite_digests.json"))
           for d in json.loads((GOLDEN / f).read_text())]

# case-name prefix -> (bound kind, relative bound on finite values):
#   "mag": rtol x (the IR on |inputs|), i.e. x sum of |terms|;
#   "ref": rtol x |reference value| + 1e-7;
#   "refmax": rtol x max |finite reference value| of the output.
FAMILIES = [
    (("m01_", "m02_", "gen_matmul_", "gen_splitk_"), "mag", 2.0 ** -15),
    (("r01_", "r02_", "r03_", "r04_", "gen_sum_5000", "gen_sum_f16_", "gen_mean_",
      "gen_rowsum_"), "mag", 1e-5),
    (("f01_", "f02_", "f03_", "gen_rmsnorm_", "gen_softmax_", "gen_l2norm_"), "ref", 1e-5),
    (("a01_", "a02_", "gen_attn_"), "refmax", 1e-4),
]


def _family(case: str):
    for prefixes, kind, rtol in FAMILIES:
        if case.startswith(prefixes):
            return kind, rtol
    return None


def _magnitude(spec, ins):
    """The IR evaluated on the absolute values of its inputs, with every
    non-finite input set to 0: for sums and contractions, the sum of the
    absolute values of the finite terms (inf where that overflows f32)."""
    absins = {}
    for name, a in ins.items():
        a = np.array(a, copy=True)
        if a.dtype.kind == "f" and not spec.args[name].output:
            with np.errstate(invalid="ignore"):
                a = np.where(np.isfinite(a), np.abs(a), 0).astype(a.dtype)
        absins[name] = a
    with np.errstate(all="ignore"):
        return interpret(spec, absins)


def _ulp16(w):
    """One f16 ulp at |w| (a sum rounded to an f16 output may land on
    either neighbour)."""
    a = np.abs(w).astype(np.float16)
    return (np.nextafter(a, np.float16(np.inf)) - a).astype(np.float64)


@pytest.mark.parametrize("rec", RECORDS, ids=[f"{r['variant']}-{r['case']}" for r in RECORDS])
def test_special_values(rec):
    from ptxgen.runtime import run_kernel
    spec = _case_spec(rec)
    ins = special_inputs(spec, rec["variant"])
    with np.errstate(all="ignore"):
        want = interpret(spec, {k: v.copy() for k, v in ins.items()})
    got = run_kernel(spec, {k: v.copy() for k, v in ins.items()})
    fam = _family(rec["case"])
    mag = _magnitude(spec, ins) if fam is not None and fam[0] == "mag" else None
    for name, w in want.items():
        g = np.asarray(got[name])
        w = np.asarray(w)
        assert g.shape == w.shape and g.dtype == w.dtype, name
        if fam is None:
            assert np.array_equal(g, w, equal_nan=True), (
                f"{name}: {int((~((g == w) | (np.isnan(g) & np.isnan(w)))).sum())} "
                f"of {w.size} outputs differ")
            continue
        kind, rtol = fam
        g64, w64 = g.astype(np.float64).reshape(-1), w.astype(np.float64).reshape(-1)
        free = np.zeros(w64.shape, bool)
        if kind == "mag":
            m = np.asarray(mag[name], np.float64).reshape(-1)
            free = ~np.isfinite(m)          # order-dependent overflow
            if rec["variant"] == "nonfinite":
                # no near-overflow inputs: every output is determinate
                assert not free.any(), f"{name}: {int(free.sum())} sums overflow"
            bound = rtol * np.where(free, 0.0, m)
        elif kind == "ref":
            bound = rtol * np.abs(np.nan_to_num(w64, posinf=0, neginf=0)) + 1e-7
        else:
            fin_w = w64[np.isfinite(w64)]
            bound = np.full(w64.shape, rtol * (np.abs(fin_w).max() if fin_w.size else 0.0))
        if w.dtype == np.float16:
            bound = bound + _ulp16(np.nan_to_num(w, posinf=0, neginf=0)).reshape(-1)
        chk = ~free
        assert np.array_equal(np.isnan(w64)[chk], np.isnan(g64)[chk]), \
            f"{name}: NaN positions differ"
        inf_w = np.isinf(w64)
        assert np.array_equal(inf_w[chk], np.isinf(g64)[chk]), f"{name}: inf positions differ"
        sel = chk & inf_w
        assert np.array_equal(w64[sel], g64[sel]), f"{name}: inf signs differ"
        fin = chk & np.isfinite(w64)
        err = np.abs(g64[fin] - w64[fin])
        assert np.all(err <= bound[fin] + 1e-37), (
            f"{name}: finite values outside {rtol:g} x {kind}: "
            f"max excess {float(np.max(err - bound[fin])):.3g}")
