"""The CPU oracle against the reference's golden vectors.

* every shipped problem: oracle output vs ``expected.npz`` within the
  problem's own ``rtol``/``atol`` (``scripts/verify_semantics.py:65-97``);
* every recorded case: oracle output vs the reference interpreter's output on
  the same inputs, bit for bit;
* every non-bf16 case of the family fuzzer and every statement mix of the
  soup fuzzer: the oracle's outputs against SHA-256 digests of the reference
  interpreter's (``fuzz_digests.json``, ``soup_digests.json``);
* every recorded IR with special values (NaN, infinities, signed zeros,
  subnormals, near-overflow) in its inputs, against digests of the
  reference interpreter's outputs (``special_digests.json``), and again
  with a sparser mix without near-overflow values
  (``special_nonfinite_digests.json``).
"""

import json
from pathlib import Path

import numpy as np
import pytest

from oracle.interp import interpret, make_inputs
from ptxgen.loader import load_kernel, load_kernel_data

GOLDEN = Path(__file__).parent / "golden"
PROBLEMS = sorted(p for p in (GOLDEN / "problems").iterdir() if (p / "meta.json").exists())


@pytest.mark.parametrize("pdir", PROBLEMS, ids=[p.name for p in PROBLEMS])
def test_oracle_matches_expected(pdir):
    meta = json.loads((pdir / "meta.json").read_text())
    expected = dict(np.load(pdir / "expected.npz"))
    produced = {}
    for k in meta["kernels"]:
        spec = load_kernel(pdir / f"{k['entry']}.ir.json")
        outs = interpret(spec, make_inputs(spec, produced))
        produced.update(outs)
    for name, ref in expected.items():
        got = np.asarray(produced[name], dtype=np.float32).reshape(ref.shape)
        assert np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"], equal_nan=True), name


def _rebuild(spec, off, dist):
    from tests.golden.make_golden import rebuild_inputs  # same recipe as recorded
    return rebuild_inputs(spec, off, dist)


CASES = json.loads((GOLDEN / "cases.json").read_text())


@pytest.mark.parametrize("case", CASES, ids=[c["case"] for c in CASES])
def test_oracle_bit_exact_vs_reference_interpreter(case):
    if "meta" in case:
        spec = load_kernel_data(json.loads((GOLDEN / case["ir"]).read_text()),
                                json.loads((GOLDEN / case["meta"]).read_text()), case["case"])
    else:
        spec = load_kernel(GOLDEN / case["ir"])
    outs = interpret(spec, _rebuild(spec, case["seed_offset"], case["dist"]))
    ref = np.load(GOLDEN / "ref_interp" / f"{case['case']}.npz")
    for name in ref.files:
        assert np.array_equal(np.asarray(outs[name]), ref[name], equal_nan=True), name


def _digests(fname, module):
    return [dict(d, module=module) for d in json.loads((GOLDEN / fname).read_text())
            if "outputs" in d]


FUZZ = _digests("fuzz_digests.json", "fuzz_ir") + _digests("soup_digests.json", "fuzz_soup")


def test_fuzz_digests_cover_the_fuzzers():
    from tests.golden.make_golden import FUZZ_CASES, SOUP_FUZZ_CASES
    from tests.test_gpu_fuzz import N_CASES
    from tests.test_gpu_fuzz_soup import N_CASES as N_SOUP
    assert FUZZ_CASES == N_CASES and SOUP_FUZZ_CASES == N_SOUP
    assert sum(d["module"] == "fuzz_ir" for d in FUZZ) >= 170
    assert sum(d["module"] == "fuzz_soup" for d in FUZZ) == N_SOUP


@pytest.mark.parametrize("rec", FUZZ, ids=[f"{d['module']}{d['seed']}_{d['family']}" for d in FUZZ])
def test_oracle_bit_exact_on_fuzz_cases(rec):
    """Every case of the family fuzzer but the bf16 ones, and every
    statement mix (the GPU fuzz tests' checker): the oracle's outputs hash
    to the reference interpreter's."""
    import importlib
    from tests.golden.make_golden import output_digest
    c = importlib.import_module(f"tests.{rec['module']}").case(rec["seed"])
    outs = interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})
    assert sorted(outs) == sorted(rec["outputs"])
    for name, want in rec["outputs"].items():
        assert output_digest(outs[name]) == want, name


SPECIAL = [dict(d, variant=v) for v, f in (("all", "special_digests.json"),
                                             ("nonfinite", "special_nonfinite_digests.json"))
           for d in json.loads((GOLDEN / f).read_text())]


def test_special_digests_cover_every_recorded_ir():
    for v in ("all", "nonfinite"):
        assert len([d for d in SPECIAL if d["variant"] == v]) == len({c["ir"] for c in CASES})


@pytest.mark.parametrize("rec", SPECIAL, ids=[f"{d['variant']}-{d['case']}" for d in SPECIAL])
def test_oracle_bit_exact_on_special_values(rec):
    """NaN, infinities, signed zeros, subnormals and (variant ``all``)
    near-overflow values in the inputs of every recorded IR: the oracle's
    outputs, NaN payloads included, hash to the reference interpreter's."""
    from tests.golden.make_golden import _case_spec, output_digest, special_inputs
    spec = _case_spec(rec)
    with np.errstate(all="ignore"):
        outs = interpret(spec, special_inputs(spec, rec["variant"]))
    assert sorted(outs) == sorted(rec["outputs"])
    for name, want in rec["outputs"].items():
        assert output_digest(outs[name]) == want, name
