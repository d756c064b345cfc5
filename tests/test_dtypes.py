"""f16 and f64 data paths on the CPU: the generated golden kernels in those
dtypes pick the template of their family (the per-thread-loop column sum has
none and takes the generic lowering), and every path -- template, generic,
range-checked generic -- gives PTX that ptxas accepts for sm_100a.  The
oracle's bit-exact agreement with the reference interpreter on the same
cases is ``tests/test_oracle.py``'s."""

import json
import re
import shutil
import subprocess
from pathlib import Path

import pytest

from ptxgen.emit import compile_kernel
from ptxgen.loader import load_kernel_data

GOLDEN = Path(__file__).parent / "golden"
CASES = [c for c in json.loads((GOLDEN / "cases.json").read_text())
         if "meta" in c and re.search(r"_f(16|64)_", c["case"])]
EXPECT = {"gen_add": "pointwise", "gen_relu_mul": "pointwise", "gen_sum_f16acc": "generic",
          "gen_sum": "reduce_full",
          "gen_mean": "reduce_full", "gen_rowsum": "rows", "gen_colsum": "generic"}


def spec_of(case):
    return load_kernel_data(json.loads((GOLDEN / case["ir"]).read_text()),
                            json.loads((GOLDEN / case["meta"]).read_text()), case["case"])


def test_both_dtypes_are_covered():
    names = " ".join(c["case"] for c in CASES)
    assert "_f16_" in names and "_f64_" in names and len(CASES) >= 9


@pytest.mark.parametrize("case", CASES, ids=[c["case"] for c in CASES])
def test_dtype_case_compiles(case, tmp_path):
    spec = spec_of(case)
    family = next(v for k, v in EXPECT.items() if case["case"].startswith(k + "_"))
    for kw, want in (({}, family), ({"generic": True}, "generic"),
                     ({"generic": True, "checked": True}, "generic")):
        ptx = compile_kernel(spec, **kw)
        tmpl = re.search(r'"template": "(\w+)"', ptx).group(1)
        assert tmpl == want, (case["case"], kw, tmpl)
        if shutil.which("ptxas") is None:
            continue
        p = tmp_path / "k.ptx"
        p.write_text(ptx)
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(p)],
                           capture_output=True, text=True)
        assert r.returncode == 0, (case["case"], kw, r.stderr)
