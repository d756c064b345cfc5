"""Checked mode on the B200: an IR whose tile reaches past its input is
reported (buffer and first index) instead of reading outside the buffer, and
the in-range part of the result is still right."""

import numpy as np
import pytest

from ptxgen.emit import compile_kernel
from ptxgen.runtime import EmmyError, run_kernel
from tests.test_checked import N_IN, N_TILE, oob_spec

pytestmark = pytest.mark.gpu


def test_out_of_bounds_is_reported_and_skipped():
    from ptxgen.runtime import Device, PreparedKernel
    spec = oob_spec()
    x = np.random.default_rng(0).standard_normal(N_IN).astype(np.float32)
    pk = PreparedKernel(spec, ptx=compile_kernel(spec, checked=True), dev=Device.get(0),
                        geometry="meta")
    try:
        pk.upload({"x": x})
        pk.launch()
        with pytest.raises(EmmyError, match=r"out-of-bounds access to x\[(\d+)\]") as ei:
            pk.check_errors()
        first = int(str(ei.value).split("x[")[1].split("]")[0])
        assert N_IN <= first < N_TILE
        y = pk.download()["y"]
        assert np.array_equal(y[:N_IN], x * x)
        assert not y[N_IN:].any()
        # the report was cleared: a second in-bounds check passes
        pk.check_errors()
    finally:
        pk.close()


def test_checked_in_bounds_runs_clean():
    from ptxgen import irgen
    from ptxgen.loader import load_kernel_data
    spec = load_kernel_data(*irgen.pointwise(4096, 4), "pw")
    rng = np.random.default_rng(1)
    a, b = (rng.standard_normal(4096).astype(np.float32) for _ in range(2))
    out = run_kernel(spec, {"x0": a, "x1": b}, geometry="meta",
                     ptx=compile_kernel(spec, checked=True))
    assert np.array_equal(out["add"], a + b)
