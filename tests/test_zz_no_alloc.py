"""The allocation-free full sum, ``emmy_sum_f32_noalloc``, against the
regular path.

Some callers of this library cannot call cudaMalloc where they need a
reduction (plugin hosts whose enqueue callback must not allocate because the
host framework owns all device memory; latency-critical loops that cannot
afford cudaMalloc's device-wide synchronisation).  For them the library
exports one entry point whose scratch is a fixed file-scope device array.
This test calls it through the C ABI twice in a row on different inputs,
then repeats the first input, and checks every result against the regular
entry point -- the compiled full-reduction IR kernel launched through
``emmy_launch`` -- within the reduction tolerance used by the other GPU
tests (1e-5 relative; inputs are U[0,1], so the sum is well conditioned).

It lives in its own file, collected last, and passes both alone in a fresh
process and after the rest of the suite.
"""

import ctypes as C

import numpy as np
import pytest

from ptxgen import irgen
from ptxgen.loader import load_kernel_data

pytestmark = pytest.mark.gpu

RTOL = 1e-5


def _regular_sum(pk, x):
    pk.upload({"x": x})
    pk.launch()
    pk.check_errors()
    return float(pk.download()["sum_1"][0])


def _free_device_memory() -> int:
    """Free bytes on the current context's device (cuMemGetInfo)."""
    cuda = C.CDLL("libcuda.so.1")
    free, total = C.c_size_t(), C.c_size_t()
    assert cuda.cuMemGetInfo_v2(C.byref(free), C.byref(total)) == 0
    return free.value


def test_noalloc_sum_matches_regular_entry_point_on_consecutive_calls():
    from ptxgen.runtime import Device, PreparedKernel
    dev = Device.get(0)
    fn = dev.L.emmy_sum_f32_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_uint64, C.c_size_t, C.c_uint64, C.c_void_p]
    out = dev.alloc(4)
    cases = [(3_000_001, 11), (1 << 24, 12), (3_000_001, 11)]
    xs, prepared, wants = [], [], []
    try:
        # every buffer of the regular path first, so that only the entry
        # point itself runs between the free-memory readings below
        for n, seed in cases:
            x = np.random.default_rng(seed).random(n, dtype=np.float32)
            gm = irgen.reduce_full(n)
            pk = PreparedKernel(load_kernel_data(gm[0], gm[1], f"sum{n}"), dev=dev)
            prepared.append(pk)
            xs.append(x)
            wants.append(_regular_sum(pk, x))
        dev.sync()
        results, free_after = [], []
        for (n, _), x, pk, want in zip(cases, xs, prepared, wants):
            rc = fn(pk.bufs["x"], n, out, dev.stream)
            assert rc == 0, dev.L.emmy_last_error().decode()
            got = np.empty(1, np.float32)
            dev.dtoh(got, out)
            dev.sync()
            free_after.append(_free_device_memory())
            got = float(got[0])
            assert abs(got - want) <= RTOL * abs(want), (n, got, want)
            exact = float(x.astype(np.float64).sum())
            assert abs(got - exact) <= RTOL * exact
            results.append(got)
        # the shared scratch keeps nothing from call to call
        assert results[0] == results[2]
        # after the first (set-up) call, calls take no device memory
        assert free_after[1] == free_after[0] and free_after[2] == free_after[0], free_after
    finally:
        for pk in prepared:
            pk.close()
        dev.free(out)


def test_noalloc_rejects_bad_sizes():
    from ptxgen.runtime import Device
    dev = Device.get(0)
    fn = dev.L.emmy_sum_f32_noalloc
    fn.restype = C.c_int
    fn.argtypes = [C.c_uint64, C.c_size_t, C.c_uint64, C.c_void_p]
    buf = dev.alloc(64)
    try:
        assert fn(buf, 0, buf, dev.stream) == -3
        assert fn(buf, 1 << 31, buf, dev.stream) == -3
        assert b"2^31" in dev.L.emmy_last_error()
        assert fn(buf, 16, buf + 2, dev.stream) == -3
        assert b"4-byte" in dev.L.emmy_last_error()
    finally:
        dev.free(buf)
