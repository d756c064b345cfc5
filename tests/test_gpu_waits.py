"""Failure detection on the GPU: every spin-wait in these kernels is bounded,
and when its limit runs out the kernel records an error code in its error
word, leaves its waits, releases what it holds and returns -- the context
stays usable.  Each test makes one wait run out on purpose with a flag that
nothing ever sets (no fault, no trap, no endless loop) and checks the
status the host reads, then runs the same kernel again normally.

* the cross-GPU exchange of the full reduction (``tmpl_mem``): one GPU, a
  fake second rank whose inbox slot is a local buffer nobody flags; the
  last CTA waits 2 s for that rank's flag, then reports 0x203;
* the tcgen05 matmul's mbarrier waits (``tmpl_mma``): the wait limit
  lowered to 0.2 s through the module global ``emmy_wait_ns`` and the test
  hook ``emmy_test_stall`` set, so the MMA issuer waits on a barrier nothing
  arrives on; it reports 0x201, the producer and the epilogue leave their
  waits on the abort flag, the copies in flight land, TMEM is freed.

The reference reports the failures of its remote runner as stages of its
HTTP reply (``docs/API.md:55-58``); here the kernel's error word plays that
part for the local launcher.
"""

import time

import numpy as np
import pytest

from ptxgen import irgen
from ptxgen.loader import load_kernel_data

pytestmark = pytest.mark.gpu


class _Inbox:
    def __init__(self, ptrs):
        self.ptrs, self.world, self.rank = list(ptrs), len(ptrs), 0


def test_peer_exchange_wait_runs_out():
    from ptxgen.runtime import Device, EmmyError, PreparedKernel
    dev = Device.get(0)
    n = 1 << 20
    spec = load_kernel_data(*irgen.reduce_full(n, pid="xwait"), "sum_xwait")
    x = np.random.default_rng(1).random(n, dtype=np.float32)
    pk = PreparedKernel(spec, dev=dev)
    own, fake = dev.alloc(4096), dev.alloc(4096)
    try:
        assert pk.plan.get("xgpu"), "the full reduction has no cross-GPU exchange"
        for b in (own, fake):
            dev.memset32(b, 0, 1024)
        pk.upload({"x": x})
        pk.attach_peers(_Inbox([own, fake]))     # rank 1 never raises its flag
        t0 = time.perf_counter()
        pk.launch()
        with pytest.raises(EmmyError, match="0x203"):
            pk.check_errors()
        waited = time.perf_counter() - t0
        assert 1.9 < waited < 30, waited
        # alone again: the same kernel runs and sums correctly
        pk.attach_peers(_Inbox([own]))
        pk.launch()
        pk.check_errors()
        got = float(pk.download()["sum_1"][0])
        exact = float(x.astype(np.float64).sum())
        assert abs(got - exact) <= 1e-5 * exact
    finally:
        pk.close()
        dev.free(own)
        dev.free(fake)


def test_matmul_mbarrier_wait_runs_out():
    from ptxgen.runtime import Device, EmmyError, PreparedKernel
    dev = Device.get(0)
    m, n, k = 384, 256, 128          # a shape no other test compiles (own module)
    spec = load_kernel_data(*irgen.matmul(m, n, k), "mm_wait")
    rng = np.random.default_rng(2)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    pk = PreparedKernel(spec, dev=dev)
    lim, _ = pk.mod.global_ptr("emmy_wait_ns")
    stall, _ = pk.mod.global_ptr("emmy_test_stall")
    try:
        pk.upload({"x0": a, "x1": b})
        dev.htod(lim, np.array([200_000_000], np.uint64))
        dev.htod(stall, np.array([1], np.uint32))
        t0 = time.perf_counter()
        pk.launch()
        with pytest.raises(EmmyError, match="0x201"):
            pk.check_errors()
        waited = time.perf_counter() - t0
        assert 0.19 < waited < 30, waited
    finally:
        dev.htod(stall, np.array([0], np.uint32))
        dev.htod(lim, np.array([4_000_000_000], np.uint64))
        dev.sync()
    try:
        # the hook cleared: the same kernel runs on tcgen05 and is right
        pk.launch()
        pk.check_errors()
        got = pk.download()["matmul"].astype(np.float64)
        ref = a.astype(np.float64) @ b.astype(np.float64)
        assert np.abs(got - ref).max() <= 1e-4 * np.abs(ref).max()
    finally:
        pk.close()


def test_closed_kernel_leaves_no_peer_state():
    """Modules are shared by every prepared kernel of the same PTX: closing a
    kernel that joined an exchange resets the module's world and peer
    addresses, so the next kernel of that PTX runs alone instead of storing
    into a freed inbox."""
    from ptxgen.runtime import Device, PreparedKernel
    dev = Device.get(0)
    n = 1 << 16
    spec = load_kernel_data(*irgen.reduce_full(n, pid="xdetach"), "sum_xdetach")
    x = np.random.default_rng(3).random(n, dtype=np.float32)
    own, other = dev.alloc(4096), dev.alloc(4096)
    pk = PreparedKernel(spec, dev=dev)
    xg = pk.plan["xgpu"]
    pk.attach_peers(_Inbox([own, other]))
    pk.close()
    dev.free(own)
    dev.free(other)
    pk2 = PreparedKernel(spec, dev=dev)
    try:
        assert pk2.mod is pk.mod
        world = np.zeros(1, np.uint32)
        peers = np.ones(int(xg["max_ranks"]), np.uint64)
        dev.dtoh(world, pk2.mod.global_ptr(xg["world"])[0])
        dev.dtoh(peers, pk2.mod.global_ptr(xg["peers"])[0])
        dev.sync()
        assert world[0] == 0 and not peers.any()
        pk2.upload({"x": x})
        pk2.launch()
        pk2.check_errors()
        got = float(pk2.download()["sum_1"][0])
        assert abs(got - float(x.astype(np.float64).sum())) <= 1e-5 * float(x.sum())
    finally:
        pk2.close()
