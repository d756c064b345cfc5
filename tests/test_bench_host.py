"""Host-side logic of bench.py and of the matmul plan, on the CPU.

* block-seeded inputs: any shard of a generated array holds the same
  numbers as the same rows of the whole array, whatever the shard bounds
  (so a strong-scaling run splits one fixed problem);
* the strong-scaling shards of every record cover the named shape exactly
  (no gap, no overlap) at 1, 2, 4 and 8 ranks;
* the matmul's K-slice choice: unsliced by default, split-K IR split only
  to give every SM a unit, and the opt-in slicing bounded by its maximum.
"""

import numpy as np
import pytest

import bench
from ptxgen import irgen, tmpl_mma
from ptxgen.loader import load_kernel_data


@pytest.mark.parametrize("kind", ["u01", "u11", "normal"])
def test_shards_equal_rows_of_the_whole(kind):
    shape = (3000, 700)
    whole = bench.gen_rows(kind, 7, shape, 0, shape[0])
    for lo, hi in ((0, 1), (1, 2999), (1497, 1498), (800, 2300), (2999, 3000)):
        assert np.array_equal(bench.gen_rows(kind, 7, shape, lo, hi), whole[lo:hi])
    one_d = bench.gen_rows(kind, 9, ((1 << 21) + 5,), 0, (1 << 21) + 5)
    assert np.array_equal(bench.gen_rows(kind, 9, ((1 << 21) + 5,), 1 << 20, (1 << 21) + 5),
                          one_d[1 << 20:])


def test_generated_distributions():
    u01 = bench.gen_rows("u01", 1, (1 << 20,), 0, 1 << 20)
    u11 = bench.gen_rows("u11", 2, (1 << 20,), 0, 1 << 20)
    nrm = bench.gen_rows("normal", 3, (1 << 20,), 0, 1 << 20, scale=0.1, offset=1.0)
    assert u01.min() >= 0 and u01.max() < 1 and abs(u01.mean() - 0.5) < 0.01
    assert u11.min() >= -1 and u11.max() < 1 and abs(u11.mean()) < 0.01
    assert abs(nrm.mean() - 1.0) < 0.01 and abs(nrm.std() - 0.1) < 0.01
    assert u01.dtype == u11.dtype == nrm.dtype == np.float32


@pytest.mark.parametrize("world", [1, 2, 4, 8])
def test_strong_shards_cover_the_shapes(world):
    for n, align in ((1 << 26, 256), (1 << 28, 256), (8192, 1), (65536, 1), (8192, 128),
                     (16384, 128), (512, 32)):
        spans = [bench.shard(n, world, r, align) for r in range(world)]
        assert spans[0][0] == 0 and spans[-1][1] == n
        for (a0, a1), (b0, b1) in zip(spans, spans[1:]):
            assert a1 == b0 and a0 < a1
        assert all(s % align == 0 for s, _ in spans)


def _plan(gm):
    return tmpl_mma.match_matmul(load_kernel_data(*gm, "x"))


def test_matmul_unsliced_by_default(monkeypatch):
    monkeypatch.delenv("EMMY_MATMUL_MAX_SLICE_K", raising=False)
    for m, n, k in ((8192, 8192, 8192), (16384, 4096, 1024), (1024, 8192, 8192)):
        assert _plan(irgen.matmul(m, n, k)).slices == 1


def test_splitk_ir_splits_only_to_fill_the_sms(monkeypatch):
    monkeypatch.delenv("EMMY_MATMUL_MAX_SLICE_K", raising=False)
    # 2048 tiles: every SM already has work, the IR's 8 slices collapse to 1
    assert _plan(irgen.matmul_splitk(16384, 4096, 1024, slice_k=128)).slices == 1
    # 2 tiles: as many slices as the IR has (16 units, fewer than 148)
    assert _plan(irgen.matmul_splitk(256, 256, 1024, slice_k=128)).slices == 8
    # 64 tiles: 4 slices give every SM a unit (256 >= 148), 2 do not
    assert _plan(irgen.matmul_splitk(1024, 2048, 1024, slice_k=128)).slices == 4


def test_opt_in_slicing_bounds_the_slice(monkeypatch):
    monkeypatch.setenv("EMMY_MATMUL_MAX_SLICE_K", "1024")
    p = _plan(irgen.matmul(8192, 8192, 8192))
    assert p.slices == 8 and p.slice_k == 1024
    p = _plan(irgen.matmul(16384, 4096, 1024))
    assert p.slices == 1
    monkeypatch.setenv("EMMY_MATMUL_MAX_SLICE_K", "2048")
    assert _plan(irgen.matmul(8192, 8192, 8192)).slice_k == 2048


def test_sliced_plan_asks_the_launcher_to_clear_c(monkeypatch):
    from ptxgen.emit import compile_kernel
    from ptxgen.runtime import parse_plan
    monkeypatch.setenv("EMMY_MATMUL_MAX_SLICE_K", "1024")
    plan = parse_plan(compile_kernel(load_kernel_data(*irgen.matmul(1024, 1024, 4096), "y")))
    assert plan["split_k"] == 4 and plan["zero"] == ["matmul"] and "overwrites" not in plan
    monkeypatch.delenv("EMMY_MATMUL_MAX_SLICE_K")
    plan = parse_plan(compile_kernel(load_kernel_data(*irgen.matmul(1024, 1024, 4096), "z")))
    assert plan["split_k"] == 1 and plan["overwrites"] == ["matmul"] and "zero" not in plan


def test_record_table_names_every_baseline_config():
    assert set(bench.RECORDS) == {"reductions", "pointwise", "rows", "matmul_square",
                                  "matmul_rect", "matmul_splitk8", "attention_f32",
                                  "attention_bf16"}
    assert bench.ALIASES["matmul"] == ["matmul_square", "matmul_rect", "matmul_splitk8"]


def test_live_durations_apportion_the_timed_step():
    """The roofline's kernel durations: one kernel takes the whole timed
    step; several share it in proportion to their back-to-back times alone
    (which the power cap may stretch uniformly after the timed region)."""
    assert bench.live_durations(3.6, {"attention_bf16": 3.85}) == {"attention_bf16": 3.6}
    live = bench.live_durations(4.35, {"m.pre": 0.27, "m": 4.33})
    assert abs(sum(live.values()) - 4.35) < 1e-12
    assert abs(live["m"] / live["m.pre"] - 4.33 / 0.27) < 1e-9


def test_e2e_copies_each_shared_input_once():
    """The end-to-end step copies every distinct host array once: a job
    reading an array an earlier job takes is bound to that job's device
    copy and bound back afterwards; an argument a kernel also writes is
    never shared."""
    from types import SimpleNamespace as NS

    class PK:
        def __init__(self, bufs):
            self.bufs = dict(bufs)

        def bind(self, name, ptr):
            old, self.bufs[name] = self.bufs[name], ptr
            return old

    def job(key, bufs, inputs, outs=()):
        args = {n: NS(output=n in outs) for n in bufs}
        return NS(key=key, pk=PK(bufs), inputs=inputs, spec=NS(args=args))

    x, xr = np.zeros(4), np.ones(4)
    s = job("sum", {"x": 100}, {"x": x})
    m = job("mean", {"x": 200}, {"x": x})
    r = job("row_sum", {"x": 300}, {"x": xr})
    w = job("inplace", {"x": 400}, {"x": x}, outs=("x",))
    copies, rebound = bench.e2e_copy_plan([s, m, r, w])
    assert [(c[0].key, c[1]) for c in copies] == [("sum", "x"), ("row_sum", "x"), ("inplace", "x")]
    assert m.pk.bufs["x"] == 100 and [(j.key, n, own) for j, n, own in rebound] == [("mean", "x", 200)]
    for j, n, own in rebound:
        j.pk.bind(n, own)
    assert m.pk.bufs["x"] == 200
