#!/usr/bin/env python3
"""Benchmark of the Emmy Kernel IR -> B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--records all|none|NAME,...] [--impl ours|reference]

One step = one pass of the compiled IR kernels of a BASELINE configuration
over one batch of synthetic inputs already resident in HBM.  The printed
line is the default workload, BASELINE configs[1] (the reductions:
full-array sum and mean over 2**26 f32 ~ U[0,1] and the row sum of an
8192 x 8192 f32 ~ N(0,1) matrix), with every other BASELINE configuration
measured in the same process as a sub-record under ``workloads``:

* ``pointwise``       configs[0] at the bench size: c = a + b, 2**28 f32;
* ``rows``            configs[2]: RMSNorm, softmax, L2-norm on 65536 x 4096;
* ``matmul_square``   configs[3]: C = A.B, 8192^3 (3xTF32 on tcgen05);
* ``matmul_rect``     configs[3]: 16384 x 4096 x 1024;
* ``matmul_splitk8``  configs[3]: the split-K = 8 atomic variant;
* ``attention_f32``   configs[4]: [16, 32, 4096, 128] f32 (3xTF32);
* ``attention_bf16``  configs[4]: the bf16 variant.

Each record carries its own ``value``, ``dtype``, ``kernels_ms``,
``roofline`` (dominant kernel against ``MEASURED_PEAKS.json``), ``e2e``
(host buffers, copies inside the timed region), ``clocks``, ``parity``
(the shard's outputs checked before timing) and, on one GPU,
``cpu_baseline``.

Multi-GPU (launched by torch.distributed.run, one process per GPU): the
printed line stays weak scaling -- every rank owns a full-size reductions
workload, and the full sum and mean exchange their per-rank totals inside
the reduction kernel over NVLink peer inboxes (``--collective p2p``,
default) or with an NCCL all-reduce after it.  The sub-records are strong
scaling: ONE named shape is split across the ranks -- pointwise by element
range, rows and row sums by row blocks, matmul by M rows with the same B on
every rank, attention by batch x head, sum and mean by element range plus
the in-kernel exchange (record ``reductions``).  Value = the shape's total
algorithmic bytes or FLOPs / the max over ranks of the time.  Inputs come
from a block-seeded generator, so a shard holds the same numbers whatever
N is.  Where a rank's shard would fit in L2, the record cycles through
enough copies of its inputs that every step reads HBM.

``--impl reference`` times the reference's own CPU algorithm -- the oracle
restating ``ptxgen/interp.py`` -- on the full default configuration,
partitioned over every host core (rank 0 only).
"""

from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import sys
import time
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "emmy-ptx_b200"))
sys.path.insert(0, str(ROOT))

METRIC = "HBM GB/s (% of 8 TB/s) for mem-bound kernels; TFLOP/s for matmul/attn"
SPEC_HBM_GBS = 8000.0
FALLBACK_HBM_GBS = 6650.0
FALLBACK_BF16_TFLOPS = 1590.0
L2_BYTES = 126 << 20


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return {"hbm_gbs": float(d["hbm_gbs"]), "bf16_tflops": float(d["bf16_tflops"]),
                "bf16_tflops_sustained": float(d.get("bf16_tflops_sustained", d["bf16_tflops"])),
                "source": "measured"}
    return {"hbm_gbs": FALLBACK_HBM_GBS, "bf16_tflops": FALLBACK_BF16_TFLOPS,
            "bf16_tflops_sustained": 1400.0, "source": "fallback"}


# ---------------------------------------------------------------------------
# block-seeded synthetic inputs
# ---------------------------------------------------------------------------

BLOCK_ELEMS = 1 << 20


def gen_rows(kind: str, seed: int, shape, lo: int, hi: int, scale: float = 1.0,
             offset: float = 0.0) -> np.ndarray:
    """Rows [lo, hi) of a global f32 array of ``shape`` (split on its first
    axis).  Blocks of about 2**20 elements are drawn from
    ``default_rng([seed, block])``, so any shard holds the same numbers as
    the same rows of the whole array.  ``kind``: ``u01`` U[0,1), ``u11``
    U[-1,1), ``normal`` N(0,1); then ``x * scale + offset``."""
    from concurrent.futures import ThreadPoolExecutor
    shape = tuple(int(s) for s in shape)
    row = int(np.prod(shape[1:])) if len(shape) > 1 else 1
    rpb = max(1, BLOCK_ELEMS // row)
    out = np.empty((hi - lo,) + shape[1:], np.float32)

    def fill(b):
        r0, r1 = b * rpb, min((b + 1) * rpb, shape[0])
        rng = np.random.default_rng([seed, b])
        size = (r1 - r0,) + shape[1:]
        if kind == "u01":
            x = rng.random(size, dtype=np.float32)
        elif kind == "u11":
            x = rng.random(size, dtype=np.float32) * np.float32(2) - np.float32(1)
        else:
            x = rng.standard_normal(size, dtype=np.float32)
        if scale != 1.0 or offset != 0.0:
            x = (x * np.float32(scale) + np.float32(offset)).astype(np.float32)
        s0, s1 = max(r0, lo), min(r1, hi)
        out[s0 - lo:s1 - lo] = x[s0 - r0:s1 - r0]

    with ThreadPoolExecutor(max_workers=min(16, os.cpu_count() or 1)) as ex:
        list(ex.map(fill, range(lo // rpb, (hi + rpb - 1) // rpb)))
    return out


def shard(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    from ptxgen.dist import shard_range
    return shard_range(n, world, rank, align)


# ---------------------------------------------------------------------------
# records: jobs over this rank's shard
# ---------------------------------------------------------------------------


class Job:
    """One compiled kernel of a record with its inputs, work and check."""

    def __init__(self, key, spec, inputs, algo_bytes, algo_flops=0.0, allreduce=None,
                 check=None, local_ref=None, ref_div=1.0):
        self.key = key
        self.spec = spec
        self.inputs = inputs          # host arrays (uploaded per step in e2e)
        self.algo_bytes = algo_bytes  # per launch, this rank
        self.algo_flops = algo_flops  # per launch, this rank
        self.allreduce = allreduce    # output name reduced across ranks, or None
        self.check = check            # (outputs) -> None, raises on mismatch
        self.local_ref = local_ref    # this rank's f64 share of an all-reduced result
        self.ref_div = ref_div        # global result = sum over ranks of local_ref / ref_div
        self.inbox = None
        self.pk = None
        self.rot = []                 # extra input-buffer sets cycled through per step


def _spec(gm, name):
    from ptxgen.loader import load_kernel_data
    return load_kernel_data(gm[0], gm[1], name)


def _rows_f64(fam, x, g=None, eps=1e-6):
    x = x.astype(np.float64)
    if fam == "rmsnorm":
        return x / np.sqrt((x * x).mean(-1, keepdims=True) + eps) * g.astype(np.float64)
    if fam == "l2norm":
        return x / np.sqrt((x * x).sum(-1, keepdims=True))
    e = np.exp(x - x.max(-1, keepdims=True))
    return e / e.sum(-1, keepdims=True)


def record_reductions(rank, world, strong):
    """configs[1].  Weak: every rank the full 2**26 and 8192 x 8192 (its
    own seed).  Strong: element range of the 2**26 and row block of the
    8192 rows; the sum and mean exchange totals across the ranks."""
    from ptxgen import irgen
    N, R, Ccols = 1 << 26, 8192, 8192
    seed = 1000 if strong else 1000 + 7919 * rank
    lo, hi = shard(N, world, rank, 256) if strong else (0, N)
    r0, r1 = shard(R, world, rank) if strong else (0, R)
    n, rows = hi - lo, r1 - r0
    x = gen_rows("u01", seed, (N,), lo, hi)
    xr = gen_rows("normal", seed + 1, (R, Ccols), r0, r1)
    total = N * world if not strong else N
    s_spec = _spec(irgen.reduce_full(n, pid="sum_2p26"), "sum")
    m_spec = _spec(irgen.reduce_full(n, mean=True, pid="mean_2p26"), "mean")
    m_spec.args["mean_keepdim_count"].data = [float(total)]
    r_spec = _spec(irgen.reduce_rows(rows, Ccols, pid="row_sum"), "row_sum")
    local_sum = float(x.astype(np.float64).sum())

    def chk_sum(out, key="sum_1", div=1.0):
        got = float(out[key][0])
        want = local_sum / div
        if abs(got - want) > 1e-5 * abs(want):
            raise AssertionError(f"{key}: {got} vs {want}")

    def chk_rows(out):
        for a in range(0, rows, 1024):
            xs = xr[a:a + 1024].astype(np.float64)
            bound = 1e-5 * np.abs(xs).sum(-1)
            if np.any(np.abs(out["sum_1"][a:a + 1024] - xs.sum(-1)) > bound):
                raise AssertionError("row sums outside 1e-5 x sum|x|")

    jobs = [
        Job("sum", s_spec, {"x": x}, n * 4 + 4, allreduce="sum_1", check=chk_sum,
            local_ref=local_sum),
        Job("mean", m_spec, {"x": x}, n * 4 + 4, allreduce="mean",
            check=lambda o: chk_sum(o, "mean", float(total)), local_ref=local_sum,
            ref_div=float(total)),
        Job("row_sum", r_spec, {"x": xr}, rows * Ccols * 4 + rows * 4, check=chk_rows),
    ]
    cfg = {"workload": "configs[1] reductions: sum+mean over 2^26 f32 U[0,1], row sum "
                       "8192x8192 f32 N(0,1)",
           "shard": (f"elements [{lo}, {hi}) of 2^26, rows [{r0}, {r1}) of 8192" if strong
                     else "full size on every rank")}
    parity = ("sum and mean within 1e-5 of float64 (across ranks: of the ranks' float64 "
              "partials summed); every row sum within 1e-5 x sum|x| of float64")
    return jobs, cfg, "f32", parity


def record_pointwise(rank, world, strong=True):
    from ptxgen import irgen
    N = 1 << 28
    lo, hi = shard(N, world, rank, 256)
    n = hi - lo
    a = gen_rows("u11", 2000, (N,), lo, hi)
    b = gen_rows("u11", 2001, (N,), lo, hi)
    spec = _spec(irgen.pointwise(n, 4, "add", pid="vector_add_2p28"), "add")

    def chk(out):
        if not np.array_equal(out["add"], a + b):
            raise AssertionError("vector add not bit-exact")

    return ([Job("vector_add", spec, {"x0": a, "x1": b}, 12 * n, check=chk)],
            {"workload": "configs[0] at the bench size: c=a+b over 2^28 f32 U[-1,1]",
             "shard": f"elements [{lo}, {hi})"}, "f32",
            "every output bit for bit equal to IEEE f32 a + b")


def record_rows(rank, world, strong=True):
    from ptxgen import irgen
    R, Ccols = 65536, 4096
    r0, r1 = shard(R, world, rank)
    rows = r1 - r0
    x = gen_rows("normal", 3000, (R, Ccols), r0, r1)
    g = gen_rows("normal", 3001, (Ccols,), 0, Ccols, scale=0.1, offset=1.0)
    jobs = []
    for key, gm in (("rmsnorm", irgen.rmsnorm(rows, Ccols, eps=1e-6)),
                    ("softmax", irgen.softmax(rows, Ccols)), ("l2norm", irgen.l2norm(rows, Ccols))):
        spec = _spec(gm, key)
        ins = {"x": x}
        if key == "rmsnorm":
            ins["w"] = g

        def chk(out, key=key, spec=spec):
            y = out[spec.outputs[0]]
            for a in range(0, rows, 2048):
                ref = _rows_f64(key, x[a:a + 2048], g)
                bound = 1e-5 * np.abs(ref) + 1e-6 * np.abs(ref).max(-1, keepdims=True)
                if np.any(np.abs(y[a:a + 2048] - ref) > bound):
                    raise AssertionError(f"{key} rows from {a} outside tolerance")

        jobs.append(Job(key, spec, ins, 8 * rows * Ccols + (4 * Ccols if key == "rmsnorm" else 0),
                        check=chk))
    return (jobs, {"workload": "configs[2] fused rows: RMSNorm, softmax, L2-norm on 65536x4096 "
                               "f32 N(0,1), g ~ N(1,0.1)", "shard": f"rows [{r0}, {r1})"},
            "f32", "every row within 1e-5 |ref| + 1e-6 max|ref row| of float64")


MATMUL_SHAPES = {"matmul_square": (8192, 8192, 8192, False),
                 "matmul_rect": (16384, 4096, 1024, False),
                 "matmul_splitk8": (16384, 4096, 1024, True)}


def record_matmul(name, rank, world, strong=True):
    from ptxgen import irgen
    from tests.contraction import matmul_check
    M, Nn, K, splitk = MATMUL_SHAPES[name]
    r0, r1 = shard(M, world, rank, 128)
    m = r1 - r0
    gm = (irgen.matmul_splitk(m, Nn, K, slice_k=K // 8) if splitk else irgen.matmul(m, Nn, K))
    spec = _spec(gm, name)
    seed = {"matmul_square": 4000, "matmul_rect": 4100, "matmul_splitk8": 4100}[name]
    a = gen_rows("u11", seed, (M, K), r0, r1, scale=1 / math.sqrt(K))
    b = gen_rows("u11", seed + 1, (K, Nn), 0, K, scale=1 / math.sqrt(K))   # same B on every rank

    def chk(out):
        rows = np.linspace(0, m - 1, 64).astype(np.int64)
        ok, elem, block = matmul_check(out["matmul"], a, b, rows)
        if not ok:
            raise AssertionError(f"{name} outside the contraction bounds: {elem}, {block}")

    job = Job(name, spec, {"x0": a, "x1": b}, 4 * (m * K + K * Nn + m * Nn),
              algo_flops=2.0 * m * Nn * K, check=chk)
    what = {"matmul_square": "C=A.B 8192^3", "matmul_rect": "C=A.B 16384x4096x1024",
            "matmul_splitk8": "split-K=8 (atomic IR) 16384x4096x1024"}[name]
    return ([job], {"workload": f"configs[3] f32 matmul (3xTF32 on tcgen05): {what}, "
                                "A,B ~ U[-1,1]/sqrt(K)",
                    "shard": f"rows [{r0}, {r1}) of A and C, B replicated"},
            "f32 (3xTF32)",
            "64 rows of the shard: |err| <= 2^-15 sum|a||b| and <= 1e-4 max|ref| per 16 rows")


def record_attention(dt, rank, world, strong=True):
    from ptxgen import irgen
    from tests.contraction import attention_check, attention_ref
    B, H, S, D = 16, 32, 4096, 128
    if _SMALL:
        B = 1
    h0, h1 = shard(B * H, world, rank, H)
    bh = h1 - h0
    b = bh // H
    spec = _spec(irgen.attention_bhsd(b, H, S, D, dt, pid=f"attn_{dt}"), f"attn_{dt}")
    qkv = [gen_rows("normal", 5000 + i, (B * H, S, D), h0, h1).reshape(b, H, S, D)
           for i in range(3)]
    if dt == "bf16":
        from ml_dtypes import bfloat16
        qkv = [x.astype(bfloat16) for x in qkv]
    q, k, v = qkv

    def chk(out):
        for (bi, hi) in ((0, 0), (b - 1, H // 2 + 1), (b // 2, H - 1)):
            rows = np.arange(0, S, 257)
            ref = attention_ref(q[bi, hi, rows], k[bi, hi], v[bi, hi])
            got = out["out"][bi, hi, rows].astype(np.float64)
            if dt == "f32":
                ok, worst = attention_check(got, ref)
            else:
                worst = float(np.abs(got - ref).max() / np.abs(ref).max())
                ok = worst <= 2e-2
            if not ok:
                raise AssertionError(f"attention {dt} ({bi},{hi}) outside tolerance: {worst}")

    e = 4 if dt == "f32" else 2
    job = Job(f"attention_{dt}", spec, {"q": q, "k": k, "v": v}, 4 * bh * S * D * e,
              algo_flops=4.0 * bh * S * S * D, check=chk)
    return ([job], {"workload": f"configs[4] attention softmax(QK^T/sqrt(d))V, [16,32,4096,128] "
                                f"{dt}{' (3xTF32)' if dt == 'f32' else ''}, non-causal",
                    "shard": f"batch x head [{h0}, {h1}) of {B * H}"},
            "f32 (3xTF32)" if dt == "f32" else "bf16",
            ("f32: per sampled query row max|err| <= 1e-4 max|ref| of float64" if dt == "f32"
             else "bf16: max|err| <= 2e-2 max|ref| of float64 on sampled rows"))


def e2e_copy_plan(jobs):
    """The host-to-device copies of one end-to-end step: every distinct
    input array once.  A job that reads an array an earlier job already
    takes (the full sum and the mean read the same x) is bound to that
    job's device copy (``PreparedKernel.bind``), unless either kernel also
    writes the argument.  Returns the copies as (job, name, array) and the
    rebindings as (job, name, the job's own buffer) for undoing them."""
    first, copies, rebound = {}, [], []
    for j in jobs:
        for n, arr in j.inputs.items():
            src = first.get(id(arr))
            if src is not None and not j.spec.args[n].output \
                    and not src[0].spec.args[src[1]].output:
                rebound.append((j, n, j.pk.bind(n, src[0].pk.bufs[src[1]])))
                continue
            first.setdefault(id(arr), (j, n))
            copies.append((j, n, arr))
    return copies, rebound


def live_durations(step_ms: float, alone_ms: dict) -> dict:
    """Each kernel's duration over the timed region: the timed step (max
    over ranks) times the kernel's share of the back-to-back launch times
    measured alone -- the step itself when a record has one kernel.  The
    back-to-back loop runs after the timed region, at whatever clock the
    power cap then allows, so it gives the shares and not the durations."""
    total = sum(alone_ms.values())
    return {k: step_ms * v / total for k, v in alone_ms.items()}


_SMALL = False
# The jobs of a record never read what another job (or the previous launch
# of the same job) writes, so kernels whose plans allow it start while the
# previous kernel in the stream finishes (programmatic dependent launch).
OVERLAP = True

RECORDS = {
    "reductions": lambda r, w, s: record_reductions(r, w, s),
    "pointwise": lambda r, w, s: record_pointwise(r, w),
    "rows": lambda r, w, s: record_rows(r, w),
    "matmul_square": lambda r, w, s: record_matmul("matmul_square", r, w),
    "matmul_rect": lambda r, w, s: record_matmul("matmul_rect", r, w),
    "matmul_splitk8": lambda r, w, s: record_matmul("matmul_splitk8", r, w),
    "attention_f32": lambda r, w, s: record_attention("f32", r, w),
    "attention_bf16": lambda r, w, s: record_attention("bf16", r, w),
}
# the workloads of round-1 command lines, kept as aliases
ALIASES = {"matmul": ["matmul_square", "matmul_rect", "matmul_splitk8"],
           "attention": ["attention_f32", "attention_bf16"]}


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------


def _nvml_handle(N, cuda_index: int):
    """NVML handle of CUDA device ``cuda_index``: NVML ignores
    CUDA_VISIBLE_DEVICES, so map through it (indices or UUIDs)."""
    vis = os.environ.get("CUDA_VISIBLE_DEVICES", "").strip()
    if vis:
        items = [v.strip() for v in vis.split(",") if v.strip()]
        if cuda_index < len(items):
            it = items[cuda_index]
            if it.isdigit():
                return N.nvmlDeviceGetHandleByIndex(int(it))
            return N.nvmlDeviceGetHandleByUUID(it)
    return N.nvmlDeviceGetHandleByIndex(cuda_index)


class ClockSampler:
    """Samples SM clock and throttle reasons while the timed region runs:
    NVML polled every half millisecond from a thread (read-only queries)."""

    REASONS = {"hw_slowdown": 0x8, "hw_thermal_slowdown": 0x40, "sw_thermal_slowdown": 0x20,
               "sw_power_cap": 0x4}

    def __init__(self, index: int):
        self.index = index
        self.samples = []
        self.smax = None
        self._stop = False
        self.error = None

    def _poll(self):
        try:
            import pynvml as N
            h = _nvml_handle(N, self.index)
            self.smax = N.nvmlDeviceGetMaxClockInfo(h, N.NVML_CLOCK_SM)
            get_reasons = getattr(N, "nvmlDeviceGetCurrentClocksEventReasons", None) or \
                getattr(N, "nvmlDeviceGetCurrentClocksThrottleReasons")
        except Exception as exc:  # noqa: BLE001
            self.error = f"{type(exc).__name__}: {exc}"
            return
        while not self._stop:
            try:
                self.samples.append((N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM), get_reasons(h)))
            except Exception as exc:  # noqa: BLE001
                self.error = f"{type(exc).__name__}: {exc}"
            time.sleep(0.0005)

    def __enter__(self):
        import threading
        self.thread = None
        try:
            import pynvml as N
            N.nvmlInit()
            self.thread = threading.Thread(target=self._poll, daemon=True)
            self.thread.start()
            t0 = time.perf_counter()
            while not self.samples and self.error is None and time.perf_counter() - t0 < 5:
                time.sleep(0.001)
        except Exception:
            self.thread = None
        self.first = 0
        return self

    def mark(self):
        """Samples from here on belong to the timed region."""
        self.first = len(self.samples)

    def __exit__(self, *a):
        self._stop = True
        if self.thread is not None:
            self.thread.join(timeout=2)

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.smax, "reasons": [], "samples": 0,
                    "source": "nvml", "error": self.error}
        window = self.samples[self.first:] or self.samples[-1:]
        mhz = [m for m, _ in window]
        reasons = sorted({n for _, r in window for n, bit in self.REASONS.items() if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.smax, "reasons": reasons,
                "samples": len(mhz), "source": "nvml"}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


class Dist:
    """This process's place in the job (torch.distributed.run env) and the
    host-side rendezvous; see ``ptxgen.dist``."""

    def __init__(self):
        from ptxgen.dist import Rendezvous
        self.rdv = Rendezvous(timeout_s=300)
        self.rank, self.world, self.local = self.rdv.rank, self.rdv.world, self.rdv.local

    def barrier(self):
        self.rdv.barrier()

    def max(self, v: float) -> float:
        return self.rdv.max(v)

    def close(self):
        self.rdv.close()


# ---------------------------------------------------------------------------
# measuring one record
# ---------------------------------------------------------------------------


def measure(name: str, args, dist: Dist, strong: bool, dev) -> dict:
    """Prepare, check and time one record on this rank; every rank takes the
    same steps in the same order (the in-kernel exchange meets every rank's
    launch)."""
    import ctypes as C
    from ptxgen.runtime import PreparedKernel, _np_dtype, check
    jobs, cfg, dtype, parity = RECORDS[name](dist.rank, dist.world, strong)
    if args.jobs:
        keep = set(args.jobs.split(","))
        jobs = [j for j in jobs if j.key in keep] or jobs
    comm = None
    for j in jobs:
        j.pk = PreparedKernel(j.spec, dev=dev)
        j.pk.upload(j.inputs)
    dev.sync()
    # HBM-bound records whose shard would fit in L2 cycle through copies of
    # their inputs, so that a step never re-reads what the previous ones left
    step_in = sum(j.pk.spec.args[n].nbytes for j in jobs for n in j.inputs)
    nrot = 1
    if not any(j.algo_flops for j in jobs) and step_in < 2 * L2_BYTES:
        nrot = math.ceil(2 * L2_BYTES / max(step_in, 1))
        for j in jobs:
            j.base = {n: j.pk.bufs[n] for n in j.inputs}
            for _ in range(nrot - 1):
                copy = {}
                for n in j.inputs:
                    nb = j.pk.spec.args[n].nbytes
                    copy[n] = dev.alloc(nb)
                    dev.dtod(copy[n], j.base[n], nb)
                j.rot.append(copy)
        dev.sync()
        cfg["l2"] = f"shard inputs below 2 x L2: {nrot} copies cycled step by step"
    else:
        cfg["l2"] = "every input is larger than the 126 MB L2" if not any(
            j.algo_flops for j in jobs) else "compute-bound; operands re-read through L2 by design"
    if dist.world > 1 and args.collective == "p2p":
        from ptxgen.dist import PeerInbox
        for j in jobs:
            if j.allreduce and j.pk.plan.get("xgpu"):
                j.inbox = PeerInbox(dev, dist.rdv)
                j.pk.attach_peers(j.inbox)
                j.allreduce = None
                cfg["collective"] = "fused in-kernel exchange over NVLink peer inboxes"
    if dist.world > 1 and any(j.allreduce for j in jobs):
        from ptxgen.dist import NcclComm
        comm = NcclComm(dev, dist.rdv)
        nccl_stream = dev.new_stream()
        ev_ready, ev_done = dev.event(), dev.event()
        cfg["collective"] = "NCCL all-reduce on a second stream"
    last_ar = max((i for i, j in enumerate(jobs) if j.allreduce), default=-1)
    # With the in-kernel exchange, a reduction's last CTA waiting for the other
    # GPUs must overlap the step's other kernels: with overlapped launches the
    # next kernel in the one stream streams meanwhile; without them each job
    # runs on its own stream (forked from and joined back to the main stream
    # every step -- the event waits would break the launches' adjacency).
    concurrent = any(j.inbox is not None for j in jobs) and not OVERLAP
    if concurrent:
        ev_fork = dev.event()
        for j in jobs:
            j.stream, j.ev_join = dev.new_stream(), dev.event()
        cfg["streams"] = "one stream per job, forked and joined every step"
    if OVERLAP and any(j.pk.plan.get("overlap") for j in jobs):
        cfg["launch"] = ("programmatic dependent launch: kernels whose plan allows it start "
                         "while the previous one finishes and wait for it before their "
                         "first write")
    counter = [0]

    def rotate():
        if nrot > 1:
            r = counter[0] % nrot
            for j in jobs:
                j.pk.bufs.update(j.base if r == 0 else j.rot[r - 1])
        counter[0] += 1

    def launch_all():
        if concurrent:
            dev.record(ev_fork)
            for j in jobs:
                dev.wait_event(j.stream, ev_fork)
                if j.pk.has_pre:
                    j.pk.launch_pre(j.stream)
                j.pk.launch_main(j.stream, overlap=OVERLAP)
                dev.record(j.ev_join, j.stream)
            for j in jobs:
                dev.wait_event(dev.stream, j.ev_join)
            return
        pending = []
        for i, j in enumerate(jobs):
            if j.pk.has_pre:
                j.pk.launch_pre()
            j.pk.launch_main(overlap=OVERLAP)
            if comm is not None and j.allreduce:
                pending.append(j)
            if pending and i == last_ar:
                # all-reduce the per-rank results on a second stream,
                # overlapped with the kernels still to run on the main stream
                dev.record(ev_ready)
                dev.wait_event(nccl_stream, ev_ready)
                for pj in pending:
                    a = pj.spec.args[pj.allreduce]
                    comm.allreduce_sum_f32(pj.pk.bufs[pj.allreduce], a.numel, nccl_stream)
                dev.record(ev_done, nccl_stream)
        if pending:
            dev.wait_event(dev.stream, ev_done)

    def step():
        rotate()
        launch_all()

    for _ in range(args.warmup):
        step()
    dev.sync()
    # untimed ramp: about 0.3 s of steps so the GPU leaves idle clocks; the
    # step count is agreed across ranks
    t_ramp = time.perf_counter()
    for _ in range(4):
        step()
    dev.sync()
    per4 = dist.max(time.perf_counter() - t_ramp)
    for _ in range(min(400, max(1, int(0.3 / max(per4, 1e-4))))):
        for _ in range(4):
            step()
    dev.sync()
    # parity of this rank's shard, on the outputs of the steps just run
    for j in jobs:
        j.pk.check_errors()
        if j.allreduce is None and j.inbox is None and j.check is not None:
            j.check(j.pk.download())
        elif j.local_ref is not None:
            name_o = j.spec.outputs[0]
            got = float(j.pk.download([name_o])[name_o].reshape(-1)[0])
            want = dist.rdv.sum(j.local_ref) / j.ref_div
            if abs(got - want) > 1e-5 * abs(want):
                raise AssertionError(f"{j.key} over {dist.world} ranks: {got} vs {want}")
    # ---- timed region: device-resident inputs, events only at its ends ----
    t0, t1 = dev.event(), dev.event()
    dist.barrier()
    dev.sync()
    with ClockSampler(dist.local) as clk:
        for _ in range(4):           # re-warm after the set-up's idle gap
            step()
        clk.mark()
        dev.record(t0)
        for _ in range(args.steps):
            step()
        dev.record(t1)
        dev.sync()
    dist.barrier()
    total_ms = dev.elapsed_ms(t0, t1)
    # ---- per-kernel durations: each job alone, ``steps`` back-to-back
    # launches between two events on the launching stream ----
    per_kernel = {}
    dev.sync()
    for j in jobs:
        batches = ([(j.key + ".pre", j.pk.launch_pre)] if j.pk.has_pre else [])
        batches.append((j.key, lambda j=j: j.pk.launch_main(overlap=OVERLAP)))
        for key, launch in batches:
            a, b = dev.event(), dev.event()
            dev.record(a)
            for _ in range(args.steps):
                rotate()
                launch()
            dev.record(b)
            dev.sync()
            per_kernel[key] = dev.elapsed_ms(a, b) / args.steps
    for j in jobs:
        j.pk.check_errors()
    ms = dist.max(total_ms) / args.steps
    # ---- e2e: host buffers through the public launch API ----
    pinned = {}
    for j in jobs:
        for n, arr in j.inputs.items():
            if id(arr) in pinned:
                continue
            raw = np.ascontiguousarray(arr).view(np.uint8).reshape(-1)
            p = dev.host_alloc(raw.nbytes)
            np.ctypeslib.as_array((C.c_uint8 * raw.nbytes).from_address(p))[:] = raw
            pinned[id(arr)] = (p, raw.nbytes)
    # results land in pinned host memory too (a pageable destination makes
    # the driver stage the copy and halves its rate)
    out_pinned = []

    def pinned_array(shape, dtype):
        nb = int(np.prod(shape)) * np.dtype(dtype).itemsize
        p = dev.host_alloc(max(nb, 1))
        out_pinned.append(p)
        return np.ctypeslib.as_array((C.c_uint8 * nb).from_address(p)).view(dtype).reshape(shape)

    out_host = {j.key: {o: pinned_array(j.spec.args[o].shape, _np_dtype(j.spec.args[o].dtype))
                        for o in j.spec.outputs} for j in jobs}
    if nrot > 1:
        for j in jobs:
            j.pk.bufs.update(j.base)
    copies, rebound = e2e_copy_plan(jobs)

    def e2e_step():
        nb_in = nb_out = 0
        for j, n, arr in copies:
            p, nb = pinned[id(arr)]
            check(dev.L.emmy_memcpy_htod(C.c_uint64(j.pk.bufs[n]), C.c_void_p(p), nb,
                                         dev.stream), "htod")
            nb_in += nb
        launch_all()
        for j in jobs:
            for o, host in out_host[j.key].items():
                dev.dtoh(host, j.pk.bufs[o])
                nb_out += host.nbytes
        return nb_in, nb_out

    for _ in range(max(1, min(args.warmup, 2))):
        e2e_step()
    dev.sync()
    e0, e1 = dev.event(), dev.event()
    dist.barrier()
    dev.sync()
    esteps = max(1, min(args.steps, 5))
    dev.record(e0)
    for _ in range(esteps):
        h2d, d2h = e2e_step()
    dev.record(e1)
    dev.sync()
    dist.barrier()
    e2e_ms = dist.max(dev.elapsed_ms(e0, e1)) / esteps
    for p, _ in pinned.values():
        dev.host_free(p)
    out_host = None
    for p in out_pinned:
        dev.host_free(p)
    for j, n, own in rebound:
        j.pk.bind(n, own)

    # ---- figures ----
    # the whole job's work: every rank's shard (weak: every rank's copy)
    bytes_step = dist.rdv.sum(sum(j.algo_bytes for j in jobs))
    flops_step = dist.rdv.sum(sum(j.algo_flops for j in jobs))
    pk = peaks()
    dom = max(jobs, key=lambda j: per_kernel[j.key])
    live_ms = live_durations(ms, per_kernel)
    dom_ms = live_ms[dom.key]
    traffic = None
    tpath = ROOT / "profiles" / "traffic.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get(f"{name}:{dom.key}")
        if traffic is not None and dist.world > 1:
            traffic = None            # captured on the full one-GPU shape
    clocks = clk.summary()
    if dom.algo_flops:
        achieved = dom.algo_flops / (dom_ms * 1e-3) / 1e12
        # a tensor-bound kernel whose clocks the power cap held down (the cap
        # seen and the median SM clock 5 % or more below the maximum) is held
        # to the sustained dense-bf16 figure (cuBLAS over seconds under the
        # cap), any other to the burst figure; both fractions are reported
        smax = clocks.get("sm_max_mhz") or 0
        capped = ("sw_power_cap" in clocks.get("reasons", []) and smax
                  and (clocks.get("sm_mhz") or smax) < 0.95 * smax)
        tf = pk["bf16_tflops_sustained"] if capped else pk["bf16_tflops"]
        which = "sustained" if capped else "burst"
        div = 1.0 if dtype == "bf16" else 6.0
        roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(tf / div, 1),
                "unit": "TFLOP/s",
                "frac_burst": round(achieved / (pk["bf16_tflops"] / div), 4),
                "frac_sustained": round(achieved / (pk["bf16_tflops_sustained"] / div), 4)}
        if dtype == "bf16":
            roof["peak_note"] = (f"measured dense bf16, {which} (the power cap "
                                 f"{'held' if capped else 'did not hold'} this record's median "
                                 f"SM clock below 95 % of the maximum)")
        else:
            # 3xTF32: three TF32 products per useful f32 product; TF32 runs at
            # half the dense bf16 rate, so the useful-flop ceiling is bf16 / 6
            roof["peak_note"] = (f"3xTF32 useful-flop ceiling = measured dense bf16 {which} "
                                 f"{tf} / 2 (tf32) / 3 (passes)")
            roof["tensor_pipe_tflops_tf32"] = round(3 * achieved, 1)
    else:
        achieved = dom.algo_bytes / (dom_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                "unit": "GB/s", "frac_of_spec_8tbs": round(achieved / SPEC_HBM_GBS, 4)}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    roof["peak_source"] = pk["source"]
    roof["kernel"] = dom.key
    roof["traffic"] = traffic
    if flops_step:
        unit = "TFLOP/s"
        value = flops_step / (ms * 1e-3) / 1e12
        e2e_val = flops_step / (e2e_ms * 1e-3) / 1e12
    else:
        unit = "GB/s"
        value = bytes_step / (ms * 1e-3) / 1e9
        e2e_val = bytes_step / (e2e_ms * 1e-3) / 1e9
    launches_per_step = sum(1 + len(j.pk.plan.get("pre", [])) if j.pk.has_pre else 1
                            for j in jobs)
    rec = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "strong" if strong else "weak",
        "vs_baseline": None, "dtype": dtype,
        "data": "synthetic (block-seeded numpy, BASELINE shapes and distributions)",
        "config": dict(cfg, parallelism=(f"{dist.world} ranks" + (
            f", {cfg['collective']}" if cfg.get("collective") else ""))),
        "kernels_ms": {k: round(v, 4) for k, v in live_ms.items()},
        "kernels_ms_alone": {k: round(v, 4) for k, v in per_kernel.items()},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 2), "unit": unit, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clocks,
        "parity": "checked before timing on this shard: " + parity,
    }
    for j in jobs:
        if j.inbox is not None:
            j.pk.detach_peers()       # the module forgets the inbox before it goes
            j.inbox.close()
        for copy in j.rot:
            for p in copy.values():
                dev.free(p)
        if j.rot:
            j.pk.bufs.update(j.base)
        j.pk.close()
    if comm is not None:
        dev.sync(nccl_stream)
        comm.close()
    return rec


# ---------------------------------------------------------------------------
# the CPU oracle (the reference's algorithm) on the host cores
# ---------------------------------------------------------------------------


def _reductions_parts(cores: int):
    """The default configuration cut into ``cores`` parts: element ranges of
    the 2**26 (sum and mean) and row blocks of the 8192 x 8192 (row sum)."""
    N, R = 1 << 26, 8192
    return [(shard(N, cores, w, 256), shard(R, cores, w)) for w in range(cores)]


_WORKER = None


def _worker_init_full(cores: int, w: int) -> None:
    """Build worker ``w``'s part of the full reductions configuration: the
    same block-seeded numbers the GPU arm's one-rank run uses."""
    global _WORKER
    for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[v] = "1"
    from ptxgen import irgen
    (lo, hi), (r0, r1) = _reductions_parts(cores)[w]
    x = gen_rows("u01", 1000, (1 << 26,), lo, hi)
    xr = gen_rows("normal", 1001, (8192, 8192), r0, r1)
    n = hi - lo
    s = _spec(irgen.reduce_full(n), "s")
    m = _spec(irgen.reduce_full(n, mean=True), "m")
    m.args["mean_keepdim_count"].data = [float(1 << 26)]
    r = _spec(irgen.reduce_rows(r1 - r0, 8192), "r")
    _WORKER = [(s, {"x": x}), (m, {"x": x, "mean_keepdim_count": np.array([float(1 << 26)],
                                                                           np.float32)}),
               (r, {"x": xr})]


def _worker_pass(_=None):
    """One pass of the oracle over this worker's part; returns its outputs
    (the sum and mean partials, the row sums) and its time."""
    from oracle.interp import interpret, make_inputs
    t0 = time.perf_counter()
    outs = []
    for spec, ins in _WORKER:
        full = make_inputs(spec)
        full.update(ins)
        o = interpret(spec, full)
        outs.append({k: np.asarray(v) for k, v in o.items()})
    return time.perf_counter() - t0, outs


def _host_cores() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 64))


class FullConfigPool:
    """``cores`` spawned single-threaded workers (no CUDA state inherited),
    worker w holding part w of the full default configuration; ``step()``
    runs one pass on every worker and returns its wall time, after folding
    the parts: sum and mean partials added, row sums concatenated."""

    def __init__(self, cores: int | None = None):
        import multiprocessing as mp
        self.cores = cores or _host_cores()
        ctx = mp.get_context("spawn")
        self.pools = [ctx.Pool(1, initializer=_worker_init_full, initargs=(self.cores, w))
                      for w in range(self.cores)]

    def step(self):
        t0 = time.perf_counter()
        res = [p.apply_async(_worker_pass) for p in self.pools]
        outs = [r.get() for r in res]
        s = float(np.sum([o[1][0]["sum_1"][0] for o in outs], dtype=np.float32))
        m = float(np.sum([o[1][1]["mean"][0] for o in outs], dtype=np.float32))
        rows = np.concatenate([o[1][2]["sum_1"] for o in outs])
        return time.perf_counter() - t0, (s, m, rows)

    def close(self):
        for p in self.pools:
            p.close()
            p.join()


FULL_BYTES = 2 * ((1 << 26) * 4 + 4) + 8192 * 8192 * 4 + 8192 * 4
FULL_DESC = ("the full configs[1] workload (sum+mean over 2^26 f32 U[0,1], row sum of "
             "8192x8192 f32 N(0,1)), the same block-seeded inputs as the GPU arm, interpreted "
             "by the oracle in {c} parts (element ranges / row blocks) on {c} spawned "
             "single-threaded workers, one per host core; parts folded on the host")


def _check_full(res):
    """The CPU arm's folded result against float64 of the same inputs."""
    s, m, rows = res
    x = gen_rows("u01", 1000, (1 << 26,), 0, 1 << 26).astype(np.float64)
    exact = x.sum()
    if abs(s - exact) > 1e-5 * exact or abs(m - exact / (1 << 26)) > 1e-5 * exact / (1 << 26):
        raise AssertionError(f"CPU arm sum/mean {s}, {m} vs {exact}")
    xr = gen_rows("normal", 1001, (8192, 8192), 0, 256).astype(np.float64)
    if np.any(np.abs(rows[:256] - xr.sum(-1)) > 1e-5 * np.abs(xr).sum(-1)):
        raise AssertionError("CPU arm row sums")


def cpu_baseline_full(passes: int = 2):
    pool = FullConfigPool()
    try:
        pool.step()                                   # imports, first touch
        total, res = 0.0, None
        for _ in range(passes):
            dt, res = pool.step()
            total += dt
    finally:
        pool.close()
    _check_full(res)
    value = FULL_BYTES * passes / total / 1e9
    return {"value": round(value, 6), "unit": "GB/s", "cores": pool.cores, "kind": "port",
            "sample": FULL_DESC.format(c=pool.cores) + f"; {passes} passes in {total:.1f} s"}


def _oracle_sample(name: str):
    """(description, [(spec, inputs, work)]) of a bounded sample of a
    sub-record's workload, for its ``cpu_baseline``."""
    from ptxgen import irgen
    rng = np.random.default_rng(7)
    out = []
    if name == "pointwise":
        n = 1 << 22
        a = rng.uniform(-1, 1, n).astype(np.float32)
        b = rng.uniform(-1, 1, n).astype(np.float32)
        out.append((_spec(irgen.pointwise(n, 4, "add"), "a"), {"x0": a, "x1": b}, 12 * n))
        return "c=a+b over 2^22 f32", out
    if name == "rows":
        x = rng.standard_normal((512, 4096), dtype=np.float32)
        g = np.ones(4096, np.float32)
        for gm in (irgen.rmsnorm(512, 4096, eps=1e-6), irgen.softmax(512, 4096),
                   irgen.l2norm(512, 4096)):
            spec = _spec(gm, "r")
            ins = {"x": x}
            if "w" in spec.args:
                ins["w"] = g
            out.append((spec, ins, 8 * x.size))
        return "RMSNorm, softmax, L2-norm on 512x4096 f32", out
    if name.startswith("matmul"):
        m = n = k = 256
        a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
        gm = (irgen.matmul_splitk(m, n, k, slice_k=k // 8) if name.endswith("splitk8")
              else irgen.matmul(m, n, k))
        out.append((_spec(gm, "m"), {"x0": a, "x1": b}, 2.0 * m * n * k))
        return f"the same IR family at 256^3 (work = 2MNK flops)", out
    if name.startswith("attention"):
        b, h, s, d = 1, 2, 64, 64
        q, k, v = (rng.standard_normal((b, h, s, d), dtype=np.float32) for _ in range(3))
        out.append((_spec(irgen.attention_bhsd(b, h, s, d, "f32"), "a"), {"q": q, "k": k, "v": v},
                    4.0 * b * h * s * s * d))
        return "the attention IR at [1,2,64,64] f32 (work = 4BHS^2D flops)", out
    raise ValueError(name)


def _sample_worker_init(name: str) -> None:
    global _WORKER
    for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[v] = "1"
    _WORKER = _oracle_sample(name)[1]


def _sample_worker_pass(_=None) -> float:
    from oracle.interp import interpret, make_inputs
    t0 = time.perf_counter()
    for spec, ins, _w in _WORKER:
        full = make_inputs(spec)
        full.update(ins)
        interpret(spec, full)
    return time.perf_counter() - t0


def cpu_baseline_sample(name: str, budget_s: float = 6.0):
    """The oracle on a bounded sample, one copy per host core."""
    import multiprocessing as mp
    desc, sample = _oracle_sample(name)
    work1 = sum(w for _, _, w in sample)
    cores = _host_cores()
    pool = mp.get_context("spawn").Pool(cores, initializer=_sample_worker_init, initargs=(name,))
    try:
        pool.map(_sample_worker_pass, range(cores), chunksize=1)
        total, reps = 0.0, 0
        while total < budget_s / 2 and reps < 4:
            t0 = time.perf_counter()
            pool.map(_sample_worker_pass, range(cores), chunksize=1)
            total += time.perf_counter() - t0
            reps += 1
    finally:
        pool.close()
        pool.join()
    unit, scale = (("TFLOP/s", 1e12) if name.startswith(("matmul", "attention"))
                   else ("GB/s", 1e9))
    return {"value": round(work1 * cores * reps / total / scale, 6), "unit": unit,
            "cores": cores, "kind": "port",
            "sample": f"{desc}; one copy per worker, {reps} pass(es) in {total:.1f} s on "
                      f"{cores} spawned single-threaded workers"}


def run_reference(args, dist: Dist):
    """The reference's CPU algorithm on the full default configuration,
    rank 0 only (other ranks exit without work)."""
    if dist.rank != 0:
        return None
    if args.workload != "reductions":
        return _run_reference_sample(args, dist)
    pool = FullConfigPool()
    times = []
    try:
        res = None
        for s in range(args.warmup + args.steps):
            dt, res = pool.step()
            if s >= args.warmup:
                times.append(dt)
    finally:
        pool.close()
    _check_full(res)
    ms = 1e3 * sum(times) / len(times)
    value = FULL_BYTES / (ms * 1e-3) / 1e9
    desc = FULL_DESC.format(c=pool.cores)
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": "GB/s",
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (block-seeded numpy)",
        "config": {"workload": "configs[1] reductions: sum+mean over 2^26 f32 U[0,1], row sum "
                               "8192x8192 f32 N(0,1)", "sample": desc, "same_config": True},
        "cpu_baseline": {"value": round(value, 6), "unit": "GB/s", "cores": pool.cores,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 6), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def _run_reference_sample(args, dist: Dist):
    """Another workload's reference arm: the oracle on a bounded sample of
    it, one copy per host core, each step one pass on every core."""
    import multiprocessing as mp
    desc, sample = _oracle_sample(args.workload)
    cores = _host_cores()
    pool = mp.get_context("spawn").Pool(cores, initializer=_sample_worker_init,
                                        initargs=(args.workload,))
    times = []
    try:
        for s in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            pool.map(_sample_worker_pass, range(cores), chunksize=1)
            if s >= args.warmup:
                times.append(time.perf_counter() - t0)
    finally:
        pool.close()
        pool.join()
    unit, scale = (("TFLOP/s", 1e12) if args.workload.startswith(("matmul", "attention"))
                   else ("GB/s", 1e9))
    ms = 1e3 * sum(times) / len(times)
    value = sum(w for _, _, w in sample) * cores / (ms * 1e-3) / scale
    desc = f"{desc}; one copy per worker on {cores} spawned single-threaded workers"
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit,
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy)",
        "config": {"workload": args.workload, "sample": desc, "same_config": False},
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": cores, "kind": "port",
                         "sample": desc},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def run_ours(args, dist: Dist):
    from ptxgen.runtime import Device
    dev = Device.get(dist.local)
    # the printed line: weak scaling of the reductions unless asked otherwise
    # (on one GPU the two coincide); other workloads split one shape
    top_strong = dist.world == 1 or args.workload != "reductions" or args.scaling == "strong"
    line = measure(args.workload, args, dist, strong=top_strong, dev=dev)
    if args.workload == "reductions" and args.scaling == "weak":
        line["scaling"] = "weak"
    if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline:
        line["cpu_baseline"] = (cpu_baseline_full() if args.workload == "reductions"
                                else cpu_baseline_sample(args.workload, args.cpu_budget))
    subs = {}
    for name in _record_names(args):
        if name == args.workload and top_strong:
            continue
        rec = measure(name, args, dist, strong=True, dev=dev)
        if dist.world == 1 and dist.rank == 0 and not args.no_cpu_baseline:
            rec["cpu_baseline"] = cpu_baseline_sample(name, args.cpu_budget)
        subs[name] = rec
    if subs:
        line["workloads"] = subs
    return line


def _record_names(args):
    if args.records == "none":
        return []
    if args.records == "all":
        return list(RECORDS)
    names = []
    for n in args.records.split(","):
        names += ALIASES.get(n, [n])
    bad = [n for n in names if n not in RECORDS]
    if bad:
        raise SystemExit(f"unknown records {bad}; choose from {sorted(RECORDS)}")
    return names


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="reductions",
                    help=f"the printed line's record: one of {sorted(RECORDS)}")
    ap.add_argument("--records", default="all",
                    help="sub-records under 'workloads': all, none, or a comma list")
    ap.add_argument("--scaling", default="weak", choices=["weak", "strong"],
                    help="multi-GPU mode of the printed reductions line (sub-records are "
                         "always strong scaling)")
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=6.0)
    ap.add_argument("--collective", default="p2p", choices=["p2p", "nccl"],
                    help="multi-GPU full reductions: in-kernel exchange over peer inboxes "
                         "(p2p) or an NCCL all-reduce after the kernel")
    ap.add_argument("--jobs", default="",
                    help="comma-separated job keys to keep in each record (default: all)")
    ap.add_argument("--small", action="store_true",
                    help="reduced shapes (attention: B=1) for profiler captures only")
    ap.add_argument("--no-overlap", action="store_true",
                    help="launch every kernel after the previous one completes")
    args = ap.parse_args(argv)
    global _SMALL, OVERLAP
    _SMALL = args.small
    OVERLAP = not args.no_overlap
    if args.workload in ALIASES:
        first, *rest = ALIASES[args.workload]
        args.workload = first
        if args.records == "all":
            args.records = ",".join(rest) if rest else "none"
    if args.workload not in RECORDS:
        raise SystemExit(f"unknown workload {args.workload}")
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist()
    try:
        line = run_reference(args, dist) if args.impl == "reference" else run_ours(args, dist)
        if dist.rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
