#!/usr/bin/env python3
"""Benchmark of the Emmy Kernel IR -> B200 hot path.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--impl ours|reference]

One step = one pass of the compiled IR kernels of a BASELINE configuration
over one batch of synthetic inputs already resident in HBM.  The default
workload is BASELINE configs[1], the reductions: full-array sum and mean over
2**26 f32 ~ U[0,1] and the row sum of an 8192 x 8192 f32 ~ N(0,1) matrix.
Other workloads: ``pointwise`` (c = a + b, 2**28), ``rows`` (RMSNorm,
softmax, L2-norm on 65536 x 4096), ``matmul``, ``attention``.

Multi-GPU (launched by torch.distributed.run): one process per GPU, weak
scaling -- each rank owns a full-size shard; full reductions exchange their
per-rank totals inside the reduction kernel over NVLink peer inboxes
(``--collective p2p``, default) or with an NCCL all-reduce after it
(``--collective nccl``); the mean's divisor is the global count, so the
reduced value is the global mean.  Time is taken on the device with events
on the launching stream, and the reported time is the max over ranks.

``value`` comes from a loop of K steps with events only at its ends;
``kernels_ms`` and the roofline from a second pass that times each job alone
over K back-to-back launches, again with events only at the batch ends.

``--impl reference`` times the reference's own CPU algorithm -- the CPU
oracle restating ``ptxgen/interp.py`` -- on the same configuration, rank 0
only, each step a bounded sample of the workload.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
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
# workloads
# ---------------------------------------------------------------------------


class Job:
    """One compiled kernel of a workload with its inputs and work figures."""

    def __init__(self, key, spec, inputs, algo_bytes, algo_flops=0.0, allreduce=None,
                 check=None, local_ref=None, ref_div=1.0):
        self.local_ref = local_ref    # this rank's f64 share of an all-reduced result
        self.ref_div = ref_div        # global result = sum over ranks of local_ref / ref_div
        self.inbox = None
        self.key = key
        self.spec = spec
        self.inputs = inputs          # host arrays (uploaded per step in e2e)
        self.algo_bytes = algo_bytes  # per launch
        self.algo_flops = algo_flops  # per launch
        self.allreduce = allreduce    # output name reduced across ranks, or None
        self.check = check            # (outputs) -> None, raises on mismatch
        self.pk = None


def _spec(gm, name):
    from ptxgen.loader import load_kernel_data
    return load_kernel_data(gm[0], gm[1], name)


def workload_reductions(rank: int, world: int):
    from ptxgen import irgen
    n = 1 << 26
    rows = cols = 8192
    rng = np.random.default_rng(1000 + rank)
    x = rng.random(n, dtype=np.float32)
    xr = rng.standard_normal((rows, cols), dtype=np.float32)
    total = n * world
    s_spec = _spec(irgen.reduce_full(n, pid="sum_2p26"), "sum")
    m_spec = _spec(irgen.reduce_full(n, mean=True, pid="mean_2p26"), "mean")
    m_spec.args["mean_keepdim_count"].data = [float(total)]
    r_spec = _spec(irgen.reduce_rows(rows, cols, pid="row_sum"), "row_sum")
    local_sum = float(x.astype(np.float64).sum())

    def chk_sum(out, key="sum_1", div=1.0):
        got = float(out[key][0])
        # the all-reduced value is the global figure; compare the local share
        want = local_sum / div
        tol = 1e-5 * abs(want) * (world if world > 1 else 1)
        if world == 1 and abs(got - want) > tol:
            raise AssertionError(f"{key}: {got} vs {want}")

    def chk_rows(out):
        ref = xr[:64].astype(np.float64).sum(-1)
        bound = 1e-5 * np.abs(xr[:64].astype(np.float64)).sum(-1)
        if np.any(np.abs(out["sum_1"][:64] - ref) > bound):
            raise AssertionError("row sums")

    return [
        Job("sum", s_spec, {"x": x}, n * 4 + 4, allreduce="sum_1", check=chk_sum,
            local_ref=local_sum),
        Job("mean", m_spec, {"x": x}, n * 4 + 4, allreduce="mean",
            check=lambda o: chk_sum(o, "mean", float(total)), local_ref=local_sum,
            ref_div=float(total)),
        Job("row_sum", r_spec, {"x": xr}, rows * cols * 4 + rows * 4, check=chk_rows),
    ], {"workload": "configs[1] reductions: sum+mean over 2^26 f32 U[0,1], row sum 8192x8192 "
                    "f32 N(0,1)", "elements_per_rank": 2 * n + rows * cols}


def workload_pointwise(rank: int, world: int):
    from ptxgen import irgen
    n = 1 << 28
    rng = np.random.default_rng(2000 + rank)
    a = rng.uniform(-1, 1, n).astype(np.float32)
    b = rng.uniform(-1, 1, n).astype(np.float32)
    spec = _spec(irgen.pointwise(n, 4, "add", pid="vector_add_2p28"), "add")

    def chk(out):
        if not np.array_equal(out["add"][: 1 << 20], a[: 1 << 20] + b[: 1 << 20]):
            raise AssertionError("vector add not bit-exact")

    return [Job("vector_add", spec, {"x0": a, "x1": b}, 12 * n, check=chk)], {
        "workload": "configs[0] scaled: c=a+b over 2^28 f32 U[-1,1]", "elements_per_rank": n}


def workload_rows(rank: int, world: int):
    from ptxgen import irgen
    r, c = 65536, 4096
    rng = np.random.default_rng(3000 + rank)
    x = rng.standard_normal((r, c), dtype=np.float32)
    g = (1.0 + 0.1 * rng.standard_normal(c)).astype(np.float32)
    jobs = []
    for key, gm in (("rmsnorm", irgen.rmsnorm(r, c, eps=1e-6)), ("softmax", irgen.softmax(r, c)),
                    ("l2norm", irgen.l2norm(r, c))):
        spec = _spec(gm, key)
        ins = {"x": x}
        if key == "rmsnorm":
            ins["w"] = g
        jobs.append(Job(key, spec, ins, 8 * r * c + (4 * c if key == "rmsnorm" else 0)))
    return jobs, {"workload": "configs[2] fused rows: RMSNorm, softmax, L2-norm on 65536x4096 f32",
                  "elements_per_rank": 3 * r * c}


def workload_matmul(rank: int, world: int):
    from ptxgen import irgen
    rng = np.random.default_rng(4000 + rank)
    jobs = []
    for key, (m, n, k), gm in (
            ("matmul_square", (8192, 8192, 8192), irgen.matmul(8192, 8192, 8192)),
            ("matmul_rect", (16384, 4096, 1024), irgen.matmul(16384, 4096, 1024)),
            ("matmul_splitk8", (16384, 4096, 1024),
             irgen.matmul_splitk(16384, 4096, 1024, slice_k=128))):
        spec = _spec(gm, key)
        a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)

        def chk(out, a=a, b=b):
            rows = np.arange(0, a.shape[0], a.shape[0] // 16)
            ref = a[rows].astype(np.float64) @ b.astype(np.float64)
            scale = np.abs(a[rows].astype(np.float64)) @ np.abs(b.astype(np.float64))
            if np.any(np.abs(out["matmul"][rows] - ref) > 1e-4 * scale):
                raise AssertionError("matmul outside the 1e-4 bound")

        jobs.append(Job(key, spec, {"x0": a, "x1": b}, 4 * (m * k + k * n + m * n),
                        algo_flops=2.0 * m * n * k, check=chk))
    return jobs, {"workload": "configs[3] f32 matmul (3xTF32 on tcgen05): 8192^3, "
                              "16384x4096x1024, and its split-K=8 atomic variant",
                  "rows_per_rank": "M rows sharded, B replicated"}


def workload_attention(rank: int, world: int):
    from ptxgen import irgen
    from ml_dtypes import bfloat16
    b, h, s, d = (1 if _SMALL else 16), 32, 4096, 128
    rng = np.random.default_rng(5000 + rank)
    jobs = []
    for dt in ("f32", "bf16"):
        spec = _spec(irgen.attention_bhsd(b, h, s, d, dt, pid=f"attn_{dt}"), f"attn_{dt}")
        npdt = np.float32 if dt == "f32" else bfloat16
        q, k, v = (rng.standard_normal((b, h, s, d), dtype=np.float32).astype(npdt)
                   for _ in range(3))

        def chk(out, q=q, k=k, v=v, dt=dt):
            bi, hi = 3 % b, 17
            rows = np.arange(0, s, 257)
            qq, kk, vv = (x[bi, hi].astype(np.float64) for x in (q, k, v))
            sc = qq[rows] @ kk.T / np.sqrt(d)
            sc -= sc.max(-1, keepdims=True)
            pp = np.exp(sc)
            ref = (pp / pp.sum(-1, keepdims=True)) @ vv
            got = out["out"][bi, hi, rows].astype(np.float64)
            tol = 1e-4 if dt == "f32" else 2e-2
            if np.abs(got - ref).max() > tol * np.abs(ref).max():
                raise AssertionError(f"attention {dt} outside tolerance")

        e = 4 if dt == "f32" else 2
        jobs.append(Job(f"attention_{dt}", spec, {"q": q, "k": k, "v": v}, 4 * b * h * s * d * e,
                        algo_flops=4.0 * b * h * s * s * d, check=chk))
    return jobs, {"workload": "configs[4] attention softmax(QK^T/sqrt(d))V, [16,32,4096,128] "
                              "f32 (3xTF32) and bf16, non-causal",
                  "heads_per_rank": b * h}


_SMALL = False

WORKLOADS = {"reductions": workload_reductions, "pointwise": workload_pointwise,
             "rows": workload_rows, "matmul": workload_matmul, "attention": workload_attention}


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
    """Samples SM clock, power and throttle reasons while the timed region
    runs: NVML polled every millisecond from a thread (read-only queries);
    nvidia-smi as a fallback."""

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
                mhz = N.nvmlDeviceGetClockInfo(h, N.NVML_CLOCK_SM)
                reasons = get_reasons(h)
                self.samples.append((mhz, reasons, 0))
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
        mhz = [m for m, _, _ in window]
        reasons = sorted({n for _, r, _ in window for n, bit in self.REASONS.items()
                          if r & bit})
        return {"sm_mhz": statistics.median(mhz), "sm_max_mhz": self.smax, "reasons": reasons,
                "samples": len(mhz), "source": "nvml"}


# ---------------------------------------------------------------------------
# distributed plumbing
# ---------------------------------------------------------------------------


class Dist:
    """This process's place in the job (torch.distributed.run env) and the
    host-side rendezvous; see ``ptxgen.dist``."""

    def __init__(self, gpus: int):
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
# our implementation
# ---------------------------------------------------------------------------


def run_ours(args, dist: Dist):
    import ctypes as C
    from ptxgen.runtime import Device, PreparedKernel, check
    jobs, cfg = WORKLOADS[args.workload](dist.rank, dist.world)
    if args.jobs:
        keep = set(args.jobs.split(","))
        jobs = [j for j in jobs if j.key in keep]
        if not jobs:
            raise SystemExit(f"--jobs {args.jobs}: no such job in {args.workload}")
        cfg["jobs"] = sorted(keep)
    if _SMALL:
        cfg["small"] = "reduced shapes for profiler captures; not a bench configuration"
    dev = Device.get(dist.local)
    comm = None
    for j in jobs:
        j.pk = PreparedKernel(j.spec, dev=dev)
        j.pk.upload(j.inputs)
    dev.sync()
    if dist.world > 1 and args.collective == "p2p":
        # full reductions exchange their totals inside the kernel, over
        # peer inboxes (NVLink stores): no separate collective launch
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
    # With the in-kernel exchange each job runs on its own stream (forked from
    # and joined back to the main stream every step): a reduction's last CTA
    # waiting for the other GPUs then overlaps the step's other kernels.  Only
    # that CTA waits, and only on other GPUs, so concurrent kernels cannot
    # starve one another.  (On one GPU the jobs stay on one stream: measured
    # faster there.)
    concurrent = any(j.inbox is not None for j in jobs)
    if concurrent:
        ev_fork = dev.event()
        for j in jobs:
            j.stream, j.ev_join = dev.new_stream(), dev.event()
        cfg["streams"] = "one stream per job, forked and joined every step"

    def step():
        if concurrent:
            dev.record(ev_fork)
            for j in jobs:
                dev.wait_event(j.stream, ev_fork)
                if j.pk.has_pre:
                    j.pk.launch_pre(j.stream)
                j.pk.launch_main(j.stream)
                dev.record(j.ev_join, j.stream)
            for j in jobs:
                dev.wait_event(dev.stream, j.ev_join)
            return
        pending = []
        for i, j in enumerate(jobs):
            if j.pk.has_pre:
                j.pk.launch_pre()
            j.pk.launch_main()
            if comm is not None and j.allreduce:
                pending.append(j)
            if pending and i == last_ar:
                # all-reduce the per-rank results on a second stream, overlapped
                # with the kernels still to run on the main stream
                dev.record(ev_ready)
                dev.wait_event(nccl_stream, ev_ready)
                for pj in pending:
                    a = pj.spec.args[pj.allreduce]
                    comm.allreduce_sum_f32(pj.pk.bufs[pj.allreduce], a.numel, nccl_stream)
                dev.record(ev_done, nccl_stream)
        if pending:
            dev.wait_event(dev.stream, ev_done)

    for _ in range(args.warmup):
        step()
    dev.sync()
    # untimed ramp: keep the GPU busy ~0.3 s so it leaves idle clocks; the
    # number of steps is agreed across ranks (each step of a multi-rank full
    # reduction meets every other rank's)
    t_ramp = time.perf_counter()
    for _ in range(16):
        step()
    dev.sync()
    per16 = dist.max(time.perf_counter() - t_ramp)
    for _ in range(max(1, int(0.3 / max(per16, 1e-4)))):
        for _ in range(16):
            step()
        dev.sync()
    for j in jobs:
        j.pk.check_errors()
        if j.check is not None and dist.world == 1:
            j.check(j.pk.download())
        elif j.local_ref is not None and dist.world > 1:
            name = j.spec.outputs[0]
            got = float(j.pk.download([name])[name].reshape(-1)[0])
            want = dist.rdv.sum(j.local_ref) / j.ref_div
            if abs(got - want) > 1e-5 * abs(want):
                raise AssertionError(f"{j.key} over {dist.world} ranks: {got} vs {want}")
    # ---- timed region: device-resident inputs, events only at its ends ----
    t0, t1 = dev.event(), dev.event()
    dist.barrier()
    dev.sync()
    with ClockSampler(dist.local) as clk:
        for _ in range(8):  # re-warm after the idle gap of the set-up above
            step()
        clk.mark()
        dev.record(t0)
        for s in range(args.steps):
            step()
        dev.record(t1)
        dev.sync()
    dist.barrier()
    total_ms = dev.elapsed_ms(t0, t1)
    # ---- per-kernel durations: each job alone, ``steps`` back-to-back
    # launches between two events on the launching stream (an event at every
    # launch would add microseconds that a 45 us kernel carries; every input
    # is larger than L2, so a repeated launch re-reads HBM).  Every rank
    # issues the same batches in the same order. ----
    per_kernel = {}
    dev.sync()
    for j in jobs:
        batches = ([(j.key + ".pre", j.pk.launch_pre)] if j.pk.has_pre else [])
        batches.append((j.key, j.pk.launch_main))
        for key, launch in batches:
            a, b = dev.event(), dev.event()
            dev.record(a)
            for _ in range(args.steps):
                launch()
            dev.record(b)
            dev.sync()
            per_kernel[key] = [dev.elapsed_ms(a, b) / args.steps]
    for j in jobs:
        j.pk.check_errors()
    ms = dist.max(total_ms) / args.steps
    # ---- e2e: host buffers through the public launch API ----
    pinned = {}
    h2d = 0
    for j in jobs:
        for name, arr in j.inputs.items():
            key = (id(arr), name)
            if key in pinned:
                continue
            p = dev.host_alloc(arr.nbytes)
            view = np.ctypeslib.as_array((C.c_char * arr.nbytes).from_address(p))
            view[:] = np.frombuffer(np.ascontiguousarray(arr).tobytes(), dtype=np.uint8).view("S1")
            pinned[key] = (p, arr.nbytes)
    from ptxgen.runtime import _np_dtype
    out_host = {j.key: {o: np.empty(j.spec.args[o].shape, _np_dtype(j.spec.args[o].dtype))
                        for o in j.spec.outputs} for j in jobs}

    def e2e_step():
        nb_in, nb_out = 0, 0
        done = set()
        for j in jobs:
            for name, arr in j.inputs.items():
                p, nb = pinned[(id(arr), name)]
                if (id(arr), j.key, name) in done:
                    continue
                check(dev.L.emmy_memcpy_htod(C.c_uint64(j.pk.bufs[name]), C.c_void_p(p), nb,
                                             dev.stream), "htod")
                nb_in += nb
        step()
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
    dev.record(e0)
    esteps = max(1, min(args.steps, 5))
    for _ in range(esteps):
        h2d, d2h = e2e_step()
    dev.record(e1)
    dev.sync()
    dist.barrier()
    e2e_ms = dist.max(dev.elapsed_ms(e0, e1)) / esteps
    for p, _ in pinned.values():
        dev.host_free(p)

    bytes_step = sum(j.algo_bytes for j in jobs)
    flops_step = sum(j.algo_flops for j in jobs)
    pk = peaks()
    # dominant kernel and its roofline
    avg = {k: sum(v) / len(v) for k, v in per_kernel.items()}
    dom = max(jobs, key=lambda j: sum(per_kernel[j.key]))
    dom_ms = avg[dom.key]
    launches_per_step = sum(1 + len(j.pk.plan.get("pre", [])) if j.pk.has_pre else 1
                            for j in jobs)
    traffic = None
    tpath = ROOT / "profiles" / "traffic.json"
    if tpath.exists():
        traffic = json.loads(tpath.read_text()).get(f"{args.workload}:{dom.key}")
    if dom.algo_flops:
        achieved = dom.algo_flops / (dom_ms * 1e-3) / 1e12
        if dom.spec.args[dom.spec.outputs[0]].dtype == "bf16":
            roof = {"bound": "tensor", "achieved": round(achieved, 2),
                    "peak": pk["bf16_tflops"], "unit": "TFLOP/s",
                    "peak_note": "measured dense bf16 (cuBLAS burst)"}
        else:
            # 3xTF32: three TF32 products per useful f32 product; TF32 runs at
            # half the dense bf16 rate, so the useful-flop ceiling is bf16 / 6
            peak3 = pk["bf16_tflops"] / 6.0
            roof = {"bound": "tensor", "achieved": round(achieved, 2), "peak": round(peak3, 1),
                    "unit": "TFLOP/s",
                    "peak_note": f"3xTF32 useful-flop ceiling = measured dense bf16 "
                                 f"{pk['bf16_tflops']} / 2 (tf32) / 3 (passes)",
                    "tensor_pipe_tflops_tf32": round(3 * achieved, 1)}
    else:
        achieved = dom.algo_bytes / (dom_ms * 1e-3) / 1e9
        roof = {"bound": "hbm", "achieved": round(achieved, 1), "peak": pk["hbm_gbs"],
                "unit": "GB/s"}
    roof["frac"] = round(roof["achieved"] / roof["peak"], 4)
    roof["peak_source"] = pk["source"]
    roof["kernel"] = dom.key
    roof["traffic"] = traffic
    roof["frac_of_spec_8tbs"] = round(achieved / SPEC_HBM_GBS, 4) if not dom.algo_flops else None
    if flops_step:
        value = flops_step * dist.world / (ms * 1e-3) / 1e12
        unit = "TFLOP/s"
        e2e_val = flops_step * dist.world / (e2e_ms * 1e-3) / 1e12
    else:
        value = bytes_step * dist.world / (ms * 1e-3) / 1e9
        unit = "GB/s"
        e2e_val = bytes_step * dist.world / (e2e_ms * 1e-3) / 1e9
    line = {
        "metric": METRIC, "value": round(value, 2), "unit": unit, "n_gpus": dist.world,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms, 4),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic (seeded numpy, BASELINE shapes and distributions)",
        "config": dict(cfg, l2="every input is larger than the 126 MB L2",
                       parallelism=(f"shards x{dist.world}" + (
                           f", full reductions: {cfg['collective']}" if cfg.get("collective")
                           else ""))),
        "kernels_ms": {k: round(v, 4) for k, v in avg.items()},
        "roofline": roof,
        "e2e": {"value": round(e2e_val, 2), "unit": unit, "h2d_bytes_per_step": int(h2d),
                "d2h_bytes_per_step": int(d2h)},
        "gpu_launches": launches_per_step * args.steps,
        "clocks": clk.summary(),
    }
    if dist.rank == 0 and dist.world == 1 and not args.no_cpu_baseline:
        line["cpu_baseline"] = cpu_baseline(args.workload, args.cpu_budget)
    for j in jobs:
        if j.inbox is not None:
            j.inbox.close()
        j.pk.close()
    if comm is not None:
        dev.sync(nccl_stream)
        comm.close()
    return line


# ---------------------------------------------------------------------------
# the CPU oracle (reference algorithm) on a bounded sample
# ---------------------------------------------------------------------------


def _oracle_sample(workload: str):
    """(description, [(spec, inputs, algo_bytes)]) of a bounded sample."""
    from ptxgen import irgen
    rng = np.random.default_rng(7)
    out = []
    if workload == "reductions":
        n = 1 << 20
        x = rng.random(n, dtype=np.float32)
        for gm in (irgen.reduce_full(n), irgen.reduce_full(n, mean=True)):
            spec = _spec(gm, "s")
            ins = {"x": x}
            if "mean_keepdim_count" in spec.args:
                ins["mean_keepdim_count"] = np.array([float(n)], np.float32)
            out.append((spec, ins, n * 4))
        xr = rng.standard_normal((256, 8192), dtype=np.float32)
        out.append((_spec(irgen.reduce_rows(256, 8192), "r"), {"x": xr}, xr.nbytes))
        return "sum+mean over 2^20 f32 and row sum of 256x8192 (same IR, interp algorithm)", out
    if workload == "pointwise":
        n = 1 << 22
        a = rng.uniform(-1, 1, n).astype(np.float32)
        b = rng.uniform(-1, 1, n).astype(np.float32)
        out.append((_spec(irgen.pointwise(n, 4, "add"), "a"), {"x0": a, "x1": b}, 12 * n))
        return "c=a+b over 2^22 f32", out
    if workload == "rows":
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
    if workload == "matmul":
        m = n = k = 256
        a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
        b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
        out.append((_spec(irgen.matmul(m, n, k), "m"), {"x0": a, "x1": b}, 2.0 * m * n * k))
        return "m01-schedule IR matmul 256^3 (work = 2MNK flops)", out
    if workload == "attention":
        b, h, s, d = 1, 2, 64, 64
        q, k, v = (rng.standard_normal((b, h, s, d), dtype=np.float32) for _ in range(3))
        out.append((_spec(irgen.attention_bhsd(b, h, s, d, "f32"), "a"), {"q": q, "k": k, "v": v},
                    4.0 * b * h * s * s * d))
        return "a02-schedule IR attention [1,2,64,64] f32 (work = 4BHS^2D flops)", out
    raise ValueError(workload)


def _sample_unit(workload: str):
    return ("TFLOP/s", 1e12) if workload in ("matmul", "attention") else ("GB/s", 1e9)


# ---- the oracle on every host core: one spawned worker per core, each
# interpreting its own copy of the bounded sample once per step -------------

_WORKER_SAMPLE = None


def _oracle_worker_init(workload: str) -> None:
    global _WORKER_SAMPLE
    for v in ("OMP_NUM_THREADS", "OPENBLAS_NUM_THREADS", "MKL_NUM_THREADS"):
        os.environ[v] = "1"
    _WORKER_SAMPLE = _oracle_sample(workload)[1]


def _oracle_worker_pass(_=None) -> float:
    from oracle.interp import interpret, make_inputs
    t0 = time.perf_counter()
    for spec, ins, _nb in _WORKER_SAMPLE:
        full = make_inputs(spec)
        full.update(ins)
        interpret(spec, full)
    return time.perf_counter() - t0


def _host_cores() -> int:
    try:
        n = len(os.sched_getaffinity(0))
    except AttributeError:
        n = os.cpu_count() or 1
    return max(1, min(n, 64))


class OraclePool:
    """``cores`` spawned processes (no CUDA state is inherited), each with
    the workload's sample built once; ``step()`` runs one pass on every
    worker and returns the wall time of the slowest."""

    def __init__(self, workload: str, cores: int | None = None):
        import multiprocessing as mp
        self.cores = cores or _host_cores()
        self.pool = mp.get_context("spawn").Pool(self.cores, initializer=_oracle_worker_init,
                                                 initargs=(workload,))

    def step(self) -> float:
        t0 = time.perf_counter()
        self.pool.map(_oracle_worker_pass, range(self.cores), chunksize=1)
        return time.perf_counter() - t0

    def close(self) -> None:
        self.pool.close()
        self.pool.join()


def cpu_baseline(workload: str, budget_s: float = 20.0):
    desc, sample = _oracle_sample(workload)
    nb1 = sum(nb for _, _, nb in sample)
    pool = OraclePool(workload)
    try:
        pool.step()                                    # imports, first-touch
        total, reps = 0.0, 0
        while True:
            total += pool.step()
            reps += 1
            if total > budget_s / 4 or reps >= 4:
                break
    finally:
        pool.close()
    unit, scale = _sample_unit(workload)
    value = nb1 * pool.cores * reps / total / scale
    return {"value": round(value, 6), "unit": unit, "cores": pool.cores, "kind": "port",
            "sample": f"{desc}; one copy per worker, {reps} pass(es) in {total:.1f} s, "
                      f"numpy oracle on {pool.cores} spawned single-threaded workers"}


def run_reference(args, dist: Dist):
    if dist.rank != 0:
        return None
    desc, sample = _oracle_sample(args.workload)
    pool = OraclePool(args.workload)
    times = []
    try:
        for s in range(args.warmup + args.steps):
            dt = pool.step()
            if s >= args.warmup:
                times.append(dt)
    finally:
        pool.close()
    nbytes = sum(nb for _, _, nb in sample) * pool.cores
    desc = f"{desc}; one copy per worker on {pool.cores} spawned single-threaded workers"
    ms = 1e3 * sum(times) / len(times)
    unit, scale = _sample_unit(args.workload)
    value = nbytes / (ms * 1e-3) / scale
    return {
        "impl": "reference", "metric": METRIC, "value": round(value, 6), "unit": unit,
        "n_gpus": dist.world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(ms, 3), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic (seeded numpy)",
        "config": {"workload": args.workload, "sample": desc},
        "cpu_baseline": {"value": round(value, 6), "unit": unit, "cores": pool.cores,
                         "kind": "port", "sample": desc},
        "e2e": {"value": round(value, 6), "unit": unit, "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
    }


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--workload", default="reductions", choices=sorted(WORKLOADS))
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-budget", type=float, default=20.0)
    ap.add_argument("--collective", default="p2p", choices=["p2p", "nccl"],
                    help="multi-GPU full reductions: in-kernel exchange over peer inboxes "
                         "(p2p) or an NCCL all-reduce after the kernel")
    ap.add_argument("--jobs", default="",
                    help="comma-separated job keys of the workload to run (default: all)")
    ap.add_argument("--small", action="store_true",
                    help="reduced shapes (attention: B=1) for profiler captures only")
    args = ap.parse_args(argv)
    global _SMALL
    _SMALL = args.small
    if args.warmup < 3:
        args.warmup = 3
    dist = Dist(args.gpus)
    try:
        if args.impl == "reference":
            line = run_reference(args, dist)
        else:
            line = run_ours(args, dist)
        if dist.rank == 0 and line is not None:
            print(json.dumps(line), flush=True)
    finally:
        dist.close()
    return 0


if __name__ == "__main__":
    raise SystemExit(main())
