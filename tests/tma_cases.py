"""Shared cases of the bulk-async transport nodes (``TmaDescriptor``,
``TmaLoad``, ``Mbarrier*``, ``SetMaxNReg``) for the CPU and GPU tests, and a
numpy statement of what a box copy produces."""

import numpy as np

from ptxgen import irgen
from ptxgen.ir import Cond, MbarrierInit, MbarrierWait, Smem, Sync
from ptxgen.loader import load_kernel_data

# (dtype, swizzle, rows, cols, br, bc, nbr, nbc, off_r, off_c)
BOX_CASES = [
    ("f32", "NONE", 40, 40, 16, 8, 3, 6, -5, -4),      # zero fill on every side
    ("f32", "NONE", 64, 96, 32, 32, 2, 3, 0, 0),       # exact tiling
    ("f32", "B32", 33, 24, 8, 8, 5, 3, 1, 0),
    ("f32", "B64", 50, 64, 16, 16, 4, 5, -3, -16),
    ("f32", "B128", 70, 96, 24, 32, 3, 4, 2, 8),
    ("bf16", "B128", 40, 128, 16, 64, 3, 3, -5, -32),
    ("f16", "B64", 48, 80, 16, 32, 3, 3, 4, 8),
    ("f64", "NONE", 20, 20, 8, 6, 3, 4, 0, -2),
    ("f64", "B128", 24, 32, 8, 16, 3, 2, -1, 2),
]


def box_case(c, view3=False, maxnreg=None, threads=64, name="tma_box"):
    dt, swz, rows, cols, br, bc, nbr, nbc, offr, offc = c
    gm = irgen.tma_box_copy(rows, cols, br, bc, nbr, nbc, dt, swz, offr, offc, threads,
                            maxnreg=maxnreg, view3=view3, pid=name)
    return load_kernel_data(gm[0], gm[1], name)


def box_inputs(spec, seed=0):
    from oracle.interp import storage_dtype
    rng = np.random.default_rng(seed)
    a = spec.args["x0"]
    return {"x0": rng.standard_normal(a.shape).astype(storage_dtype(a.dtype))}


def box_reference(c, x):
    dt, swz, rows, cols, br, bc, nbr, nbc, offr, offc = c
    out = np.zeros((nbr * br, nbc * bc), dtype=x.dtype)
    for i in range(nbr):
        for j in range(nbc):
            r0, c0 = i * br + offr, j * bc + offc
            rs, cs = max(r0, 0), max(c0, 0)
            re, ce = min(r0 + br, rows), min(c0 + bc, cols)
            if re > rs and ce > cs:
                out[i * br + rs - r0:i * br + re - r0, j * bc + cs - c0:j * bc + ce - c0] = \
                    x[rs:re, cs:ce]
    return out


def unarrived_wait(n=64):
    """out = x, after a wait on phase 0 of an mbarrier nothing arrives on:
    the CUDA kernel's bounded wait gives up and reports it."""
    t = irgen.V("t")
    body = [Smem(name="bar", extents=(1,), dtype="unsigned long long", align=8),
            Cond(cond=irgen.EQ(t, irgen.L(0)),
                 body=(MbarrierInit(mbar="bar", count=irgen.L(1), slot=irgen.L(0)),),
                 else_body=()),
            Sync(barrier_id=0, count=None, warp=False),
            MbarrierWait(mbar="bar", phase=irgen.L(0), slot=irgen.L(0)),
            irgen.load("v", "x0", (t,)),
            irgen.write("out", (t,), "v")]
    tl = irgen.tile([irgen.ax("t", n)], body, block_threads=n)
    gm = irgen.package("k_unarrived", "copy", [tl], [("x0", (n,), "f32", 0)], [],
                       ("out", (n,), "f32"), ["x0", "out"], (1, 1, 1), (n, 1, 1),
                       pid="unarrived")
    return load_kernel_data(gm[0], gm[1], "unarrived")


def random_box_cases(n, seed=0):
    """Seeded box copies over the descriptor rules: dtype, swizzle (its box
    row fixed by the span), view and box sizes, and box origins that run
    off every edge of the view (zero fill), some through a rank-3 view."""
    rng = np.random.default_rng(seed)
    eb = {"f32": 4, "bf16": 2, "f16": 2, "f64": 8}
    out = []
    while len(out) < n:
        dt = str(rng.choice(["f32", "bf16", "f16", "f64"]))
        swz = str(rng.choice(["NONE", "NONE", "B32", "B64", "B128"]))
        q = 16 // eb[dt]                                   # elements per 16 bytes
        if swz == "NONE":
            bc = q * int(rng.integers(1, 9))
        else:
            bc = {"B32": 32, "B64": 64, "B128": 128}[swz] // eb[dt]
        cols = q * int(rng.integers(1, 12))
        rows = int(rng.integers(2, 70))
        br = int(rng.integers(1, 33))
        nbr, nbc = int(rng.integers(1, 4)), int(rng.integers(1, 4))
        off_r = int(rng.integers(-br, rows))
        off_c = q * int(rng.integers(-(bc // q) - 1, cols // q + 1))
        view3 = bool(rng.integers(0, 2)) and rows % 2 == 0 and br % 2 == 0 and off_r % 2 == 0
        out.append(((dt, swz, rows, cols, br, bc, nbr, nbc, off_r, off_c), view3))
    return out
