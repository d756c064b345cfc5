"""Parity bounds for the f32 contractions (matmul, split-K, f32 attention),
tight enough to tell the 3xTF32 kernels from a one-pass TF32 kernel.

A TF32 operand keeps 10 of f32's 23 fraction bits, so one TF32 pass errs by
about 2^-11 per product; 3xTF32 (hi.hi + hi.lo + lo.hi) by about 2^-20 per
product.  On B200 the tensor core's f32 accumulation adds its own error,
which grows with K: measured per-16-row-block max|err| / max|ref| of the
3xTF32 kernel is 3.4e-6 at K = 256, 1.0e-5 at K = 1024 and 6.9e-5 at
K = 8192 (elementwise err / sum|a||b|: 1.1e-6 to 5.0e-6), against 7e-7 for
an ideal 3xTF32 sum with f32 rounding -- what an accumulator that
truncates each MMA's sum instead of rounding it gives.  ``north_star``
asks for <= 1e-4 relative on f32 contractions; the old condition-aware
bound ``|err| <= 1e-4 * sum_k |a_ik||b_kj|`` is also met by one TF32 pass
once K is large (random-sign errors grow like sqrt(K), the scale like K).
The bounds here:

* elementwise ``|err| <= 2^-15 * sum_k |a_ik||b_kj|``;
* per block of 16 rows ``max |err| <= 1e-4 * max |ref|``;
* attention: per query row ``max_d |err| <= 1e-4 * max_d |ref|``.

``tests/test_contraction_bounds.py`` shows on the CPU that they reject an
emulated one-pass TF32 product at the test shapes and accept an emulated
3xTF32 one; the GPU tests apply them to the kernels.
"""

from __future__ import annotations

import numpy as np

ELEM = 2.0 ** -15
BLOCK = 1e-4
BLOCK_ROWS = 16
ATTN_ROW = 1e-4


def matmul_check(got, a, b, rows=None):
    """(ok, worst elementwise err/scale, worst per-block err/max|ref|) of
    ``got`` against ``a @ b`` in float64 (``rows``: sampled rows of A)."""
    a64, b64 = np.asarray(a, np.float64), np.asarray(b, np.float64)
    got = np.asarray(got, np.float64)
    if rows is not None:
        a64, got = a64[rows], got[rows]
    ref = a64 @ b64
    scale = np.abs(a64) @ np.abs(b64)
    return contraction_check(got, ref, scale)


def contraction_check(got, ref, scale):
    err = np.abs(np.asarray(got, np.float64) - ref)
    elem = float(np.max(err / (scale + 1e-300)))
    block = 0.0
    for i in range(0, ref.shape[0], BLOCK_ROWS):
        block = max(block, float(err[i:i + BLOCK_ROWS].max()
                                 / max(np.abs(ref[i:i + BLOCK_ROWS]).max(), 1e-300)))
    ok = bool(np.all(err <= ELEM * scale + 1e-30)) and block <= BLOCK
    return ok, elem, block


def attention_check(got, ref):
    """(ok, worst per-row max|err| / max|ref|) over the rows of ``got``."""
    got, ref = np.asarray(got, np.float64), np.asarray(ref, np.float64)
    err = np.abs(got - ref).reshape(-1, ref.shape[-1]).max(-1)
    mx = np.abs(ref).reshape(-1, ref.shape[-1]).max(-1)
    worst = float(np.max(err / np.maximum(mx, 1e-300)))
    return worst <= ATTN_ROW, worst


# ---- emulated tensor-core products (CPU, for showing the bounds bite) ----

def tf32(x):
    """x with the 13 low fraction bits cleared (the TF32 ``hi`` part)."""
    x = np.ascontiguousarray(x, np.float32)
    return (x.view(np.uint32) & np.uint32(0xFFFFE000)).view(np.float32)


def split(x):
    x = np.asarray(x, np.float32)
    hi = tf32(x)
    return hi.astype(np.float64), tf32((x - hi).astype(np.float32)).astype(np.float64)


def matmul_1xtf32(a, b):
    """One TF32 pass: operands truncated to TF32, exact products and sums."""
    return tf32(a).astype(np.float64) @ tf32(b).astype(np.float64)


def matmul_3xtf32(a, b):
    ah, al = split(a)
    bh, bl = split(b)
    return ah @ bh + ah @ bl + al @ bh


def attention_emulated(q, k, v, passes: int):
    """softmax(q k^T / sqrt(d)) v with both products in one or three TF32
    passes and P rounded to f32."""
    mm = matmul_1xtf32 if passes == 1 else matmul_3xtf32
    s = mm(q, np.ascontiguousarray(np.asarray(k).T)) / np.sqrt(q.shape[-1])
    s -= s.max(-1, keepdims=True)
    p = np.exp(s).astype(np.float32)
    return mm(p, v) / p.astype(np.float64).sum(-1, keepdims=True)


def attention_ref(q, k, v):
    q, k, v = (np.asarray(x, np.float64) for x in (q, k, v))
    s = q @ np.swapaxes(k, -1, -2) / np.sqrt(q.shape[-1])
    s -= s.max(-1, keepdims=True)
    p = np.exp(s)
    p /= p.sum(-1, keepdims=True)
    return p @ v
