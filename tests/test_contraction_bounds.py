"""The contraction bounds of ``tests/contraction.py`` on the CPU: at every
matmul and f32-attention shape the GPU tests use (K up to 8192), they
reject an emulated one-pass TF32 product -- the mistake a kernel that
dropped the two cross-term MMAs would make -- and accept an emulated
3xTF32 one.  The old bound (1e-4 x sum |a||b|) is shown to accept the
one-pass product at K = 8192, which is why it is no longer the only one."""

import numpy as np
import pytest

from tests import contraction as C

# (m, n, k): the GPU tests' shapes, N cut to 512 columns where it is larger
# (the bound is per element and per row block; K is what matters)
SHAPES = [(256, 512, 256), (384, 192, 512), (128, 64, 1024), (64, 512, 8192),
          (64, 512, 1024), (512, 512, 512)]


@pytest.mark.parametrize("m,n,k", SHAPES)
def test_matmul_bound_rejects_one_tf32_pass(m, n, k):
    rng = np.random.default_rng(m + n + k)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    ok1, e1, b1 = C.matmul_check(C.matmul_1xtf32(a, b), a, b)
    ok3, e3, b3 = C.matmul_check(C.matmul_3xtf32(a, b), a, b)
    assert not ok1, (e1, b1)
    assert ok3, (e3, b3)
    # margins: one pass misses the block bound by >= 5x; an ideal 3xTF32
    # sum meets it by >= 50x (leaving room for the tensor core's own
    # accumulation error, measured up to 6.9e-5 at K = 8192)
    assert b1 >= 5 * C.BLOCK and b3 <= C.BLOCK / 50


def test_old_bound_accepts_one_tf32_pass_at_k8192():
    m, n, k = 64, 512, 8192
    rng = np.random.default_rng(0)
    a = (rng.uniform(-1, 1, (m, k)) / np.sqrt(k)).astype(np.float32)
    b = (rng.uniform(-1, 1, (k, n)) / np.sqrt(k)).astype(np.float32)
    ref = a.astype(np.float64) @ b.astype(np.float64)
    scale = np.abs(a.astype(np.float64)) @ np.abs(b.astype(np.float64))
    err = np.abs(C.matmul_1xtf32(a, b) - ref)
    assert np.all(err <= 1e-4 * scale)


def test_splitk_normal_inputs():
    """test_gpu_mma's split-K case draws N(0,1) operands."""
    rng = np.random.default_rng(9)
    a = rng.standard_normal((64, 1024)).astype(np.float32)
    b = rng.standard_normal((1024, 256)).astype(np.float32)
    assert not C.matmul_check(C.matmul_1xtf32(a, b), a, b)[0]
    assert C.matmul_check(C.matmul_3xtf32(a, b), a, b)[0]


@pytest.mark.parametrize("s,d", [(256, 64), (384, 128), (256, 32), (1024, 128), (4096, 128)])
def test_attention_bound_rejects_one_tf32_pass(s, d):
    rng = np.random.default_rng(s + d)
    q, k, v = (rng.standard_normal((s, d)).astype(np.float32) for _ in range(3))
    rows = np.arange(0, s, max(1, s // 128))
    ref = C.attention_ref(q[rows], k, v)
    ok1, w1 = C.attention_check(C.attention_emulated(q[rows], k, v, 1), ref)
    ok3, w3 = C.attention_check(C.attention_emulated(q[rows], k, v, 3), ref)
    assert not ok1 and w1 >= 5 * C.ATTN_ROW, w1
    assert ok3 and w3 <= C.ATTN_ROW / 20, w3
