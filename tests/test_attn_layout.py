"""TMEM placement of P in the attention template (``ptxgen/tmpl_attn.py``).

The softmax thread of half h of a query row writes P for its keys
[h*hs, (h+1)*hs) (hs = BKV / split) over its own S columns: bf16 packed two
keys per column into the first hs/2 of them, f32 one column per key.  The
P . V issuer reads P one 32-byte K-step at a time (16 bf16 or 8 f32 keys, 8
TMEM columns).  Checked here for both dtypes and both splits: every K-step
reads only columns its keys' writer wrote, inside that writer's own S
columns (with split O nothing orders the two halves within a block, so a
write over the partner's scores would race with the partner's load), and
the steps cover every key of the block exactly once."""

import pytest

from ptxgen.tmpl_attn import _p_col

# (dtype, BKV, element bytes) as the template plans them
PLANS = {"bf16": (128, 2), "f32": (32, 4)}


def _writer_cols(key, bkv, split, f32):
    """Columns the writing softmax thread uses for ``key``."""
    hs = bkv // split
    h, i = divmod(key, hs)
    return h, (h * hs + i if f32 else h * hs + i // 2)


@pytest.mark.parametrize("split", [1, 2])
@pytest.mark.parametrize("dtype", ["bf16", "f32"])
def test_pv_reads_what_the_owning_half_wrote(dtype, split):
    bkv, e = PLANS[dtype]
    f32 = dtype == "f32"
    atom = 128 // e
    hs = bkv // split
    per_step = 32 // e                     # keys in one 32-byte K-step
    seen = []
    for c in range(max(1, bkv // atom)):
        for kk in range(min(4, bkv * e // 32)):
            k0 = c * atom + kk * per_step
            col = _p_col(k0, bkv, split, f32)
            keys = range(k0, k0 + per_step)
            owners = {_writer_cols(k, bkv, split, f32)[0] for k in keys}
            assert len(owners) == 1, (c, kk, owners)
            h = owners.pop()
            want = sorted({_writer_cols(k, bkv, split, f32)[1] for k in keys})
            assert list(range(col, col + 8)) == want, (c, kk, col, want)
            assert h * hs <= col and col + 8 <= (h + 1) * hs, (c, kk, col)
            seen += list(keys)
    assert sorted(seen) == list(range(bkv))
