"""The IR generator reproduces the reference's shipped problems byte for byte
(graph, kernel body and launch contract), which pins the IR it writes at the
benchmark shapes to the reference's schedules."""

import json
from pathlib import Path

import pytest

from ptxgen import irgen

GOLDEN = Path(__file__).parent / "golden" / "problems"

CASES = {
    "p00_scalar_add": lambda: irgen.pointwise(128, 2, "add"),
    "p01_vector_add": lambda: irgen.pointwise(1024, 2, "add"),
    "p02_scale_shift": lambda: irgen.pointwise(4096, 4, "scale_shift",
                                               constants=[("mul_c1", 2.0), ("add_c1", 1.0)]),
    "p03_relu_mul": lambda: irgen.pointwise(2048, 4, "relu_mul", out="mul", entry="k_mul_pointwise"),
    "r01_array_sum": lambda: irgen.reduce_full(1024),
    "r02_big_sum": lambda: irgen.reduce_full(65536),
    "r03_mean": lambda: irgen.reduce_full(32768, mean=True),
    "r04_row_sum": lambda: irgen.reduce_rows(64, 512),
    "f01_rmsnorm": lambda: irgen.rmsnorm(64, 1024),
    "f02_row_softmax": lambda: irgen.softmax(64, 256),
    "f03_l2norm": lambda: irgen.l2norm(64, 512),
    "m01_matmul_512": lambda: irgen.matmul(512, 512, 512),
    "m02_matmul_rect": lambda: irgen.matmul_splitk(128, 64, 256, slice_k=8),
    "a01_attention": lambda: irgen.attention_tiled(64, 64, 8.0),
    "a02_attention_128": lambda: irgen.attention(128, 32, 5.656854),
}


@pytest.mark.parametrize("prob", sorted(CASES))
def test_generated_equals_shipped(prob):
    g, m = CASES[prob]()
    ref_graph = json.loads(next((GOLDEN / prob).glob("*.ir.json")).read_text())
    ref_meta = json.loads((GOLDEN / prob / "meta.json").read_text())
    assert g == ref_graph
    k0, k1 = ref_meta["kernels"][0], m["kernels"][0]
    for key in ("entry", "arg_order", "grid", "block", "smem_bytes", "zero_outputs", "args"):
        assert k0[key] == k1[key], key


def test_bench_kernels_parse():
    from ptxgen.loader import load_kernel_data
    for name, fn in irgen.bench_kernels().items():
        g, m = fn()
        spec = load_kernel_data(g, m, name)
        assert spec.entry


def test_splitk_groups_slices_per_cta():
    """The tcgen05 matmul template keeps only as many K-slice groups of a
    split-K IR as two waves of units on 148 SMs need: a CTA accumulates the
    rest in TMEM before its one atomic add."""
    from ptxgen import tmpl_mma
    from ptxgen.loader import load_kernel_data
    big = load_kernel_data(*irgen.matmul_splitk(16384, 4096, 1024, slice_k=128), "big")
    p = tmpl_mma.match_matmul(big)
    assert p.tc and p.slices == 1 and p.slice_k == 1024      # 2048 tiles: no split needed
    small = load_kernel_data(*irgen.matmul_splitk(256, 128, 256, slice_k=64), "small")
    p = tmpl_mma.match_matmul(small)
    assert p.slices == 4 and p.slice_k == 64                 # 2 tiles: keep the slices


def test_splitk_overwrites_only_when_slices_grouped():
    """A split-K plan lists C under ``overwrites`` (no clearing needed) only
    when each tile's slices are accumulated by one CTA and stored once."""
    import json
    import re
    from ptxgen.emit import compile_kernel
    from ptxgen.loader import load_kernel_data
    for (m, n, k), grouped in (((16384, 4096, 1024), True), ((256, 256, 1024), False)):
        spec = load_kernel_data(*irgen.matmul_splitk(m, n, k, slice_k=128), "sk")
        plan = json.loads(re.search(r"// @emmy-plan (\{.*\})", compile_kernel(spec)).group(1))
        assert (plan.get("overwrites") == ["matmul"]) == grouped, (m, n, k, plan.get("split_k"))


def test_matmul_tile_width(monkeypatch):
    """The C tile width: 256 or 128 where it divides N (every BASELINE shape
    and its row shards); N itself for 160, 192, 224; 256 with a ragged edge
    for longer N that are multiples of 32 only (such N used to fall to 64-
    or 32-column tiles); the divisor rule otherwise."""
    from ptxgen import tmpl_mma
    monkeypatch.delenv("EMMY_MATMUL_BN", raising=False)
    want = {(8192, 8192): 256, (16384, 4096): 256, (1024, 8192): 256, (2048, 4096): 256,
            (4096, 4096): 256, (512, 512): 256, (256, 128): 128, (384, 192): 192,
            (1024, 4160): 256, (512, 2496): 256, (512, 2400): 256, (256, 96): 32, (128, 64): 64}
    for (m, n), bn in want.items():
        assert tmpl_mma._choose_bn(m, n) == bn, (m, n)
    monkeypatch.setenv("EMMY_MATMUL_BN", "224")
    assert tmpl_mma._choose_bn(1024, 8192) == 224
    monkeypatch.setenv("EMMY_MATMUL_BN", "100")            # not a choice: the rule
    assert tmpl_mma._choose_bn(1024, 8192) == 256


def test_matmul_ragged_edge_guards_stores(monkeypatch):
    """With a ragged N edge the C stores (and the non-finite recompute) are
    predicated on the chunk's first column being inside N; without one the
    store path is unchanged."""
    from ptxgen.emit import compile_kernel
    from ptxgen.loader import load_kernel_data
    monkeypatch.delenv("EMMY_MATMUL_BN", raising=False)
    rag = compile_kernel(load_kernel_data(*irgen.matmul(1024, 4160, 256), "rag"))
    even = compile_kernel(load_kernel_data(*irgen.matmul(8192, 8192, 256), "even"))
    store = "cp.async.bulk.tensor.2d.global.shared::cta.bulk_group"
    assert sum(1 for ln in rag.splitlines() if store in ln) == 256 // 32
    # each guarded store names its own predicate; unguarded ones the issuer's
    preds_rag = {ln.split()[0] for ln in rag.splitlines() if store in ln}
    preds_even = {ln.split()[0] for ln in even.splitlines() if store in ln}
    assert len(preds_even) == 1 and len(preds_rag) == 256 // 32
