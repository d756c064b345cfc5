"""The range-checked compile mode (``compile_kernel(spec, checked=True)`` or
``EMMY_CHECKED=1``): every global access of an IR whose tile reaches past its
input goes through an index clamped to 0 when out of range, so the kernel can
never touch memory outside its buffers; it assembles for sm_100a."""

import re
import shutil
import subprocess

import pytest

from ptxgen import irgen
from ptxgen.emit import compile_kernel, compile_module
from ptxgen.irgen import V, ax, assign, load, package, tile, write
from ptxgen.loader import load_kernel_data

N_IN, N_TILE = 1000, 1024


def oob_spec():
    """y[i] = x[i] * x[i] for i < 1024, with x only 1000 elements long."""
    body = [tile([ax("a0", N_TILE)], [load("in0", "x", (V("a0"),)),
                                      assign("v0", "multiply", "in0", "in0"),
                                      write("y", (V("a0"),), ("v0",))])]
    g, m = package("k_oob", "y", body, [("x", (N_IN,), "f32", 0)], [], ("y", (N_TILE,), "f32"),
                   ["x", "y"], (N_TILE // 256, 1, 1), (256, 1, 1), pid="oob")
    return load_kernel_data(g, m, "oob")


def _defs(ptx):
    d = {}
    for line in ptx.splitlines():
        m = re.match(r"\s*(?:@%p\d+ )?([a-z][\w.]*)\s+(%\w+),", line)
        if m:
            d.setdefault(m.group(2), []).append(line.strip())
    return d


def test_every_global_access_uses_a_clamped_index():
    ptx = compile_kernel(oob_spec(), checked=True)
    defs = _defs(ptx)
    accesses = re.findall(r"(?:ld|st)\.global\.\w+\s+(?:%\w+, )?\[(%rd\d+)\]", ptx)
    assert accesses, ptx
    for a in accesses:
        mad = [l for l in defs.get(a, []) if l.startswith("mad.wide.s32")]
        assert mad, (a, defs.get(a))
        idx = mad[0].split()[2].rstrip(",")
        assert all(l.startswith("selp.s32") and l.split()[-2].rstrip(",") == "0"
                   for l in defs[idx]), (idx, defs[idx])


def test_checked_plan_names_buffers():
    mod = compile_module(oob_spec(), checked=True)
    assert mod.plan["checked"] and mod.plan["oob_names"] == ["x", "y"]
    assert "emmy_oob_buf" in mod.render()


def test_checked_assembles(tmp_path):
    if shutil.which("ptxas") is None:
        pytest.skip("ptxas not on PATH")
    for spec in (oob_spec(), load_kernel_data(*irgen.matmul_splitk(256, 128, 256, 64), "sk")):
        p = tmp_path / "k.ptx"
        p.write_text(compile_kernel(spec, checked=True))
        r = subprocess.run(["ptxas", "-arch=sm_100a", "-o", "/dev/null", str(p)],
                           capture_output=True, text=True)
        assert r.returncode == 0, r.stderr
