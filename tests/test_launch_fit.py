"""Every form of the attention template assembles for sm_100a and fits its
launch, on the CPU: f32 and bf16, head dims 32-256, split O on and off, and
the exp2 polynomial share at 0, 1 and 4 pairs of four.  So do the benchmark
kernels of every template, pre-pass kernels included, and a quarter of the
family fuzzer's cases, template and range-checked generic.

"Fits" means the main kernel's registers (allocated per thread in multiples
of 8) fit both the SM's 64K-register file for the whole block and each
sub-partition's 16K registers for the warps it hosts (warp w runs on
sub-partition w % 4).  A launch over either limit fails with "too many
resources requested", which ptxas alone does not report."""

import json
import re
import shutil
import subprocess

import pytest

from ptxgen import irgen
from ptxgen.emit import compile_kernel
from ptxgen.loader import load_kernel_data

VARIANTS = ([("f32", d, "1", None) for d in (32, 64, 128)]
            + [("bf16", d, so, None) for d in (32, 64, 128, 256) for so in ("1", "0")]
            + [("bf16", 128, "1", poly) for poly in ("0", "4")])


def _main_registers(ptxas_log: str, entry: str) -> int:
    """Registers of ``entry`` from ``ptxas -v`` output."""
    cur = None
    for line in ptxas_log.splitlines():
        m = re.search(r"Compiling entry function '(\w+)'", line)
        if m:
            cur = m.group(1)
        m = re.search(r"Used (\d+) registers", line)
        if m and cur == entry:
            return int(m.group(1))
    raise AssertionError(f"no register count for {entry}")


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
@pytest.mark.parametrize("dtype,d,split_o,poly", VARIANTS,
                         ids=[f"{t}-d{d}-so{s}-poly{p}" for t, d, s, p in VARIANTS])
def test_attention_form_assembles_and_fits(dtype, d, split_o, poly, tmp_path, monkeypatch):
    monkeypatch.setenv("EMMY_ATTN_SPLIT_O", split_o)
    if poly is not None:
        monkeypatch.setenv("EMMY_ATTN_EXP_POLY", poly)
    spec = load_kernel_data(*irgen.attention_bhsd(1, 2, 512, d, dtype), "av")
    ptx = compile_kernel(spec)
    plan = json.loads(re.search(r"// @emmy-plan (\{.*\})", ptx).group(1))
    assert plan["template"] == "attention"
    _assert_fits(spec, ptx, tmp_path)


def _assert_fits(spec, ptx, tmp_path):
    """Assemble ``ptx`` and check every launch it plans (the plan's main and
    pre-pass kernels, or meta.json's block for a kernel without a plan)."""
    m = re.search(r"// @emmy-plan (\{.*\})", ptx)
    plan = json.loads(m.group(1)) if m else None
    f = tmp_path / "k.ptx"
    f.write_text(ptx)
    r = subprocess.run(["ptxas", "-arch=sm_100a", "-v", "-o", "/dev/null", str(f)],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    launches = ([(plan["entry"], plan["block"])] + [(p["entry"], p["block"])
                                                    for p in plan.get("pre", [])]
                if plan else [(spec.entry, spec.block[0] * spec.block[1] * spec.block[2])])
    for entry, threads in launches:
        regs = -(-_main_registers(r.stderr, entry) // 8) * 8
        assert threads * regs <= 65536, (entry, threads, regs)
        assert -(-(threads // 32) // 4) * 32 * regs <= 16384, (entry, threads, regs)


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
@pytest.mark.parametrize("name", sorted(irgen.bench_kernels()))
def test_bench_kernel_fits(name, tmp_path):
    """Every benchmark kernel and its pre-pass kernels fit their launches."""
    spec = load_kernel_data(*irgen.bench_kernels()[name](), name)
    _assert_fits(spec, compile_kernel(spec), tmp_path)


@pytest.mark.skipif(shutil.which("ptxas") is None, reason="needs ptxas")
@pytest.mark.parametrize("seed", range(0, 192, 4))
def test_fuzz_kernel_fits(seed, tmp_path):
    """A quarter of the family fuzzer's cases, through their template and
    through the range-checked generic lowering under meta.json's block."""
    from tests import fuzz_ir
    c = fuzz_ir.case(seed)
    for checked in (False, True):
        _assert_fits(c.spec, compile_kernel(c.spec, checked=checked), tmp_path)
