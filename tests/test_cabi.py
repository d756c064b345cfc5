"""The C-ABI library: builds, loads on a CPU-only machine, exports every
symbol ``include/emmyrt.h`` declares, and reports a missing driver as a
status instead of crashing."""

import ctypes
import re
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parent.parent
HEADER = ROOT / "include" / "emmyrt.h"


def _declared():
    text = HEADER.read_text()
    return sorted(set(re.findall(r"\b(emmy_[a-z0-9_]+)\s*\(", text)))


@pytest.fixture(scope="module")
def lib():
    from ptxgen.runtime import lib_path
    p = lib_path()
    if not p.exists():
        import subprocess
        subprocess.run(["make", "-C", str(ROOT / "emmy-ptx_b200")], check=True)
    return ctypes.CDLL(str(p))


def test_exports_every_declared_symbol(lib):
    names = _declared()
    assert len(names) >= 30
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_error_string(lib):
    lib.emmy_version.restype = ctypes.c_char_p
    assert lib.emmy_version().startswith(b"emmyrt")


def test_invalid_arguments_are_statuses(lib):
    lib.emmy_ctx_create.argtypes = [ctypes.c_int, ctypes.c_void_p]
    assert lib.emmy_ctx_create(0, None) == -3  # EMMY_EINVAL
    lib.emmy_launch_ptrs.argtypes = [ctypes.c_void_p] * 6 + [ctypes.c_int, ctypes.c_void_p]
    assert lib.emmy_launch_ptrs(None, None, None, None, 0, None, 999, None) == -3
