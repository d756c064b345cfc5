#!/usr/bin/env python3
"""Emmy Kernel IR -> sm_100a PTX for NVIDIA B200.

Usage:
    python compile.py path/to/kernel.ir.json > out.ptx

The sibling meta.json is read implicitly.  Only PTX goes to stdout;
diagnostics go to stderr.  Same contract as the reference's ``compile.py:18-42``:
exactly one argument (else exit 2), a missing file exits 2, any compile
error exits 1 with one ``compile.py: <Type>: <message>`` line on stderr
(``PTXGEN_DEBUG=1`` prints the traceback instead), and the PTX ends with a
newline.
"""

from __future__ import annotations

import os
import sys
import traceback
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent / "emmy-ptx_b200"))


def main(argv: list[str]) -> int:
    if len(argv) != 2:
        print("usage: compile.py path/to/kernel.ir.json", file=sys.stderr)
        return 2
    path = Path(argv[1])
    if not path.is_file():
        print(f"compile.py: no such file: {path}", file=sys.stderr)
        return 2
    try:
        from ptxgen import compile_file

        ptx = compile_file(path)
    except Exception as exc:  # noqa: BLE001 - the contract is one clean line
        if os.environ.get("PTXGEN_DEBUG"):
            traceback.print_exc()
        else:
            msg = str(exc).replace("\n", " ")
            print(f"compile.py: {type(exc).__name__}: {msg}", file=sys.stderr)
        return 1
    if not ptx.endswith("\n"):
        ptx += "\n"
    sys.stdout.write(ptx)
    return 0


if __name__ == "__main__":
    raise SystemExit(main(sys.argv))
