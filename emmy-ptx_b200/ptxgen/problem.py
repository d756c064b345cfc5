"""Run a whole problem directory on the local B200: every kernel of
``meta.json`` in order, intermediates chained on the device.

This is the local counterpart of the reference runner loop
(``submit.py:80-159``): per kernel, compile (``compile_kernel``), build the
arguments -- ``seed`` -> ``default_rng(seed).standard_normal`` (one generator
per seed, drawn in ``arg_order``, ``docs/API.md:46``), ``data`` -> exact values,
outputs zeroed, ``intermediate`` -> the named output of an earlier kernel
(``submit.py:112-122``) -- launch, and collect the outputs.  Unlike the
reference, intermediates never leave the GPU: the consumer's buffer is filled
by a device-to-device copy from the producer's.  ``check`` compares against
``expected.npz`` with meta.json's ``rtol``/``atol`` the way ``submit.py:150-158``
does (``np.allclose``).

    python -m ptxgen.problem <problem_dir> [--geometry plan|meta]

prints one PASS/FAIL line per checked output and exits 1 on any failure.
"""

from __future__ import annotations

import argparse
import json
import sys
from pathlib import Path

import numpy as np

from .loader import load_kernel
from .model import KernelSpec


class ProblemError(RuntimeError):
    pass


def load_problem(pdir: str | Path) -> tuple[dict, list[KernelSpec]]:
    """meta.json and the KernelSpec of every kernel, in meta order."""
    pdir = Path(pdir)
    meta = json.loads((pdir / "meta.json").read_text())
    specs = []
    for k in meta["kernels"]:
        path = pdir / f"{k['entry']}.ir.json"
        if not path.exists():
            raise ProblemError(f"{k['entry']}: {path.name} not found in {pdir}")
        specs.append(load_kernel(path))
    return meta, specs


def seeded_inputs(spec: KernelSpec) -> dict[str, np.ndarray]:
    """Host arrays for the ``seed`` arguments of one kernel."""
    from .runtime import _np_dtype
    rngs: dict[int, np.random.Generator] = {}
    out = {}
    for name in spec.arg_order:
        a = spec.args[name]
        if a.scalar or a.output or a.intermediate or a.data is not None:
            continue
        seed = int(a.seed or 0)
        rng = rngs.setdefault(seed, np.random.default_rng(seed))
        out[name] = rng.standard_normal(a.shape).astype(_np_dtype(a.dtype))
    return out


def run_problem(pdir: str | Path, geometry: str = "plan", device: int = 0,
                return_all: bool = False) -> dict[str, np.ndarray]:
    """Run every kernel of the problem in meta order; returns the outputs
    (the graph outputs, or every kernel output with ``return_all``)."""
    from .emit import compile_kernel
    from .runtime import Device, PreparedKernel
    meta, specs = load_problem(pdir)
    dev = Device.get(device)
    producer: dict[str, PreparedKernel] = {}
    kernels: list[PreparedKernel] = []
    try:
        for spec in specs:
            pk = PreparedKernel(spec, ptx=compile_kernel(spec), dev=dev, geometry=geometry)
            kernels.append(pk)
            for name in spec.arg_order:
                a = spec.args[name]
                if not a.intermediate:
                    continue
                src = producer.get(name)
                if src is None:
                    raise ProblemError(f"{spec.entry} needs {name} from an earlier kernel "
                                       f"- kernels run in meta.json order")
                nbytes = src.spec.args[name].nbytes
                if nbytes != a.nbytes:
                    raise ProblemError(f"{spec.entry}: intermediate {name} is {a.nbytes} B, "
                                       f"its producer wrote {nbytes} B")
                dev.dtod(pk.bufs[name], src.bufs[name], nbytes)
            pk.upload(seeded_inputs(spec))
            pk.launch()
            dev.sync()
            pk.check_errors()
            for name in spec.outputs:
                producer[name] = pk
        wanted = (list(producer) if return_all
                  else [n for n in meta.get("graph_outputs", []) if n in producer] or list(producer))
        out = {}
        for name in wanted:
            out.update(producer[name].download([name]))
        return out
    finally:
        for pk in kernels:
            pk.close()


def check(outputs: dict[str, np.ndarray], pdir: str | Path) -> list[tuple[str, bool, float]]:
    """(name, passed, max abs error) per output that ``expected.npz`` holds."""
    pdir = Path(pdir)
    meta = json.loads((pdir / "meta.json").read_text())
    exp_path = pdir / "expected.npz"
    if not exp_path.exists():
        return []
    expected = np.load(exp_path)
    res = []
    for name in expected.files:
        if name not in outputs:
            continue
        ref = expected[name]
        got = np.asarray(outputs[name], dtype=np.float32).reshape(ref.shape)
        ok = bool(np.allclose(got, ref, rtol=meta["rtol"], atol=meta["atol"]))
        err = float(np.max(np.abs(got - ref))) if got.size else 0.0
        res.append((name, ok, err))
    return res


def main(argv=None) -> int:
    ap = argparse.ArgumentParser(prog="python -m ptxgen.problem")
    ap.add_argument("problem")
    ap.add_argument("--geometry", default="plan", choices=["plan", "meta"])
    args = ap.parse_args(argv)
    try:
        outs = run_problem(args.problem, geometry=args.geometry, return_all=True)
    except Exception as exc:  # one line, like compile.py's failures
        print(f"{args.problem}: {type(exc).__name__}: {exc}", file=sys.stderr)
        return 1
    results = check(outs, args.problem)
    if not results:
        for name, arr in outs.items():
            print(f"{name}: shape {list(arr.shape)} (no expected.npz to check against)")
        return 0
    ok = True
    for name, passed, err in results:
        print(f"{'PASS' if passed else 'FAIL'}  {name}: max abs err {err:.3e}")
        ok &= passed
    return 0 if ok else 1


if __name__ == "__main__":
    raise SystemExit(main())
