#!/usr/bin/env python3
"""Regenerate the golden fixtures under ``tests/golden/`` from the reference.

Run where the reference checkout exists (``--ref PATH``, required).  It
writes:

* ``problems/<id>/``: each shipped problem's ``*.ir.json``, ``meta.json`` and
  ``expected.npz`` -- the reference's own golden vectors (numpy float64
  results cast to f32, ``tools/expressions_open.py:52-104``), copied as data;
* ``special_digests.json``, ``special_nonfinite_digests.json``: digests of
  the reference interpreter's outputs on every recorded IR with NaN,
  infinities, signed zeros, subnormals and (in the first) near-overflow
  values mixed into its inputs (``special_inputs``);
* ``fuzz_digests.json``, ``soup_digests.json``: SHA-256 digests of the
  reference interpreter's outputs on every case of the family fuzzer
  (``tests/fuzz_ir.py``) and of the statement-mix fuzzer
  (``tests/fuzz_soup.py``);
* ``ref_interp/<case>.npz``: outputs of the reference's golden model
  ``ptxgen/interp.py`` run here on extra inputs (every problem reseeded, plus
  IR that ``ptxgen.irgen`` generates at other shapes, plus random statement
  mixes from ``tests/fuzz_soup.py``).  The reference
  interpreter is imported from the checkout and fed IR objects built by this
  repository's own deserialiser, which stands in for the absent ``emmy-ml``
  package.  Inputs are not stored: ``cases.json`` records how to rebuild them.

Nothing at test time reads the reference checkout; only these files.
"""

from __future__ import annotations

import argparse
import hashlib
import importlib.util
import json
import shutil
import sys
import types
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
REPO = HERE.parent.parent
sys.path.insert(0, str(REPO / "emmy-ptx_b200"))
sys.path.insert(0, str(REPO))

from ptxgen import ir  # noqa: E402
from ptxgen.loader import load_kernel, load_kernel_data  # noqa: E402


def install_emmy_standin() -> None:
    """Register ``emmy.compiler.*`` modules whose classes are ours."""
    names = {
        "emmy": {},
        "emmy.compiler": {},
        "emmy.compiler.graph": {"Graph": ir.Graph},
        "emmy.compiler.ir": {},
        "emmy.compiler.ir.expr": {k: getattr(ir, k) for k in (
            "BinaryExpr", "Builtin", "CastExpr", "FlatIndex", "FuncCallExpr", "Literal",
            "TernaryExpr", "Var")},
        "emmy.compiler.ir.kernel": {k: getattr(ir, k) for k in (
            "Accum", "Assign", "Cond", "Load", "Loop", "Select", "Smem", "StridedLoop",
            "Sync", "Tile", "TreeHalve", "WarpShuffle", "Write", "KernelOp")},
        "emmy.compiler.ir.kernel.ir": {k: getattr(ir, k) for k in (
            "CpAsyncCommit", "CpAsyncCopy", "CpAsyncWait")},
        "emmy.compiler.ir.stmt": {k: getattr(ir, k) for k in ("Init", "Let", "ZeroPrologue")},
    }
    for mod, attrs in names.items():
        m = types.ModuleType(mod)
        m.__path__ = []  # mark as package
        for k, v in attrs.items():
            setattr(m, k, v)
        sys.modules[mod] = m


def import_reference(ref: Path):
    """Import the reference ``ptxgen`` package under the name ``refptxgen``."""
    install_emmy_standin()
    pkg = ref / "ptxgen"
    spec = importlib.util.spec_from_file_location(
        "refptxgen", pkg / "__init__.py", submodule_search_locations=[str(pkg)])
    mod = importlib.util.module_from_spec(spec)
    sys.modules["refptxgen"] = mod
    spec.loader.exec_module(mod)
    return importlib.import_module("refptxgen.interp")


def rebuild_inputs(spec, seed_offset: int, dist: str) -> dict[str, np.ndarray]:
    """Deterministic inputs for a case: runner argument forms with each
    ``seed`` shifted by ``seed_offset``; ``dist`` picks the distribution.
    Values are drawn in f64, rounded to f32 and then stored in the
    argument's own dtype (f16 and f64 arguments included)."""
    from ptxgen.runtime import _np_dtype
    out: dict[str, np.ndarray] = {}
    for name in spec.arg_order:
        a = spec.args[name]
        if a.scalar:
            continue
        dt = _np_dtype(a.dtype)
        if a.output:
            out[name] = np.zeros(a.shape, dtype=dt)
        elif a.data is not None:
            out[name] = np.asarray(a.data, dtype=np.float64).astype(np.float32).astype(
                dt).reshape(a.shape)
        else:
            rng = np.random.default_rng(int(a.seed or 0) + seed_offset)
            if dist == "normal":
                x = rng.standard_normal(a.shape)
            elif dist == "uniform01":
                x = rng.random(a.shape)
            else:
                x = rng.uniform(-1.0, 1.0, a.shape)
            out[name] = x.astype(np.float32).astype(dt)
    for name in spec.zero_outputs:
        if name in out:
            out[name][...] = 0
    return out


SOUP_CASES = 24


def generated_cases():
    """Extra IR at other shapes, produced by ``ptxgen.irgen``."""
    from ptxgen import irgen
    return irgen.golden_cases()


def main() -> int:
    ap = argparse.ArgumentParser()
    ap.add_argument("--ref", required=True, help="path of the reference checkout")
    ap.add_argument("--only", choices=["special"],
                    help="re-record only the special-value digests (every variant) of the "
                         "recorded IRs in cases.json")
    args = ap.parse_args()
    ref = Path(args.ref)
    if not (ref / "ptxgen" / "interp.py").exists():
        print(f"no reference checkout at {ref}", file=sys.stderr)
        return 2
    if args.only == "special":
        ref_interp = import_reference(ref)
        cases = json.loads((HERE / "cases.json").read_text())
        for variant in SPECIAL_VARIANTS:
            n = record_special_digests(ref_interp, cases, variant)
            print(f"{n} special-value digests written ({variant})")
        return 0

    # 1. copy the shipped problems
    pdst = HERE / "problems"
    if pdst.exists():
        shutil.rmtree(pdst)
    for pdir in sorted((ref / "problems").iterdir()):
        if not (pdir / "meta.json").exists():
            continue
        d = pdst / pdir.name
        d.mkdir(parents=True)
        for f in sorted(pdir.iterdir()):
            if f.name == "meta.json" or f.name == "expected.npz" or f.name.endswith(".ir.json"):
                shutil.copyfile(f, d / f.name)

    # 2. run the reference interpreter on extra inputs
    ref_interp = import_reference(ref)
    odst = HERE / "ref_interp"
    if odst.exists():
        shutil.rmtree(odst)
    odst.mkdir()
    cases = []
    for pdir in sorted(pdst.iterdir()):
        meta = json.loads((pdir / "meta.json").read_text())
        for k in meta["kernels"]:
            ir_path = pdir / f"{k['entry']}.ir.json"
            spec = load_kernel(ir_path)
            for off, dist in ((1000, "normal"), (2000, "uniform")):
                inputs = rebuild_inputs(spec, off, dist)
                outs = ref_interp.interpret(spec, inputs)
                case = f"{pdir.name}__{k['entry']}__{dist}{off}"
                np.savez_compressed(odst / f"{case}.npz", **{n: np.asarray(v) for n, v in outs.items()})
                cases.append({"case": case, "ir": f"problems/{pdir.name}/{ir_path.name}",
                              "seed_offset": off, "dist": dist})
    for name, data, meta, off, dist in generated_cases():
        spec = load_kernel_data(data, meta, source=name)
        gdir = HERE / "generated"
        gdir.mkdir(exist_ok=True)
        (gdir / f"{name}.ir.json").write_text(json.dumps(data, indent=1) + "\n")
        (gdir / f"{name}.meta.json").write_text(json.dumps(meta, indent=1) + "\n")
        inputs = rebuild_inputs(spec, off, dist)
        outs = ref_interp.interpret(spec, inputs)
        np.savez_compressed(odst / f"{name}.npz", **{n: np.asarray(v) for n, v in outs.items()})
        cases.append({"case": name, "ir": f"generated/{name}.ir.json",
                      "meta": f"generated/{name}.meta.json", "seed_offset": off, "dist": dist})
    # random statement mixes (Cond/Select/Loop/Let/Accum, tests/fuzz_soup.py)
    from tests import fuzz_soup
    for seed in range(SOUP_CASES):
        c = fuzz_soup.case(seed)
        name = f"soup_{seed:02d}"
        gdir = HERE / "generated"
        (gdir / f"{name}.ir.json").write_text(json.dumps(c.graph, indent=1) + "\n")
        (gdir / f"{name}.meta.json").write_text(json.dumps(c.meta, indent=1) + "\n")
        inputs = rebuild_inputs(c.spec, 0, "normal")
        outs = ref_interp.interpret(c.spec, inputs)
        np.savez_compressed(odst / f"{name}.npz", **{n: np.asarray(v) for n, v in outs.items()})
        cases.append({"case": name, "ir": f"generated/{name}.ir.json",
                      "meta": f"generated/{name}.meta.json", "seed_offset": 0, "dist": "normal"})
    (HERE / "cases.json").write_text(json.dumps(cases, indent=1) + "\n")
    print(f"{len(cases)} reference-interpreter cases written")
    n = record_fuzz_digests(ref_interp)
    print(f"{n} family-fuzzer digests written")
    n = record_fuzz_digests(ref_interp, "fuzz_soup", SOUP_FUZZ_CASES, "soup_digests.json")
    print(f"{n} statement-mix digests written")
    for variant in SPECIAL_VARIANTS:
        n = record_special_digests(ref_interp, cases, variant)
        print(f"{n} special-value digests written ({variant})")
    return 0


SPECIAL_VALUES = (np.nan, np.inf, -np.inf, -0.0, 1e-40, -1e-40, 3e38, -3e38, 0.0, 1.0)
# no near-overflow values: no sum of these inputs can overflow, so every
# output's NaN / +-inf / finite class is fixed by the inputs alone
NONFINITE_VALUES = (np.nan, np.inf, -np.inf, -0.0, 1e-40, -1e-40, 0.0, 1.0)

# variant -> (values, one element in ``every`` replaced, generator seed)
SPECIAL_VARIANTS = {"all": (SPECIAL_VALUES, 50, 1), "nonfinite": (NONFINITE_VALUES, 400, 2)}


def special_inputs(spec, variant: str = "all") -> dict[str, np.ndarray]:
    """``rebuild_inputs(spec, 5000, "normal")`` with special values mixed
    into every floating input of 8 or more elements (as stored in the
    argument's dtype).  Variant ``all``: one element in 50 replaced by NaN,
    +-inf, -0.0, an f32 subnormal, +-3e38, 0 or 1.  Variant ``nonfinite``:
    one in 400 replaced by the same values without +-3e38, sparse enough
    that finite, infinite and NaN outputs all occur in a contraction."""
    values, every, seed = SPECIAL_VARIANTS[variant]
    inputs = rebuild_inputs(spec, 5000, "normal")
    rng = np.random.default_rng(seed)
    special = np.array(values, np.float64)
    for name, a in inputs.items():
        if spec.args[name].output or a.dtype.kind != "f" or a.size < 8:
            continue
        flat = a.reshape(-1)
        idx = rng.choice(flat.size, size=max(1, flat.size // every), replace=False)
        with np.errstate(over="ignore"):
            flat[idx] = rng.choice(special, size=idx.size).astype(a.dtype)
    return inputs


SPECIAL_FILES = {"all": "special_digests.json", "nonfinite": "special_nonfinite_digests.json"}


def record_special_digests(ref_interp, cases, variant: str = "all") -> int:
    """``special_digests.json`` (variant ``all``) or
    ``special_nonfinite_digests.json``: the reference interpreter's outputs,
    as digests, on every recorded IR (shipped and generated) with
    ``special_inputs(spec, variant)``."""
    out, seen = [], set()
    for c in cases:
        if c["ir"] in seen:
            continue
        seen.add(c["ir"])
        spec = _case_spec(c)
        with np.errstate(all="ignore"):
            res = ref_interp.interpret(spec, special_inputs(spec, variant))
        out.append({"case": c["case"], "ir": c["ir"], **({"meta": c["meta"]} if "meta" in c else {}),
                    "outputs": {k: output_digest(v) for k, v in sorted(res.items())}})
    (HERE / SPECIAL_FILES[variant]).write_text(json.dumps(out, indent=1) + "\n")
    return len(out)


def _case_spec(c):
    if "meta" in c:
        return load_kernel_data(json.loads((HERE / c["ir"]).read_text()),
                                json.loads((HERE / c["meta"]).read_text()), c["case"])
    return load_kernel(HERE / c["ir"])


FUZZ_CASES = 192
SOUP_FUZZ_CASES = 128


def output_digest(arr) -> dict:
    """dtype, shape and SHA-256 of an output's bytes (C order)."""
    a = np.ascontiguousarray(np.asarray(arr))
    return {"dtype": str(a.dtype), "shape": list(a.shape),
            "sha256": hashlib.sha256(a.tobytes()).hexdigest()}


def record_fuzz_digests(ref_interp, module="fuzz_ir", n_cases=FUZZ_CASES,
                        fname="fuzz_digests.json") -> int:
    """``fname``: the reference interpreter's outputs on every case of a
    fuzzer (``tests/fuzz_ir.py``, the family fuzzer, or ``tests/fuzz_soup.py``,
    the statement mixes), as digests, so the oracle can be held to them bit
    for bit without storing the arrays.  Cases in a dtype the reference
    lacks (bf16) are listed as skipped."""
    import importlib
    fuzz = importlib.import_module(f"tests.{module}")
    out = []
    for seed in range(n_cases):
        c = fuzz.case(seed)
        try:
            res = ref_interp.interpret(c.spec, {k: v.copy() for k, v in c.inputs.items()})
        except NotImplementedError as exc:
            out.append({"seed": seed, "family": getattr(c, "family", "soup"), "skipped": str(exc)})
            continue
        out.append({"seed": seed, "family": getattr(c, "family", "soup"),
                    "outputs": {k: output_digest(v) for k, v in sorted(res.items())}})
    (HERE / fname).write_text(json.dumps(out, indent=1) + "\n")
    return sum("outputs" in o for o in out)


if __name__ == "__main__":
    raise SystemExit(main())
