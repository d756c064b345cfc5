"""Kernel IR -> sm_100a PTX: template selection.

The reference lowers every IR statement by statement for sm_89
(``ptxgen/emit.py:1553-1558``).  This backend recognises the IR's structure
and specialises a hand-written sm_100a template instead; the templates are
tried in order and the first whose ``match`` accepts the IR is used:

1. ``tmpl_mem.match_pointwise``    -- p00..p03 family
2. ``tmpl_mem.match_full_reduce``  -- r01..r03 family
3. ``tmpl_mem.match_rows``         -- r04, f01..f03 family
4. ``tmpl_mma.match_matmul``       -- m01/m02 family (tcgen05 + TMA)
5. ``tmpl_attn.match_attention``   -- a01/a02 family (tcgen05)
6. ``generic.emit_generic``        -- statement-by-statement lowering for
                                      anything else (the correctness floor)

There is no matching by problem or kernel name.
"""

from __future__ import annotations

import os
from pathlib import Path

from .analysis import NoMatch
from .loader import load_kernel
from .lower import LowerError
from .model import KernelSpec


def _candidates():
    from . import tmpl_mem
    out = [
        ("pointwise", tmpl_mem.match_pointwise, tmpl_mem.emit_pointwise),
        ("reduce_full", tmpl_mem.match_full_reduce, tmpl_mem.emit_full_reduce),
        ("rows", tmpl_mem.match_rows, tmpl_mem.emit_rows),
    ]
    try:
        from . import tmpl_mma
        out.append(("matmul", tmpl_mma.match_matmul, tmpl_mma.emit_matmul))
    except ImportError:
        pass
    try:
        from . import tmpl_attn
        out.append(("attention", tmpl_attn.match_attention, tmpl_attn.emit_attention))
    except ImportError:
        pass
    return out


def select_template(spec: KernelSpec):
    """Name and plan of the first template that accepts ``spec``."""
    reasons = []
    only = os.environ.get("EMMY_TEMPLATE")
    for name, match, emit in _candidates():
        if only and name != only:
            continue
        try:
            return name, match(spec), emit
        except NoMatch as exc:
            reasons.append(f"{name}: {exc}")
    return None, reasons, None


def compile_module(spec: KernelSpec, generic: bool = False, checked: bool = False):
    """Return the ``ptx.Module`` for ``spec`` (plan header included);
    ``generic=True`` (or ``EMMY_TEMPLATE=generic``) skips the templates.
    ``checked=True`` (or ``EMMY_CHECKED=1``) is the range-checked variant:
    the generic lowering with every global and shared index checked against
    its buffer; a violation skips the access and is reported through
    ``emmy_err`` (0x301) with the first offending buffer and index."""
    checked = checked or os.environ.get("EMMY_CHECKED", "") not in ("", "0")
    if checked or generic or os.environ.get("EMMY_TEMPLATE") == "generic":
        from . import generic as g
        mod = g.emit_generic(spec, checked=checked)
        mod.plan.setdefault("template", "generic")
        return mod
    name, plan, emit = select_template(spec)
    if name is not None:
        try:
            mod = emit(spec, plan)
            mod.plan = dict(mod.plan or {})
            mod.plan.setdefault("template", name)
            return mod
        except (NoMatch, LowerError) as exc:
            plan = [f"{name}: {exc}"]
    from . import generic
    try:
        mod = generic.emit_generic(spec)
        mod.plan.setdefault("template", "generic")
        return mod
    except (NoMatch, LowerError) as exc:
        why = "; ".join(plan) if isinstance(plan, list) else ""
        raise NotImplementedError(f"no template accepts this IR ({why}); generic lowering: {exc}")


def compile_kernel(spec: KernelSpec, generic: bool = False, checked: bool = False) -> str:
    """``KernelSpec`` -> PTX text (``ptxgen/emit.py:1553``)."""
    return compile_module(spec, generic=generic, checked=checked).render()


def compile_file(path: str | Path) -> str:
    """IR json path (sibling meta.json read implicitly) -> PTX text
    (``ptxgen/emit.py:1557``)."""
    return compile_kernel(load_kernel(path))
