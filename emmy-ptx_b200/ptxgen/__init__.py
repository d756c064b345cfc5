"""ptxgen: Emmy Kernel IR -> sm_100a PTX for NVIDIA B200.

Same public names as the reference package (``ptxgen/__init__.py:3-7``)
except ``interpret``: the CPU golden model is test infrastructure here
(``oracle/``), and the product's way to *run* a kernel is ``run_kernel``,
which executes it on the GPU through ``libemmyrt.so``.
"""

from .loader import load_kernel
from .emit import compile_file, compile_kernel


def run_kernel(spec, inputs, **kw):
    """Compile ``spec``, run it on the local B200 and return its outputs."""
    from .runtime import run_kernel as _run
    return _run(spec, inputs, **kw)


def run_problem(pdir, **kw):
    """Run every kernel of a problem directory in meta.json order on the
    local B200, intermediates chained on the device (``submit.py:80-159``)."""
    from .problem import run_problem as _run
    return _run(pdir, **kw)


__all__ = ["load_kernel", "compile_kernel", "compile_file", "run_kernel", "run_problem"]
