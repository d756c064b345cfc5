"""Statement-by-statement sm_100a lowering of any Kernel IR (placeholder)."""

from .analysis import NoMatch


def emit_generic(spec):
    raise NoMatch("generic lowering not available")
