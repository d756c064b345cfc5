"""Elementwise op names, arities and reduce identities.

Same vocabulary and semantics as the reference's ``ptxgen/ops.py:6-67``:
emmy and C operator spellings map to one canonical name, and a reduce
accumulator is seeded with the identity of its op.  The max identity is
``-1e30``, not ``-inf`` (``ptxgen/ops.py:33-41``); kernels and oracle both
keep that value so an all-masked accumulator matches bit for bit.
"""

from __future__ import annotations

ALIASES = {
    "sum": "add",
    "prod": "multiply",
    "abs": "absolute",
    "neg": "negative",
    "pad": "copy",
    "positive": "copy",
    "pow": "power",
    "clamp": "clip",
    "amax": "maximum",
    "amin": "minimum",
    "max": "maximum",
    "min": "minimum",
    "__rshift__": "shr",
    "bitwise_right_shift": "shr",
    "right_shift": "shr",
    "+": "add",
    "-": "subtract",
    "*": "multiply",
    "/": "divide",
    "//": "floor_divide",
    "%": "remainder",
    "&": "bitand",
    "|": "bitor",
    "^": "bitxor",
    "<<": "shl",
    ">>": "shr",
}

IDENTITY = {
    "add": 0.0,
    "multiply": 1.0,
    "maximum": -1.0e30,
    "minimum": 1.0e30,
}

BINARY = {
    "add", "subtract", "multiply", "divide", "maximum", "minimum",
    "power", "where", "clip", "floor_divide", "remainder",
    "bitand", "bitor", "bitxor", "shl", "shr", "fmod",
    "logical_and", "logical_or",
}

TERNARY = {"fma", "where", "clip"}

UNARY = {
    "copy", "negative", "absolute", "relu", "exp", "exp_fast", "expm1", "log",
    "log1p", "log2", "log10", "sqrt", "rsqrt", "reciprocal", "tanh", "sigmoid",
    "silu", "softplus", "gelu", "gelu_tanh", "erf", "floor", "ceil",
    "trunc", "round", "sin", "cos", "sinh", "cosh", "bitcast", "square",
    "sign", "logical_not", "isnan", "isinf",
}

COMPARE = {"==", "!=", "<", "<=", ">", ">="}
LOGICAL = {"&&", "||"}


def canon(name: str) -> str:
    return ALIASES.get(name, name)


def identity(name: str) -> float:
    c = canon(name)
    if c not in IDENTITY:
        raise NotImplementedError(f"reduce op {name!r} has no known identity")
    return IDENTITY[c]
