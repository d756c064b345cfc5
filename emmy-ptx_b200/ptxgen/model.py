"""Kernel-level model: argument specs, buffers and dtype facts.

Mirrors the reference's ``ptxgen/model.py:8-88`` interface (``DTYPE``,
``dtype_info``, ``ArgSpec``, ``Buffer``, ``KernelSpec``) and extends the dtype
table with ``bf16``, which the reference lacks (``ptxgen/model.py:8-31``) and
the bf16 attention variant needs.
"""

from __future__ import annotations

from dataclasses import dataclass, field

# emmy dtype name -> (value kind, ptx storage type, element bytes)
DTYPE = {
    "f32": ("f32", "f32", 4),
    "f64": ("f64", "f64", 8),
    "f16": ("f16", "b16", 2),
    "bf16": ("bf16", "b16", 2),
    "i32": ("s32", "s32", 4),
    "u32": ("s32", "u32", 4),
    "i64": ("s64", "s64", 8),
    "u64": ("s64", "u64", 8),
    "bool": ("pred", "pred", 1),
    # C spellings that reach Smem declarations
    "float": ("f32", "f32", 4),
    "double": ("f64", "f64", 8),
    "half": ("f16", "b16", 2),
    "__half": ("f16", "b16", 2),
    "__nv_bfloat16": ("bf16", "b16", 2),
    "int": ("s32", "s32", 4),
    "long": ("s64", "s64", 8),
    "unsigned long long": ("s64", "u64", 8),
    "float32": ("f32", "f32", 4),
    "float64": ("f64", "f64", 8),
    "float16": ("f16", "b16", 2),
    "bfloat16": ("bf16", "b16", 2),
    "int32": ("s32", "s32", 4),
    "int64": ("s64", "s64", 8),
}


def dtype_name(dtype) -> str:
    return str(getattr(dtype, "name", dtype))


def dtype_info(dtype) -> tuple[str, str, int]:
    key = dtype_name(dtype)
    if key not in DTYPE:
        raise NotImplementedError(f"unsupported dtype {key!r}")
    return DTYPE[key]


def kind_of(dtype) -> str:
    return dtype_info(dtype)[0]


def elem_bytes(dtype) -> int:
    return dtype_info(dtype)[2]


@dataclass
class ArgSpec:
    """One kernel parameter, as ``meta.json`` describes it (``TASK.md:21-33``)."""

    name: str
    dtype: str
    shape: tuple[int, ...]
    scalar: bool = False
    value: float | int | None = None
    output: bool = False
    seed: int | None = None
    data: list | None = None
    intermediate: bool = False

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n

    @property
    def nbytes(self) -> int:
        return self.numel * elem_bytes(self.dtype)


@dataclass
class Buffer:
    name: str
    dtype: str
    shape: tuple[int, ...]

    @property
    def elem_bytes(self) -> int:
        return elem_bytes(self.dtype)

    @property
    def kind(self) -> str:
        return kind_of(self.dtype)

    @property
    def numel(self) -> int:
        n = 1
        for s in self.shape:
            n *= int(s)
        return n


@dataclass
class KernelSpec:
    """A loaded kernel: the IR op plus its launch contract from ``meta.json``."""

    op: object
    entry: str
    arg_order: list[str]
    args: dict[str, ArgSpec]
    grid: tuple[int, int, int] = (1, 1, 1)
    block: tuple[int, int, int] = (1, 1, 1)
    smem_bytes: int = 0
    zero_outputs: list[str] = field(default_factory=list)
    source: str = ""

    def buffer(self, name: str) -> Buffer:
        arg = self.args.get(name)
        if arg is None:
            raise KeyError(f"buffer {name!r} is not in meta.json arg_order")
        return Buffer(name=arg.name, dtype=arg.dtype, shape=arg.shape)

    @property
    def outputs(self) -> list[str]:
        return [n for n in self.arg_order if self.args[n].output]
