"""A small PTX text builder: virtual registers, labels, modules.

Kernels in this package are written as Python functions that emit PTX
instructions through this builder; ptxas does the register allocation.
Nothing here lowers through nvcc or any other compiler.
"""

from __future__ import annotations

import struct

PTX_VERSION = "8.8"
PTX_TARGET = "sm_100a"

# register class per value kind
_CLASS = {
    "pred": ("%p", ".pred"),
    "b16": ("%h", ".b16"),
    "s32": ("%r", ".b32"), "u32": ("%r", ".b32"), "b32": ("%r", ".b32"),
    "f32": ("%f", ".f32"),
    "s64": ("%rd", ".b64"), "u64": ("%rd", ".b64"), "b64": ("%rd", ".b64"),
    "f64": ("%fd", ".f64"),
}


def f32_hex(v: float) -> str:
    """Exact PTX literal of an f32 value (``0fXXXXXXXX``)."""
    return "0f%08X" % struct.unpack("<I", struct.pack("<f", float(v)))[0]


def f64_hex(v: float) -> str:
    return "0d%016X" % struct.unpack("<Q", struct.pack("<d", float(v)))[0]


class Reg(str):
    """A register name that remembers its kind."""

    kind: str

    def __new__(cls, name: str, kind: str):
        s = super().__new__(cls, name)
        s.kind = kind
        return s


class Kernel:
    """One ``.entry``: parameters, register declarations, body lines."""

    def __init__(self, entry: str, params: list[tuple[str, str]], maxntid: int | None = None,
                 minctas: int | None = None):
        self.entry = entry
        self.params = params  # (name, ptx type) e.g. ("p_x", ".u64")
        self.maxntid = maxntid
        self.minctas = minctas
        self.lines: list[str] = []
        self.counts: dict[str, int] = {}
        self._label = 0
        self.shared_decls: list[str] = []

    # -- registers / labels ------------------------------------------------

    def reg(self, kind: str) -> Reg:
        prefix, _ = _CLASS[kind]
        n = self.counts.get(prefix, 0)
        self.counts[prefix] = n + 1
        return Reg(f"{prefix}{n}", kind)

    def regs(self, kind: str, n: int) -> list[Reg]:
        return [self.reg(kind) for _ in range(n)]

    def label(self, hint: str = "L") -> str:
        self._label += 1
        return f"$L_{hint}_{self._label}"

    # -- emission ----------------------------------------------------------

    def __call__(self, text: str) -> None:
        self.lines.append("\t" + text + ";")

    def raw(self, text: str) -> None:
        self.lines.append(text)

    def place(self, label: str) -> None:
        self.lines.append(label + ":")

    def comment(self, text: str) -> None:
        self.lines.append("\t// " + text.encode("ascii", "replace").decode("ascii"))

    def shared(self, decl: str) -> None:
        self.shared_decls.append(decl)

    # -- common sequences --------------------------------------------------

    def param_ptr(self, pname: str) -> Reg:
        """Load a .u64 pointer parameter and convert it to a global address."""
        r = self.reg("u64")
        self(f"ld.param.u64 {r}, [{pname}]")
        self(f"cvta.to.global.u64 {r}, {r}")
        return r

    def sreg(self, name: str) -> Reg:
        r = self.reg("u32")
        self(f"mov.u32 {r}, {name}")
        return r

    def imm_u32(self, v: int) -> Reg:
        r = self.reg("u32")
        self(f"mov.u32 {r}, {int(v)}")
        return r

    def imm_f32(self, v: float) -> Reg:
        r = self.reg("f32")
        self(f"mov.f32 {r}, {f32_hex(v)}")
        return r

    def addr(self, base: Reg, index: Reg, scale: int) -> Reg:
        """base + index * scale with a 32-bit unsigned index."""
        a = self.reg("u64")
        if scale == 1:
            self(f"cvt.u64.u32 {a}, {index}")
            self(f"add.u64 {a}, {base}, {a}")
        else:
            self(f"mad.wide.u32 {a}, {index}, {scale}, {base}")
        return a

    def render(self) -> str:
        ps = ",\n".join(f"\t.param {t} {n}" for n, t in self.params)
        perf = ""
        if self.maxntid:
            perf += f".maxntid {self.maxntid}, 1, 1\n"
        if self.minctas:
            perf += f".minnctapersm {self.minctas}\n"
        decls = []
        for prefix, n in sorted(self.counts.items()):
            t = {"%p": ".pred", "%h": ".b16", "%r": ".b32", "%f": ".f32", "%rd": ".b64",
                 "%fd": ".f64"}[prefix]
            decls.append(f"\t.reg {t} {prefix}<{n}>;")
        body = "\n".join(self.shared_decls + decls + self.lines)
        return f".visible .entry {self.entry}(\n{ps}\n)\n{perf}{{\n{body}\n\tret;\n}}\n"


class Module:
    """A PTX module: header, module-scope variables, entries."""

    def __init__(self, comment: str = ""):
        self.comment = comment
        self.globals: list[str] = []
        self.kernels: list[Kernel] = []
        self.plan: dict | None = None

    def add_global(self, decl: str) -> None:
        if decl not in self.globals:
            self.globals.append(decl)

    def render(self) -> str:
        import json
        head = [f".version {PTX_VERSION}", f".target {PTX_TARGET}", ".address_size 64", ""]
        if self.comment:
            for line in self.comment.splitlines():
                head.append("// " + line.encode("ascii", "replace").decode("ascii"))
        if self.plan is not None:
            head.append("// @emmy-plan " + json.dumps(self.plan, sort_keys=True))
        head.append("")
        out = "\n".join(head) + "\n"
        if self.globals:
            out += "\n".join(self.globals) + "\n\n"
        out += "\n".join(k.render() for k in self.kernels)
        out.encode("ascii")  # PTX must be ASCII
        return out
