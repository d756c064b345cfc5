"""ctypes launcher over ``libemmyrt.so``: the local replacement for the
reference's remote runner and ``submit.py``.

``run_kernel(spec, inputs)`` is the end-to-end call: host numpy arrays in,
host numpy arrays out, exactly the runner's argument semantics
(``docs/API.md:40-50``, ``submit.py:112-135``): inputs are copied to the
device, outputs start zeroed, ``zero_outputs`` are cleared before every
launch, and the kernel runs under either the PTX's own ``@emmy-plan`` launch
(default) or meta.json's grid/block/smem (``geometry="meta"``).

There is no CPU fallback: without the built library or a GPU every call
raises ``RuntimeError``.
"""

from __future__ import annotations

import ctypes as C
import hashlib
import json
import os
import re
from pathlib import Path

import numpy as np

from .model import KernelSpec, dtype_info


def _value_kind(dtype) -> str:
    """Register kind of a value of ``dtype`` (f16/bf16 values live in f32)."""
    k = dtype_info(dtype)[0]
    return "f32" if k in ("f16", "bf16") else k

_LIBDIR = Path(__file__).resolve().parent / "_lib"
_lib = None


class EmmyError(RuntimeError):
    pass


def lib_path() -> Path:
    return _LIBDIR / "libemmyrt.so"


def load_library():
    """Load and type ``libemmyrt.so`` (raises if it was not built)."""
    global _lib
    if _lib is not None:
        return _lib
    p = lib_path()
    if not p.exists():
        raise EmmyError(f"{p} is missing: run __graft_entry__.build() (or `make -C emmy-ptx_b200`)")
    L = C.CDLL(str(p))
    vp, i32, u32, u64, sz = C.c_void_p, C.c_int, C.c_uint32, C.c_uint64, C.c_size_t
    sig = {
        "emmy_version": (C.c_char_p, []),
        "emmy_last_error": (C.c_char_p, []),
        "emmy_device_count": (i32, [C.POINTER(i32)]),
        "emmy_ctx_create": (i32, [i32, C.POINTER(vp)]),
        "emmy_ctx_destroy": (i32, [vp]),
        "emmy_ctx_make_current": (i32, [vp]),
        "emmy_ctx_synchronize": (i32, [vp]),
        "emmy_device_info": (i32, [vp, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32),
                                   C.POINTER(sz), C.c_char_p, i32]),
        "emmy_module_load": (i32, [vp, C.c_char_p, C.POINTER(vp), C.c_char_p, sz]),
        "emmy_module_unload": (i32, [vp]),
        "emmy_module_global": (i32, [vp, C.c_char_p, C.POINTER(u64), C.POINTER(sz)]),
        "emmy_func_info": (i32, [vp, C.c_char_p, C.POINTER(i32), C.POINTER(i32), C.POINTER(i32),
                                 C.POINTER(i32)]),
        "emmy_launch": (i32, [vp, C.c_char_p, C.POINTER(u32), C.POINTER(u32), u32,
                              C.POINTER(vp), vp]),
        "emmy_launch_ptrs": (i32, [vp, C.c_char_p, C.POINTER(u32), C.POINTER(u32), u32,
                                   C.POINTER(u64), i32, vp]),
        "emmy_launch_ex": (i32, [vp, C.c_char_p, C.POINTER(u32), C.POINTER(u32), u32,
                                 C.POINTER(vp), vp, u32]),
        "emmy_tmap_encode": (i32, [vp, vp]),
        "emmy_tmap_fill": (i32, [vp, C.c_char_p, vp, vp]),
        "emmy_mem_alloc": (i32, [vp, sz, C.POINTER(u64)]),
        "emmy_mem_free": (i32, [vp, u64]),
        "emmy_host_alloc": (i32, [vp, sz, C.POINTER(vp)]),
        "emmy_host_free": (i32, [vp, vp]),
        "emmy_memcpy_htod": (i32, [u64, vp, sz, vp]),
        "emmy_memcpy_dtoh": (i32, [vp, u64, sz, vp]),
        "emmy_memcpy_dtod": (i32, [u64, u64, sz, vp]),
        "emmy_memset_d32": (i32, [u64, u32, sz, vp]),
        "emmy_ipc_handle": (i32, [vp, u64, vp]),
        "emmy_ipc_open": (i32, [vp, vp, C.POINTER(u64)]),
        "emmy_ipc_close": (i32, [vp, u64]),
        "emmy_stream_create": (i32, [vp, C.POINTER(vp)]),
        "emmy_stream_destroy": (i32, [vp]),
        "emmy_stream_sync": (i32, [vp]),
        "emmy_event_create": (i32, [vp, C.POINTER(vp)]),
        "emmy_event_destroy": (i32, [vp]),
        "emmy_event_record": (i32, [vp, vp]),
        "emmy_event_elapsed": (i32, [vp, vp, C.POINTER(C.c_float)]),
        "emmy_stream_wait_event": (i32, [vp, vp]),
        "emmy_error_word": (i32, [vp, C.POINTER(u32), i32, vp]),
        "emmy_nccl_unique_id": (i32, [vp]),
        "emmy_nccl_init": (i32, [vp, i32, i32, vp, C.POINTER(vp)]),
        "emmy_allreduce_sum_f32": (i32, [vp, u64, sz, vp]),
        "emmy_nccl_async_error": (i32, [vp, C.POINTER(i32)]),
        "emmy_nccl_abort": (i32, [vp]),
        "emmy_nccl_destroy": (i32, [vp]),
    }
    for name, (res, args) in sig.items():
        f = getattr(L, name)
        f.restype = res
        f.argtypes = args
    _lib = L
    return L


def check(rc: int, what: str = "") -> None:
    if rc != 0:
        msg = load_library().emmy_last_error().decode(errors="replace")
        raise EmmyError(f"{what}: {msg} (status {rc})" if what else f"{msg} (status {rc})")


class TmapDesc(C.Structure):
    _fields_ = [("base", C.c_uint64), ("rank", C.c_uint32), ("dtype", C.c_uint32),
                ("dims", C.c_uint64 * 5), ("strides", C.c_uint64 * 4), ("box", C.c_uint32 * 5),
                ("swizzle", C.c_uint32), ("l2_promote", C.c_uint32)]


TMAP_DTYPE = {"f32": 0, "bf16": 1, "f16": 2, "u8": 3}


def parse_plan(ptx: str) -> dict:
    m = re.search(r"^// @emmy-plan (\{.*\})$", ptx, re.M)
    return json.loads(m.group(1)) if m else {}


# ---------------------------------------------------------------------------
# device
# ---------------------------------------------------------------------------


class Device:
    """One GPU: its primary context, a stream, and loaded modules."""

    _cache: dict[int, "Device"] = {}

    @classmethod
    def get(cls, ordinal: int = 0) -> "Device":
        d = cls._cache.get(ordinal)
        if d is None:
            d = cls(ordinal)
            cls._cache[ordinal] = d
        return d

    def __init__(self, ordinal: int = 0):
        L = load_library()
        self.L = L
        self.ordinal = ordinal
        self.ctx = C.c_void_p()
        check(L.emmy_ctx_create(ordinal, C.byref(self.ctx)), "emmy_ctx_create")
        sm, ma, mi = C.c_int(), C.c_int(), C.c_int()
        mem = C.c_size_t()
        name = C.create_string_buffer(128)
        check(L.emmy_device_info(self.ctx, C.byref(sm), C.byref(ma), C.byref(mi), C.byref(mem),
                                 name, 128), "emmy_device_info")
        self.sm_count, self.cc = sm.value, (ma.value, mi.value)
        self.total_mem, self.name = mem.value, name.value.decode()
        if self.cc != (10, 0):
            raise EmmyError(f"device {ordinal} is {self.name} sm_{ma.value}{mi.value}; "
                            "this backend emits sm_100a code for B200")
        self.stream = C.c_void_p()
        check(L.emmy_stream_create(self.ctx, C.byref(self.stream)), "emmy_stream_create")
        self.modules: dict[str, "LoadedModule"] = {}

    # -- memory ------------------------------------------------------------

    def alloc(self, nbytes: int) -> int:
        """Device memory rounded up to 16 bytes, so word-wise zeroing of a
        buffer whose size is not a multiple of 4 (an odd count of f16)
        stays inside the allocation."""
        p = C.c_uint64()
        check(self.L.emmy_mem_alloc(self.ctx, max(16, (int(nbytes) + 15) & ~15), C.byref(p)),
              "emmy_mem_alloc")
        return p.value

    def free(self, ptr: int) -> None:
        check(self.L.emmy_mem_free(self.ctx, C.c_uint64(ptr)), "emmy_mem_free")

    def host_alloc(self, nbytes: int) -> int:
        p = C.c_void_p()
        check(self.L.emmy_host_alloc(self.ctx, max(16, int(nbytes)), C.byref(p)), "emmy_host_alloc")
        return p.value

    def host_free(self, ptr: int) -> None:
        check(self.L.emmy_host_free(self.ctx, C.c_void_p(ptr)), "emmy_host_free")

    def ipc_handle(self, ptr: int) -> bytes:
        """64-byte handle another process can open to address ``ptr``."""
        buf = C.create_string_buffer(64)
        check(self.L.emmy_ipc_handle(self.ctx, C.c_uint64(ptr), buf), "ipc handle")
        return buf.raw

    def ipc_open(self, handle: bytes) -> int:
        """Device pointer, valid in this context, to a peer's allocation."""
        if len(handle) != 64:
            raise EmmyError("an IPC handle is 64 bytes")
        out = C.c_uint64()
        buf = C.create_string_buffer(handle, 64)
        check(self.L.emmy_ipc_open(self.ctx, buf, C.byref(out)), "ipc open")
        return out.value

    def ipc_close(self, ptr: int) -> None:
        check(self.L.emmy_ipc_close(self.ctx, C.c_uint64(ptr)), "ipc close")

    def dtod(self, dst: int, src: int, nbytes: int, stream=None) -> None:
        check(self.L.emmy_memcpy_dtod(C.c_uint64(dst), C.c_uint64(src), nbytes,
                                      stream or self.stream), "dtod")

    def htod(self, dst: int, arr: np.ndarray, stream=None) -> None:
        arr = np.ascontiguousarray(arr)
        check(self.L.emmy_memcpy_htod(C.c_uint64(dst), arr.ctypes.data_as(C.c_void_p),
                                      arr.nbytes, stream or self.stream), "htod")

    def dtoh(self, arr: np.ndarray, src: int, stream=None) -> None:
        check(self.L.emmy_memcpy_dtoh(arr.ctypes.data_as(C.c_void_p), C.c_uint64(src),
                                      arr.nbytes, stream or self.stream), "dtoh")

    def memset32(self, dst: int, value: int, count: int, stream=None) -> None:
        check(self.L.emmy_memset_d32(C.c_uint64(dst), value, count, stream or self.stream),
              "memset")

    def sync(self, stream=None) -> None:
        check(self.L.emmy_stream_sync(stream or self.stream), "stream sync")

    # -- modules -----------------------------------------------------------

    def load(self, ptx: str) -> "LoadedModule":
        key = hashlib.sha256(ptx.encode()).hexdigest()
        m = self.modules.get(key)
        if m is None:
            h = C.c_void_p()
            log = C.create_string_buffer(16384)
            rc = self.L.emmy_module_load(self.ctx, ptx.encode(), C.byref(h), log, 16384)
            if rc != 0:
                raise EmmyError(f"PTX rejected: {self.L.emmy_last_error().decode()}\n"
                                f"{log.value.decode(errors='replace')}")
            m = LoadedModule(self, h, ptx)
            self.modules[key] = m
        return m

    # -- events ------------------------------------------------------------

    def event(self):
        e = C.c_void_p()
        check(self.L.emmy_event_create(self.ctx, C.byref(e)), "event create")
        return e

    def record(self, ev, stream=None) -> None:
        check(self.L.emmy_event_record(ev, stream or self.stream), "event record")

    def new_stream(self):
        s = C.c_void_p()
        check(self.L.emmy_stream_create(self.ctx, C.byref(s)), "stream create")
        return s

    def wait_event(self, stream, ev) -> None:
        check(self.L.emmy_stream_wait_event(stream, ev), "stream wait event")

    def elapsed_ms(self, a, b) -> float:
        ms = C.c_float()
        check(self.L.emmy_event_elapsed(a, b, C.byref(ms)), "event elapsed")
        return ms.value


class LoadedModule:
    def __init__(self, dev: Device, handle, ptx: str):
        self.dev = dev
        self.h = handle
        self.ptx = ptx
        self.plan = parse_plan(ptx)

    def has_global(self, sym: str) -> bool:
        p = C.c_uint64()
        n = C.c_size_t()
        return self.dev.L.emmy_module_global(self.h, sym.encode(), C.byref(p), C.byref(n)) == 0

    def global_ptr(self, sym: str) -> tuple[int, int]:
        p = C.c_uint64()
        n = C.c_size_t()
        check(self.dev.L.emmy_module_global(self.h, sym.encode(), C.byref(p), C.byref(n)),
              f"global {sym}")
        return p.value, n.value

    def func_info(self, entry: str) -> dict:
        r, s, t, l = C.c_int(), C.c_int(), C.c_int(), C.c_int()
        check(self.dev.L.emmy_func_info(self.h, entry.encode(), C.byref(r), C.byref(s),
                                        C.byref(t), C.byref(l)), "func info")
        return {"registers": r.value, "static_smem": s.value, "max_threads": t.value,
                "local_bytes": l.value}

    def fill_tmap(self, sym: str, base: int, dtype: str, dims, strides, box, swizzle: int) -> None:
        d = TmapDesc()
        d.base = base
        d.rank = len(dims)
        d.dtype = TMAP_DTYPE[dtype]
        for i, v in enumerate(dims):
            d.dims[i] = int(v)
        for i, v in enumerate(strides):
            d.strides[i] = int(v)
        for i, v in enumerate(box):
            d.box[i] = int(v)
        d.swizzle = int(swizzle)
        d.l2_promote = 256
        check(self.dev.L.emmy_tmap_fill(self.h, sym.encode(), C.byref(d), self.dev.stream),
              f"tensor map {sym}")

    def launch(self, entry: str, grid, block, smem: int, ptrs: list, stream=None,
               overlap: bool = False) -> None:
        """``ptrs``: one kernel argument per parameter, in ``arg_order``: a
        buffer address (int) or a by-value scalar (a ctypes value, the
        runner's ``"scalar": true`` argument form, ``docs/API.md:49``).
        ``overlap``: programmatic dependent launch (``emmy_launch_ex``)."""
        g = (C.c_uint32 * 3)(*[int(x) for x in grid])
        b = (C.c_uint32 * 3)(*[int(x) for x in block])
        if overlap:
            vals = [C.c_uint64(p) if isinstance(p, int) else p for p in ptrs]
            argv = (C.c_void_p * max(1, len(vals)))(
                *[C.cast(C.pointer(v), C.c_void_p) for v in vals])
            check(self.dev.L.emmy_launch_ex(self.h, entry.encode(), g, b, int(smem), argv,
                                            stream or self.dev.stream, 1), f"launch {entry}")
            return
        if all(isinstance(p, int) for p in ptrs):
            arr = (C.c_uint64 * max(1, len(ptrs)))(*[int(p) for p in ptrs])
            check(self.dev.L.emmy_launch_ptrs(self.h, entry.encode(), g, b, int(smem), arr,
                                              len(ptrs), stream or self.dev.stream),
                  f"launch {entry}")
            return
        vals = [C.c_uint64(p) if isinstance(p, int) else p for p in ptrs]
        argv = (C.c_void_p * max(1, len(vals)))(
            *[C.cast(C.pointer(v), C.c_void_p) for v in vals])
        check(self.dev.L.emmy_launch(self.h, entry.encode(), g, b, int(smem), argv,
                                     stream or self.dev.stream), f"launch {entry}")

    def error_word(self, clear: bool = True) -> int:
        if not self.has_global("emmy_err"):
            return 0
        v = C.c_uint32()
        check(self.dev.L.emmy_error_word(self.h, C.byref(v), 1 if clear else 0, self.dev.stream),
              "error word")
        return v.value


# ---------------------------------------------------------------------------
# launch geometry
# ---------------------------------------------------------------------------


def plan_geometry(plan: dict, dev: Device) -> tuple[tuple, tuple, int]:
    """The B200 launch a template asks for in its ``@emmy-plan`` header."""
    block = int(plan.get("block", 256))
    gmax = max(1, int(plan.get("grid_max", 1)))
    per_sm = int(plan.get("grid_per_sm", 0))
    grid = min(gmax, per_sm * dev.sm_count) if per_sm > 0 else gmax
    return (max(1, grid), 1, 1), (block, 1, 1), int(plan.get("smem", 0))


def meta_geometry(spec: KernelSpec) -> tuple[tuple, tuple, int]:
    return tuple(spec.grid), tuple(spec.block), int(spec.smem_bytes)


# ---------------------------------------------------------------------------
# prepared kernels (device-resident buffers) and the end-to-end call
# ---------------------------------------------------------------------------


class PreparedKernel:
    """A compiled kernel with device buffers for every argument.

    ``upload`` copies host inputs, ``launch`` runs one launch (re-zeroing
    ``zero_outputs`` first, like the runner), ``download`` copies outputs
    back.  Buffers are freed by ``close``."""

    def __init__(self, spec: KernelSpec, ptx: str | None = None, dev: Device | None = None,
                 geometry: str = "plan"):
        from .emit import compile_kernel
        self.spec = spec
        self.dev = dev or Device.get(0)
        self.ptx = ptx or compile_kernel(spec)
        self.mod = self.dev.load(self.ptx)
        self.plan = self.mod.plan
        if geometry == "meta":
            self.grid, self.block, self.smem = meta_geometry(spec)
        else:
            self.grid, self.block, self.smem = plan_geometry(self.plan, self.dev)
        self.geometry = geometry
        self.ws = 0
        self.bufs: dict[str, int] = {}
        self._own: dict[str, int] = {}      # what this kernel allocated (close frees it)
        self.scalars: dict[str, object] = {}
        for name in spec.arg_order:
            a = spec.args[name]
            if a.scalar:
                # passed by value, in the parameter type the kernel declares
                # for the argument's value kind (0 when meta.json gives none)
                ct = {"f32": C.c_float, "f64": C.c_double, "s32": C.c_int32,
                      "s64": C.c_int64}.get(_value_kind(a.dtype))
                if ct is None:
                    raise EmmyError(f"scalar argument {name} of dtype {a.dtype}")
                v = a.value if a.value is not None else 0
                self.scalars[name] = ct(float(v) if ct in (C.c_float, C.c_double) else int(v))
                continue
            self.bufs[name] = self._own[name] = self.dev.alloc(a.nbytes)
        for name in spec.arg_order:
            a = spec.args[name]
            if a.scalar:
                continue
            if a.output:
                self.dev.memset32(self.bufs[name], 0, (a.nbytes + 3) // 4)
            elif a.data is not None:
                self.dev.htod(self.bufs[name], np.asarray(a.data, np.float64).astype(
                    _np_dtype(a.dtype)).reshape(a.shape))
        if geometry != "meta":
            self._fill_tmaps()
        self.launches = 0

    def _fill_tmaps(self) -> None:
        """Workspace, tensor maps, then the flags that tell the kernel its
        plan (tensor maps, block size, shared memory) is in place."""
        w = self.plan.get("workspace")
        if w:
            self.ws = self.dev.alloc(int(w["bytes"]))
            ptr, _ = self.mod.global_ptr(w["sym"])
            self.dev.htod(ptr, np.array([self.ws], dtype=np.uint64))
        for t in self.plan.get("tmaps", []):
            base = self.ws if t["buf"] == "@ws" else self.bufs[t["buf"]]
            self.mod.fill_tmap(t["sym"], base + int(t.get("offset", 0)),
                               t["dtype"], t["dims"], t["strides"], t["box"], t["swizzle"])
        for f in self.plan.get("flags", []):
            ptr, size = self.mod.global_ptr(f["sym"])
            self.dev.htod(ptr, np.array([int(f["value"])], dtype=np.uint32))
        self.dev.sync()

    def bind(self, name: str, ptr: int) -> int:
        """Read argument ``name`` from the device buffer at ``ptr`` -- another
        kernel's copy of the same array, say, so that one host-to-device copy
        feeds both -- instead of the buffer it points at now; tensor maps over
        that argument are refilled.  Returns the previous address.  The
        caller keeps ``ptr`` alive while this kernel uses it; ``upload`` to
        ``name`` writes into it; ``close`` frees only the buffers this kernel
        allocated, whatever is bound."""
        a = self.spec.args[name]
        if a.scalar:
            raise EmmyError(f"bind: {name} is a by-value argument")
        old = self.bufs[name]
        self.bufs[name] = int(ptr)
        if self.geometry != "meta":
            for t in self.plan.get("tmaps", []):
                if t["buf"] == name:
                    self.mod.fill_tmap(t["sym"], int(ptr) + int(t.get("offset", 0)),
                                       t["dtype"], t["dims"], t["strides"], t["box"],
                                       t["swizzle"])
            self.dev.sync()
        return old

    def attach_peers(self, inbox) -> None:
        """Join a multi-GPU full reduction: the kernel's cross-GPU exchange
        (plan ``xgpu``) publishes into and reads from ``inbox``'s buffers
        (``ptxgen.dist.PeerInbox``).  Every rank must launch this kernel the
        same number of times: each launch meets the others' once."""
        x = self.plan.get("xgpu")
        if not x:
            raise EmmyError(f"{self.spec.entry}: this kernel has no cross-GPU exchange")
        if not 1 <= inbox.world <= int(x["max_ranks"]):
            raise EmmyError(f"cross-GPU exchange supports 1..{x['max_ranks']} ranks")
        ptrs = np.zeros(int(x["max_ranks"]), dtype=np.uint64)
        ptrs[:inbox.world] = inbox.ptrs
        for sym, arr in ((x["peers"], ptrs),
                         (x["rank"], np.array([inbox.rank], np.uint32)),
                         (x["epoch"], np.array([0], np.uint32)),
                         (x["world"], np.array([inbox.world], np.uint32))):
            ptr, _ = self.mod.global_ptr(sym)
            self.dev.htod(ptr, arr)
        self.dev.sync()
        self.peers_attached = True

    def detach_peers(self) -> None:
        """Leave the multi-GPU exchange: world 0 and no peer addresses in the
        module.  Modules are shared by every PreparedKernel of the same PTX,
        so an inbox's addresses must not outlive it there: a later kernel of
        this PTX would otherwise store into freed or unmapped memory."""
        x = self.plan.get("xgpu")
        if not x or not getattr(self, "peers_attached", False):
            return
        self.dev.sync()
        for sym, arr in ((x["world"], np.array([0], np.uint32)),
                         (x["peers"], np.zeros(int(x["max_ranks"]), dtype=np.uint64))):
            ptr, _ = self.mod.global_ptr(sym)
            self.dev.htod(ptr, arr)
        self.dev.sync()
        self.peers_attached = False

    def upload(self, inputs: dict[str, np.ndarray], stream=None) -> int:
        nbytes = 0
        for name, arr in inputs.items():
            if name not in self.bufs:
                continue
            a = self.spec.args[name]
            host = np.ascontiguousarray(np.asarray(arr).astype(_np_dtype(a.dtype), copy=False))
            if host.nbytes != a.nbytes:
                raise EmmyError(f"input {name}: {host.nbytes} bytes, expected {a.nbytes}")
            self.dev.htod(self.bufs[name], host, stream)
            nbytes += host.nbytes
        return nbytes

    @property
    def has_pre(self) -> bool:
        return self.geometry != "meta" and bool(self.plan.get("pre"))

    def launch_pre(self, stream=None) -> None:
        """The plan's preparatory launches (operand splitting), if any."""
        if self.geometry == "meta":
            return
        ptrs = self.kernel_args()
        for pre in self.plan.get("pre", []):
            g, b, sm = plan_geometry(pre, self.dev)
            self.mod.launch(pre["entry"], g, b, sm, ptrs, stream)
            self.launches += 1

    def kernel_args(self) -> list:
        """The launch's arguments in ``arg_order``: buffer addresses, and
        scalars by value."""
        return [self.scalars[n] if n in self.scalars else self.bufs[n]
                for n in self.spec.arg_order]

    def launch_main(self, stream=None, overlap: bool = False) -> None:
        """The main kernel.  ``overlap``: let it start while the previous
        kernel in the stream finishes -- taken only when the plan allows it
        (the kernel waits before its first write); the caller promises that
        the previous kernel writes none of this kernel's inputs."""
        # zero_outputs are cleared before every launch, except outputs the
        # plan's kernel writes in full without reading them (``overwrites``:
        # e.g. split-K whose slices one CTA accumulates before a plain store,
        # where 0 + x == x); under meta.json's geometry they are always cleared
        skip = set(self.plan.get("overwrites", [])) if self.geometry != "meta" else set()
        # and outputs the plan's kernel accumulates into (``zero``: K slices
        # reduce-added into C)
        extra = [n for n in self.plan.get("zero", []) if self.geometry != "meta"
                 and n not in self.spec.zero_outputs]
        for name in list(self.spec.zero_outputs) + extra:
            if name in skip:
                continue
            a = self.spec.args[name]
            self.dev.memset32(self.bufs[name], 0, (a.nbytes + 3) // 4, stream)
        ptrs = self.kernel_args()
        ov = overlap and self.geometry != "meta" and bool(self.plan.get("overlap"))
        self.mod.launch(self.spec.entry, self.grid, self.block, self.smem, ptrs, stream,
                        overlap=ov)
        self.launches += 1

    def launch(self, stream=None) -> None:
        self.launch_pre(stream)
        self.launch_main(stream)

    def download(self, names=None, stream=None) -> dict[str, np.ndarray]:
        out = {}
        for name in names or self.spec.outputs:
            a = self.spec.args[name]
            host = np.empty(a.shape, dtype=_np_dtype(a.dtype))
            self.dev.dtoh(host, self.bufs[name], stream)
            out[name] = host
        self.dev.sync(stream)
        return out

    def check_errors(self) -> None:
        self.dev.sync()
        code = self.mod.error_word(clear=True)
        if not code:
            return
        msg = f"kernel {self.spec.entry} reported error 0x{code:x}"
        names = self.plan.get("oob_names")
        if names and self.mod.has_global("emmy_oob_buf"):
            info = np.zeros(2, dtype=np.uint32)
            pb, _ = self.mod.global_ptr("emmy_oob_buf")
            pi, _ = self.mod.global_ptr("emmy_oob_index")
            self.dev.dtoh(info[:1], pb)
            self.dev.dtoh(info[1:], pi)
            self.dev.sync()
            if 0 < info[0] <= len(names):
                msg += (f": out-of-bounds access to {names[info[0] - 1]}"
                        f"[{int(info[1].astype(np.int32))}] (first violation; access skipped)")
            for ptr in (pb, pi):
                self.dev.memset32(ptr, 0, 1)
        raise EmmyError(msg)

    def close(self) -> None:
        self.detach_peers()
        for p in self._own.values():
            self.dev.free(p)
        self.bufs = {}
        self._own = {}
        if self.ws:
            self.dev.free(self.ws)
            self.ws = 0


def _np_dtype(dtype) -> np.dtype:
    k = dtype_info(dtype)[0]
    if k == "bf16":
        from ml_dtypes import bfloat16
        return np.dtype(bfloat16)
    return np.dtype({"f32": np.float32, "f64": np.float64, "f16": np.float16, "s32": np.int32,
                     "s64": np.int64, "pred": np.bool_}[k])


def run_kernel(spec: KernelSpec, inputs: dict[str, np.ndarray], geometry: str = "plan",
               ptx: str | None = None, device: int = 0) -> dict[str, np.ndarray]:
    """Compile and run ``spec`` on the GPU: host arrays in, host arrays out."""
    pk = PreparedKernel(spec, ptx=ptx, dev=Device.get(device), geometry=geometry)
    try:
        pk.upload(inputs)
        pk.launch()
        pk.check_errors()
        return pk.download()
    finally:
        pk.close()
