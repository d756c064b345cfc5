"""Multi-GPU plumbing: one process per GPU, sharding, peer inboxes, NCCL.

The reference is single-GPU (no collective anywhere).  Here work that shards
naturally is partitioned across the GPUs of one node with no exchange --
element ranges for pointwise work, row blocks for row kernels, M rows for
matmul, batch*head for attention.  Full reductions exchange their per-rank
results inside the reduction kernel itself, through peer inboxes mapped over
CUDA IPC (NVLink stores, no separate collective launch); an NCCL all-reduce
of the per-rank results is the alternative path.

Host-side coordination (rendezvous, timing reductions, the NCCL unique id)
goes through ``torch.distributed`` with the ``gloo`` backend: plumbing only,
no tensors on the GPU.  A rendezvous with a timeout precedes every NCCL
communicator, so a rank that never arrives (or fails first) makes the others
fail on the host, before any collective is enqueued on a GPU.
"""

from __future__ import annotations

import ctypes as C
import datetime
import os


def env_rank() -> tuple[int, int, int]:
    """(rank, world size, local rank) from the torch.distributed.run env."""
    return (int(os.environ.get("RANK", "0")), int(os.environ.get("WORLD_SIZE", "1")),
            int(os.environ.get("LOCAL_RANK", "0")))


def shard_range(n: int, world: int, rank: int, align: int = 1) -> tuple[int, int]:
    """Contiguous [start, stop) of ``n`` units for ``rank``; boundaries on
    multiples of ``align`` (16-byte vector access), remainder to the last
    rank."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    per = (n // world) // align * align
    start = per * rank
    stop = n if rank == world - 1 else start + per
    return start, stop


class Rendezvous:
    """Host-side process group (gloo) with a timeout on every operation."""

    def __init__(self, timeout_s: float = 120.0):
        self.rank, self.world, self.local = env_rank()
        self.td = None
        if self.world > 1:
            import torch.distributed as td
            td.init_process_group("gloo", timeout=datetime.timedelta(seconds=timeout_s))
            self.td = td
            self.barrier()   # every rank present before anything touches a GPU collective

    def barrier(self) -> None:
        if self.td is not None:
            self.td.barrier()

    def max(self, v: float) -> float:
        return self._reduce(v, "max")

    def sum(self, v: float) -> float:
        return self._reduce(v, "sum")

    def _reduce(self, v: float, op: str) -> float:
        if self.td is None:
            return v
        import torch
        t = torch.tensor([float(v)], dtype=torch.float64)
        self.td.all_reduce(t, op=self.td.ReduceOp.MAX if op == "max" else self.td.ReduceOp.SUM)
        return float(t.item())

    def bcast_bytes(self, b: bytes | None, src: int = 0) -> bytes:
        if self.td is None:
            return b
        obj = [b]
        self.td.broadcast_object_list(obj, src=src)
        return obj[0]

    def allgather_bytes(self, b: bytes) -> list[bytes]:
        """Every rank's ``b``, in rank order."""
        if self.td is None:
            return [b]
        out = [None] * self.world
        self.td.all_gather_object(out, b)
        return out

    def close(self) -> None:
        if self.td is not None:
            self.td.destroy_process_group()
            self.td = None


def physical_gpu(ordinal: int) -> str:
    """Host name and the physical GPU behind CUDA ordinal ``ordinal`` (the
    ``CUDA_VISIBLE_DEVICES`` entry, or the ordinal when unset)."""
    import socket
    vis = [v.strip() for v in os.environ.get("CUDA_VISIBLE_DEVICES", "").split(",") if v.strip()]
    gpu = vis[ordinal] if ordinal < len(vis) else str(ordinal)
    return f"{socket.gethostname()}:{gpu}"


class PeerInbox:
    """A small device buffer on every rank, opened by every other rank over
    CUDA IPC: the target of a kernel that publishes its partial result
    straight into its peers' memory over NVLink and reads theirs from its own
    (the fused cross-GPU reduction of the full-reduce template).  ``ptrs[r]``
    addresses rank r's inbox from this rank's GPU."""

    BYTES = 4096

    def __init__(self, dev, rdv: Rendezvous):
        self.dev, self.rank, self.world = dev, rdv.rank, rdv.world
        # kernels of different ranks wait for one another: they must run on
        # different GPUs, never as separate launches on one
        ids = rdv.allgather_bytes(physical_gpu(dev.ordinal).encode())
        if len(set(ids)) != len(ids):
            raise RuntimeError(f"peer inboxes need one GPU per rank, got {[i.decode() for i in ids]}")
        self.local = dev.alloc(self.BYTES)
        dev.memset32(self.local, 0, self.BYTES // 4)
        dev.sync()
        handles = rdv.allgather_bytes(dev.ipc_handle(self.local))
        self.ptrs, self.opened = [], []
        for r, h in enumerate(handles):
            if r == self.rank:
                self.ptrs.append(self.local)
            else:
                p = dev.ipc_open(h)
                self.opened.append(p)
                self.ptrs.append(p)
        rdv.barrier()            # every inbox zeroed and mapped before any kernel writes
        self.rdv = rdv

    def close(self) -> None:
        if self.local:
            self.dev.sync()
            self.rdv.barrier()   # no peer is still writing into this inbox
            for p in self.opened:
                self.dev.ipc_close(p)
            self.dev.free(self.local)
            self.local, self.opened = 0, []


class NcclComm:
    """An NCCL communicator over ``libemmyrt.so`` for the GPU of this rank."""

    def __init__(self, dev, rdv: Rendezvous):
        from .runtime import check
        self.dev = dev
        uid = None
        if rdv.rank == 0:
            buf = C.create_string_buffer(128)
            check(dev.L.emmy_nccl_unique_id(buf), "nccl unique id")
            uid = buf.raw
        uid = rdv.bcast_bytes(uid)
        self.h = C.c_void_p()
        ubuf = C.create_string_buffer(uid, 128)
        check(dev.L.emmy_nccl_init(dev.ctx, rdv.world, rdv.rank, ubuf, C.byref(self.h)),
              "nccl init")

    def allreduce_sum_f32(self, ptr: int, count: int, stream) -> None:
        from .runtime import check
        check(self.dev.L.emmy_allreduce_sum_f32(self.h, C.c_uint64(ptr), count, stream),
              "nccl all-reduce")

    def close(self) -> None:
        from .runtime import check
        if self.h:
            check(self.dev.L.emmy_nccl_destroy(self.h), "nccl destroy")
            self.h = None
