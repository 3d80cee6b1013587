"""Communicator and TP plumbing mirroring python/picosgl/distributed/.

- ``PGBCommunicator`` satisfies the reference's ``PyNCCLCommunicator``
  protocol (distributed/pynccl.py:16-19): ``all_reduce(input, "sum")`` in
  place, ``all_gather(output, input)``, ``get_buffer()``. It is constructed
  like ``NCCLWrapper`` (rank, world_size, max_bytes, uid; csrc/src/pynccl.cu:76-93)
  and backed by libpgb's IPC peer buffers instead of an NCCL communicator.
- ``init_comm`` follows ``init_pynccl`` (distributed/pynccl.py:39-71): rank 0
  creates the uid, it is broadcast over the CPU (gloo) group, then the peer
  handles are exchanged over the same group and opened.
- ``DistributedCommunicator`` / ``PGBDistributedImpl`` mirror the class-level
  plug point of distributed/impl.py:34-62, and ``DistributedInfo`` /
  ``set_tp_info`` / ``get_tp_info`` mirror distributed/info.py:7-46.
"""

from __future__ import annotations

import ctypes
import sys
from abc import ABC, abstractmethod
from contextlib import contextmanager
from dataclasses import dataclass
from typing import Literal

import torch

from . import _lib
from .ops import _require_cuda, _stream, dtype_code

# ------------------------------------------------------------------ TP info --
# The tensor-parallel rank and size, process-wide. Same names and meaning as
# the reference's distributed/info.py:7-46 (DistributedInfo, set_tp_info,
# get_tp_info, try_get_tp_info, tp_override) so layer code written against
# those names runs unchanged. When this package runs inside the reference's
# process and only the reference's own module holds the TP info, the lookups
# below read it from there, so the two cannot disagree.


@dataclass(frozen=True)
class DistributedInfo:
    """Rank and size of the tensor-parallel group."""

    rank: int
    size: int

    def __post_init__(self):
        if not (self.size >= 1 and 0 <= self.rank < self.size):
            raise AssertionError(f"rank {self.rank} outside a TP group of {self.size}")

    def is_primary(self) -> bool:
        return self.rank == 0


class _TPState:
    current: DistributedInfo | None = None


def _reference_tp_info():
    mod = sys.modules.get("picosgl.distributed.info")
    getter = getattr(mod, "try_get_tp_info", None) if mod is not None else None
    info = getter() if getter is not None else None
    return None if info is None else DistributedInfo(int(info.rank), int(info.size))


def set_tp_info(tp_info: DistributedInfo) -> None:
    if _TPState.current is not None:
        raise AssertionError("the TP info is already set for this process")
    _TPState.current = tp_info


def try_get_tp_info() -> DistributedInfo | None:
    return _TPState.current if _TPState.current is not None else _reference_tp_info()


def get_tp_info() -> DistributedInfo:
    info = try_get_tp_info()
    if info is None:
        raise AssertionError("the TP info has not been set (call set_tp_info first)")
    return info


@contextmanager
def tp_override(tp_info: DistributedInfo):
    """Temporarily replace the TP info (restored on exit, errors included)."""
    before, _TPState.current = _TPState.current, tp_info
    try:
        yield
    finally:
        _TPState.current = before


# ------------------------------------------------------------- communicator --


def create_uid() -> bytes:
    """128 random bytes identifying one communicator (replaces create_nccl_uid)."""
    buf = (ctypes.c_uint8 * _lib.UID_BYTES)()
    _lib.call("pgb_create_uid", buf)
    return bytes(buf)


class PGBCommunicator:
    """libpgb communicator for one rank; see module docstring."""

    def __init__(self, rank: int, world_size: int, max_bytes: int, uid: bytes | list[int],
                 device: int | None = None):
        if isinstance(uid, (list, tuple)):
            uid = bytes((v & 0xFF) for v in uid)
        if len(uid) != _lib.UID_BYTES:
            raise ValueError(f"uid must be {_lib.UID_BYTES} bytes, got {len(uid)}")
        if device is None:
            device = torch.cuda.current_device()
        self.rank = rank
        self.world_size = world_size
        self.max_bytes = max_bytes
        self.device = device
        handle = ctypes.c_void_p()
        ubuf = (ctypes.c_uint8 * _lib.UID_BYTES).from_buffer_copy(uid)
        _lib.call("pgb_comm_create", rank, world_size, max_bytes, ubuf, device, ctypes.byref(handle))
        self._h = handle
        self._closed = False
        self.nvls = False  # NVLink multicast region bound (setup_nvls)

    # -- peer exchange ------------------------------------------------------
    def export_handle(self) -> bytes:
        n = _lib.load().pgb_comm_handle_size()
        buf = (ctypes.c_uint8 * n)()
        _lib.call("pgb_comm_export_handle", self._h, None, buf)
        return bytes(buf)

    def open_peers(self, handles: list[bytes]) -> None:
        if len(handles) != self.world_size:
            raise ValueError(f"expected {self.world_size} handles, got {len(handles)}")
        blob = b"".join(handles)
        buf = (ctypes.c_uint8 * len(blob)).from_buffer_copy(blob)
        _lib.call("pgb_comm_open_peers", self._h, buf)

    # -- PyNCCLCommunicator protocol ---------------------------------------
    def all_reduce(self, input: torch.Tensor, op: Literal["sum"] = "sum") -> None:
        _require_cuda("input", input)
        if op != "sum":
            raise ValueError(f"unsupported reduce op {op!r}")
        _lib.call("pgb_all_reduce", self._h, input.data_ptr(), input.numel(), dtype_code(input),
                  _lib.PGB_OP_SUM, _stream(input))

    def all_gather(self, output: torch.Tensor, input: torch.Tensor) -> None:
        _require_cuda("input", input)
        _require_cuda("output", output)
        if output.size(0) != input.size(0) * self.world_size:
            raise ValueError("Destination tensor has incorrect size")
        if output.dtype != input.dtype or output.numel() != input.numel() * self.world_size:
            raise ValueError("output must hold world_size copies of input's shape and dtype")
        _lib.call("pgb_all_gather", self._h, output.data_ptr(), input.data_ptr(), input.numel(),
                  dtype_code(input), _stream(input))

    def get_buffer(self) -> ctypes.c_void_p:
        out = ctypes.c_void_p()
        _lib.call("pgb_comm_get_buffer", self._h, ctypes.byref(out))
        return out

    def set_one_rank_path(self, fused: bool) -> None:
        """One rank only: run the row op as the fused kernel (True) or as the
        column GEMM followed by fused_add_rmsnorm (False, the default)."""
        _lib.call("pgb_comm_set_one_rank_path", self._h, int(bool(fused)))

    def set_exchange_mode(self, mode: str) -> None:
        """Multi-rank row ops: "auto" (the default: decode batches of up to
        256 tokens on the grid-barrier kernel, larger batches as the pair-tile
        column GEMM + all-reduce + fused_add_rmsnorm), "oneshot" / "twoshot"
        (the slice-exchange kernel), "barrier" (the grid-barrier kernel at
        every batch size), or "nvls" (NVLink multicast reduce; needs a
        communicator made with nvls=True on hardware that supports it, else
        "auto")."""
        codes = {"auto": _lib.PGB_XCHG_AUTO, "oneshot": _lib.PGB_XCHG_ONESHOT, "twoshot": _lib.PGB_XCHG_TWOSHOT,
                 "barrier": _lib.PGB_XCHG_BARRIER, "nvls": _lib.PGB_XCHG_NVLS}
        if mode not in codes:
            raise ValueError(f"unknown exchange mode {mode!r}; expected one of {sorted(codes)}")
        _lib.call("pgb_comm_set_exchange_mode", self._h, codes[mode])

    # -- health -------------------------------------------------------------
    def set_timeout(self, seconds: float) -> None:
        _lib.call("pgb_comm_set_timeout_ns", self._h, int(seconds * 1e9))

    def check_status(self, reset: bool = True) -> None:
        """Synchronise and raise PGBTimeout if a device-side wait ran out."""
        st = ctypes.c_int()
        _lib.call("pgb_comm_get_status", self._h, ctypes.byref(st), int(reset))
        if st.value:
            raise _lib.PGBTimeout(st.value, "communicator", "a bounded wait on a peer or the pipeline ran out; "
                                  "the communicator must be destroyed and re-created")

    @property
    def handle(self) -> ctypes.c_void_p:
        if self._closed:
            raise RuntimeError("communicator closed")
        return self._h

    def close(self) -> None:
        if not self._closed:
            self._closed = True
            _lib.call("pgb_comm_destroy", self._h)

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass


def _all_ok(flag: bool, group) -> bool:
    import torch.distributed as dist

    t = torch.tensor([1 if flag else 0], dtype=torch.int32)
    dist.all_reduce(t, op=dist.ReduceOp.MIN, group=group)
    return bool(t.item())


def setup_nvls(comm: PGBCommunicator, tp_rank: int, tp_size: int, tp_cpu_group, uid: bytes) -> bool:
    """Bind an NVLink multicast region to every rank of `comm` (see
    pgb_comm_nvls_create in include/pgb.h). Rank 0 creates the multicast
    object; its POSIX file descriptor reaches the other rank processes over an
    abstract Unix socket (SCM_RIGHTS) named after the communicator's uid. Every
    phase ends with an all-ranks agreement on the CPU group, so either every
    rank ends with the region bound (returns True) or none uses it (False)."""
    import os
    import socket

    lib = _lib.load()
    sup = ctypes.c_int(0)
    _lib.call("pgb_comm_nvls_supported", comm.handle, ctypes.byref(sup))
    if not _all_ok(bool(sup.value), tp_cpu_group):
        return False
    name = b"\0pgb-nvls-" + uid[:16].hex().encode()
    fd = -1
    if tp_rank == 0:
        fdc = ctypes.c_int(-1)
        created = lib.pgb_comm_nvls_create(comm.handle, ctypes.byref(fdc)) == 0
        srv = None
        if created:
            fd = fdc.value
            srv = socket.socket(socket.AF_UNIX, socket.SOCK_STREAM)
            srv.settimeout(120)
            srv.bind(name)
            srv.listen(tp_size)
        go = _all_ok(created, tp_cpu_group)  # the others connect only now
        try:
            if go:
                for _ in range(tp_size - 1):
                    conn, _ = srv.accept()
                    with conn:
                        socket.send_fds(conn, [b"f"], [fd])
        finally:
            if srv is not None:
                srv.close()
        if not go:
            if fd >= 0:
                os.close(fd)
            return False
    else:
        if not _all_ok(True, tp_cpu_group):
            return False
        with socket.socket(socket.AF_UNIX, socket.SOCK_STREAM) as cl:
            cl.settimeout(120)
            cl.connect(name)
            _, fds, _, _ = socket.recv_fds(cl, 16, 1)
        fd = fds[0]
    added = lib.pgb_comm_nvls_add(comm.handle, fd) == 0
    os.close(fd)
    if not _all_ok(added, tp_cpu_group):
        return False
    bound = lib.pgb_comm_nvls_bind(comm.handle) == 0
    comm.nvls = _all_ok(bound, tp_cpu_group)
    return comm.nvls


def init_comm(*, tp_rank: int, tp_size: int, tp_cpu_group, max_size_bytes: int = 0,
              device: int | None = None, nvls: bool = False) -> PGBCommunicator:
    """Create and connect a communicator over the CPU group (init_pynccl,
    pynccl.py:39-71). nvls=True also binds an NVLink multicast region where
    every device supports it (comm.nvls tells whether it did)."""
    import torch.distributed as dist

    ids = [create_uid()] if tp_rank == 0 else [None]
    if tp_size > 1:
        dist.broadcast_object_list(ids, src=0, group=tp_cpu_group)
    uid = ids[0]
    assert uid is not None, f"Failed to get communicator uid on {tp_rank = }"
    comm = PGBCommunicator(tp_rank, tp_size, max_size_bytes, uid, device)
    if tp_size > 1:
        handles: list = [None] * tp_size
        dist.all_gather_object(handles, comm.export_handle(), group=tp_cpu_group)
        comm.open_peers(handles)
        dist.barrier(group=tp_cpu_group)
        if nvls:
            setup_nvls(comm, tp_rank, tp_size, tp_cpu_group, uid)
    return comm


# ---------------------------------------------------- impl plug-in point --


class DistributedImpl(ABC):
    @abstractmethod
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor: ...

    @abstractmethod
    def all_gather(self, x: torch.Tensor) -> torch.Tensor: ...


class NoopDistributedImpl(DistributedImpl):
    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        return x


@dataclass
class PGBDistributedImpl(DistributedImpl):
    """PyNCCLDistributedImpl (impl.py:34-50) over a PGBCommunicator."""

    comm: PGBCommunicator

    def all_reduce(self, x: torch.Tensor) -> torch.Tensor:
        self.comm.all_reduce(x, "sum")
        return x

    def all_gather(self, x: torch.Tensor) -> torch.Tensor:
        world = self.comm.world_size
        shape = list(x.shape)
        shape[0] *= world
        result = x.new_empty(shape)
        self.comm.all_gather(result, x)
        return result


class DistributedCommunicator:
    impl: DistributedImpl = NoopDistributedImpl()
    # The libpgb communicator used by the fused row-parallel kernels (None
    # until enable_pgb_distributed or set_local_comm ran).
    comm: PGBCommunicator | None = None

    @classmethod
    def all_reduce(cls, x: torch.Tensor) -> torch.Tensor:
        return cls.impl.all_reduce(x)

    @classmethod
    def all_gather(cls, x: torch.Tensor) -> torch.Tensor:
        return cls.impl.all_gather(x)


def enable_pgb_distributed(tp_info: DistributedInfo, tp_cpu_group, max_bytes: int,
                           nvls: bool = False) -> PGBCommunicator:
    """enable_pynccl_distributed (impl.py:65-80) for the libpgb communicator."""
    comm = init_comm(tp_rank=tp_info.rank, tp_size=tp_info.size, tp_cpu_group=tp_cpu_group,
                     max_size_bytes=max_bytes, nvls=nvls)
    DistributedCommunicator.impl = PGBDistributedImpl(comm=comm)
    DistributedCommunicator.comm = comm
    return comm


def local_comm(max_bytes: int = 64 << 20) -> PGBCommunicator:
    """Single-rank communicator for TP=1: the fused row kernel still needs its
    slot buffer and counters."""
    if DistributedCommunicator.comm is None:
        DistributedCommunicator.comm = PGBCommunicator(0, 1, max_bytes, create_uid())
    return DistributedCommunicator.comm


def destroy_distributed() -> None:
    if DistributedCommunicator.comm is not None:
        DistributedCommunicator.comm.close()
    DistributedCommunicator.comm = None
    DistributedCommunicator.impl = NoopDistributedImpl()
