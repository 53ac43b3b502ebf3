"""cail-b200: Blackwell-native MPI_Allreduce interposition library.

The library itself is native (``build/lib/libcail.so``, loaded with
LD_PRELOAD by MPI programs).  This package is the Python side: building,
loading, a tensor API over the interposed MPI_Allreduce, a DDP-style
gradient-bucketing harness and the benchmark model.

    import cail_b200 as cail
    cail.init()                      # MPI_Init (cail-mpirun or torchrun env)
    cail.ops.allreduce_(tensor)      # MPI_Allreduce(MPI_IN_PLACE, ...)
    cail.finalize()
"""
from __future__ import annotations

import ctypes
from typing import Optional

from . import _lib
from ._lib import H as MPI

__version__ = "0.1.0"

_state = {"rank": 0, "size": 1, "initialized": False}


def init(impl: str = "ours", host: bool = False) -> int:
    """Loads the libraries and calls MPI_Init_thread (MPI_THREAD_SERIALIZED).

    impl: "ours" | "reference" | "none" (see cail_b200._lib.load).  Returns
    the rank in MPI_COMM_WORLD.
    """
    libs = _lib.load(impl, host=host)
    flag = ctypes.c_int(0)
    libs.mpi.MPI_Initialized(ctypes.byref(flag))
    if not flag.value:
        provided = ctypes.c_int(0)
        rc = libs.mpi.MPI_Init_thread(None, None, MPI["MPI_THREAD_SERIALIZED"], ctypes.byref(provided))
        if rc != 0:
            raise RuntimeError(f"MPI_Init_thread failed ({rc})")
    r, s = ctypes.c_int(0), ctypes.c_int(1)
    libs.mpi.MPI_Comm_rank(MPI["MPI_COMM_WORLD"], ctypes.byref(r))
    libs.mpi.MPI_Comm_size(MPI["MPI_COMM_WORLD"], ctypes.byref(s))
    _state.update(rank=r.value, size=s.value, initialized=True)
    return r.value


def rank() -> int:
    return _state["rank"]


def world_size() -> int:
    return _state["size"]


def barrier() -> None:
    _lib.loaded().mpi.MPI_Barrier(MPI["MPI_COMM_WORLD"])


def finalize() -> None:
    """MPI_Finalize through the interposer (releases its device state)."""
    libs = _lib.loaded()
    if libs is None or not _state["initialized"]:
        return
    libs.cail.MPI_Finalize()
    _state["initialized"] = False


def last_algorithm() -> Optional[str]:
    libs = _lib.loaded()
    if libs is None or libs.impl != "ours":
        return None
    return libs.cail.cail_last_algorithm().decode()


def set_stream_ordered(on: bool) -> Optional[bool]:
    """Stream-ordered completion of NVLink allreduces (one_shot, two_shot
    through the push kernel, nvls): the call returns once the kernel is queued
    and the legacy default stream waits for it, as with NCCL; the default
    (False) is MPI's host-synchronous return.
    Returns the previous mode (None when the loaded interposer is not ours)."""
    libs = _lib.loaded()
    if libs is None or libs.impl != "ours":
        return None
    return bool(libs.cail.cail_set_stream_ordered(1 if on else 0))


class Stats(ctypes.Structure):
    _fields_ = [("calls", ctypes.c_ulonglong), ("passthrough", ctypes.c_ulonglong),
                ("by_algo", ctypes.c_ulonglong * 12), ("bytes", ctypes.c_ulonglong),
                ("reg_hits", ctypes.c_ulonglong), ("reg_misses", ctypes.c_ulonglong),
                ("device_errors", ctypes.c_ulonglong), ("launches", ctypes.c_ulonglong)]


def stats() -> Optional[Stats]:
    libs = _lib.loaded()
    if libs is None or libs.impl != "ours":
        return None
    s = Stats()
    libs.cail.cail_get_stats(ctypes.byref(s))
    return s


def host_max(value: float) -> float:
    """Max of a host double over MPI_COMM_WORLD (PMPI_Allreduce on host memory)."""
    libs = _lib.loaded()
    a = ctypes.c_double(value)
    b = ctypes.c_double(0.0)
    libs.mpi.PMPI_Allreduce(ctypes.byref(a), ctypes.byref(b), 1, MPI["MPI_DOUBLE"], MPI["MPI_MAX"],
                            MPI["MPI_COMM_WORLD"])
    return b.value


from . import ops  # noqa: E402

__all__ = ["init", "finalize", "rank", "world_size", "barrier", "ops", "stats", "last_algorithm", "host_max", "MPI"]
