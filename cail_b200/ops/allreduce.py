"""PyTorch front end of the interposed ``MPI_Allreduce``.

``allreduce_(t)`` reduces a CUDA (or CPU) tensor in place across the ranks
of a communicator by calling ``MPI_Allreduce(MPI_IN_PLACE, t, ...)``; with
cail loaded that call runs the sm_100a NVLink kernels for device tensors.
The call is blocking, like every MPI_Allreduce, and, as MPI requires, the
tensor must be ready when it is made: the function synchronises the
current CUDA stream first.  ctypes releases the GIL for the duration of the
call, so a background thread can overlap communication with compute.
"""
from __future__ import annotations

import ctypes
from typing import Optional

import torch

from .. import _lib

_DTYPES = {
    torch.float32: "MPI_FLOAT",
    torch.float64: "MPI_DOUBLE",
    torch.int8: "MPI_SIGNED_CHAR",
    torch.uint8: "MPI_UNSIGNED_CHAR",
    torch.int16: "MPI_SHORT",
    torch.int32: "MPI_INT",
    torch.int64: "MPI_LONG_LONG",
}
for _name, _mpi in (("uint16", "MPI_UNSIGNED_SHORT"), ("uint32", "MPI_UNSIGNED"), ("uint64", "MPI_UNSIGNED_LONG_LONG")):
    if hasattr(torch, _name):
        _DTYPES[getattr(torch, _name)] = _mpi

_OPS = {"sum": "MPI_SUM", "prod": "MPI_PROD", "max": "MPI_MAX", "min": "MPI_MIN", "band": "MPI_BAND"}


def mpi_datatype(dtype: torch.dtype) -> int:
    try:
        return _lib.H[_DTYPES[dtype]]
    except KeyError:
        raise TypeError(f"no MPI datatype for {dtype}") from None


def mpi_op(op: str) -> int:
    return _lib.H[_OPS[op.lower()]]


def _libs() -> _lib.Libs:
    libs = _lib.loaded()
    if libs is None:
        raise RuntimeError("cail_b200.init() has not been called")
    return libs


def allreduce_(t: torch.Tensor, op: str = "sum", comm: Optional[int] = None, sync: bool = True) -> torch.Tensor:
    """In-place allreduce of a contiguous tensor; returns ``t``."""
    if not t.is_contiguous():
        raise ValueError("allreduce_ needs a contiguous tensor")
    if t.numel() >= 2**31:
        raise ValueError("MPI_Allreduce counts are int; split tensors of 2^31 elements or more")
    libs = _libs()
    if sync and t.is_cuda:
        torch.cuda.current_stream(t.device).synchronize()
    rc = libs.cail.MPI_Allreduce(ctypes.c_void_p(_lib.H["MPI_IN_PLACE"] & (2**64 - 1)),
                                 ctypes.c_void_p(t.data_ptr()), t.numel(), mpi_datatype(t.dtype),
                                 mpi_op(op), _lib.H["MPI_COMM_WORLD"] if comm is None else comm)
    if rc != 0:
        raise RuntimeError(f"MPI_Allreduce failed with error {rc}")
    return t


def allreduce(src: torch.Tensor, dst: torch.Tensor, op: str = "sum", comm: Optional[int] = None,
              sync: bool = True) -> torch.Tensor:
    """Out-of-place allreduce ``dst = reduce(src)``; returns ``dst``."""
    if not (src.is_contiguous() and dst.is_contiguous()) or src.numel() != dst.numel():
        raise ValueError("allreduce needs contiguous tensors of equal size")
    if src.dtype != dst.dtype:
        raise TypeError("src and dst dtypes differ")
    libs = _libs()
    if sync and src.is_cuda:
        torch.cuda.current_stream(src.device).synchronize()
    rc = libs.cail.MPI_Allreduce(ctypes.c_void_p(src.data_ptr()), ctypes.c_void_p(dst.data_ptr()), src.numel(),
                                 mpi_datatype(src.dtype), mpi_op(op),
                                 _lib.H["MPI_COMM_WORLD"] if comm is None else comm)
    if rc != 0:
        raise RuntimeError(f"MPI_Allreduce failed with error {rc}")
    return dst
