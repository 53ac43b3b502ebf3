"""Locating and loading the native libraries (ctypes).

The in-tree CMake build puts everything under ``build/``:

* ``build/lib/libmpi.so``        minimpi, the bundled MPI subset
* ``build/lib/libcail.so``       the interposer (CUDA backend, sm_100a kernels)
* ``build/lib/libcail_host.so``  the host-only interposer
* ``build/bin/cail-mpirun``      the launcher

``load()`` opens libmpi and one interposer with RTLD_GLOBAL, in that order,
so ``MPI_Allreduce`` resolves to the interposer and everything else to
minimpi — the same arrangement as ``LD_PRELOAD=libcail.so``.  The MPI handle
values are read from ``mpi.h`` so Python never disagrees with C.
"""
from __future__ import annotations

import ctypes
import os
import re
from dataclasses import dataclass
from typing import Dict, Optional

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
BUILD = os.path.join(ROOT, "build")
LIB_DIR = os.path.join(BUILD, "lib")
BIN_DIR = os.path.join(BUILD, "bin")
MPI_H = os.path.join(ROOT, "csrc", "minimpi", "include", "mpi.h")
REF_LIB_DIR = os.path.join(ROOT, "baseline", "_ref", "lib")


def _parse_handles() -> Dict[str, int]:
    out: Dict[str, int] = {}
    pat = re.compile(r"#define\s+(MPI_\w+)\s+\(\((?:MPI_\w+|void\s*\*|MPI_Status\s*\*)\)\s*(-?\d+)\)")
    plain = re.compile(r"#define\s+(MPI_\w+)\s+\(?(-?\d+)\)?\s*$")
    with open(MPI_H) as f:
        for line in f:
            m = pat.match(line) or plain.match(line.strip())
            if m:
                out[m.group(1)] = int(m.group(2))
    return out


H = _parse_handles()


def lib_path(name: str) -> str:
    return os.path.join(LIB_DIR, name)


def launcher() -> str:
    return os.path.join(BIN_DIR, "cail-mpirun")


@dataclass
class Libs:
    mpi: ctypes.CDLL
    cail: ctypes.CDLL
    impl: str
    path: str


_loaded: Optional[Libs] = None


def _setup(lib: ctypes.CDLL) -> None:
    vp, i = ctypes.c_void_p, ctypes.c_int
    for name, args in {
        "MPI_Allreduce": [vp, vp, i, i, i, i],
        "MPI_Init_thread": [vp, vp, i, ctypes.POINTER(i)],
        "MPI_Finalize": [],
        "MPI_Barrier": [i],
        "MPI_Comm_rank": [i, ctypes.POINTER(i)],
        "MPI_Comm_size": [i, ctypes.POINTER(i)],
        "MPI_Initialized": [ctypes.POINTER(i)],
        "MPI_Finalized": [ctypes.POINTER(i)],
        "PMPI_Allreduce": [vp, vp, i, i, i, i],
        "MPI_Bcast": [vp, i, i, i, i],
        "MPI_Comm_split": [i, i, i, ctypes.POINTER(i)],
        "MPI_Comm_free": [ctypes.POINTER(i)],
        "MPI_Comm_set_errhandler": [i, i],
    }.items():
        if hasattr(lib, name):
            fn = getattr(lib, name)
            fn.argtypes = args
            fn.restype = ctypes.c_int


def load(impl: str = "ours", host: bool = False) -> Libs:
    """Loads libmpi plus an interposer.

    impl: "ours" (this repository's libcail), "reference" (the unmodified
    reference built by baseline/build_reference.py) or "none" (plain minimpi,
    i.e. the MPI's own PMPI_Allreduce).  host=True picks the host-only build.
    """
    global _loaded
    if _loaded is not None:
        if _loaded.impl != impl:
            raise RuntimeError(f"libraries already loaded as {_loaded.impl!r}")
        return _loaded
    mpi_path = lib_path("libmpi.so")
    if not os.path.exists(mpi_path):
        raise FileNotFoundError(f"{mpi_path} missing: run cail_b200.build.build_native() first")
    name = "libcail_host.so" if host else "libcail.so"
    if impl == "ours":
        path = lib_path(name)
    elif impl == "reference":
        path = os.path.join(REF_LIB_DIR, name)
    elif impl == "none":
        path = mpi_path
    else:
        raise ValueError(impl)
    if not os.path.exists(path):
        raise FileNotFoundError(f"{path} missing")
    # The interposer goes into the global scope before libmpi (its
    # dependency), so later global lookups of MPI_Allreduce find it first.
    cail = None if impl == "none" else ctypes.CDLL(path, mode=ctypes.RTLD_GLOBAL)
    mpi = ctypes.CDLL(mpi_path, mode=ctypes.RTLD_GLOBAL)
    if cail is None:
        cail = mpi
    _setup(mpi)
    _setup(cail)
    if impl == "ours":
        cail.cail_last_algorithm.restype = ctypes.c_char_p
        cail.cail_version.restype = ctypes.c_char_p
        cail.cail_comm_uses_nvlink.argtypes = [ctypes.c_int]
        cail.cail_comm_uses_nvls.argtypes = [ctypes.c_int]
        cail.cail_set_stream_ordered.argtypes = [ctypes.c_int]
        cail.cail_set_stream_sync.argtypes = [ctypes.c_int]
    _loaded = Libs(mpi=mpi, cail=cail, impl=impl, path=path)
    return _loaded


def loaded() -> Optional[Libs]:
    return _loaded
