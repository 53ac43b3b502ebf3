"""What cail will do here: library version, the CAIL_* settings in effect and
the algorithm auto mode picks per rank count and message size on an NVLink
communicator (MPI_FLOAT SUM unless --dtype / --op say otherwise).

    python -m cail_b200.info [--ranks 2,4,8] [--dtype MPI_FLOAT] [--op MPI_SUM]

Needs no GPU and no MPI job: the table comes from cail_nvlink_auto_algorithm(),
which reads the same environment (CAIL_ONESHOT_MAX, CAIL_MSG_SMALL_THRESHOLD,
CAIL_TUNE_FILE, CAIL_NVLS_MIN_RANKS, CAIL_NVLS_MIN, CAIL_CE_MIN, CAIL_NVLS) as
the library inside a job.
"""
from __future__ import annotations

import argparse
import ctypes
import os
import sys
from typing import List, Optional

from . import _lib

SIZES = [32 << 10, 256 << 10, 512 << 10, 1 << 20, 16 << 20, 256 << 20, 1 << 30]


def _fmt(n: int) -> str:
    for unit, shift in (("GiB", 30), ("MiB", 20), ("KiB", 10)):
        if n >= 1 << shift and n % (1 << shift) == 0:
            return f"{n >> shift} {unit}"
    return f"{n} B"


def table(ranks: List[int], dtype: str, op: str) -> List[List[Optional[str]]]:
    mpi = ctypes.CDLL(os.path.join(_lib.LIB_DIR, "libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    del mpi
    cail = ctypes.CDLL(os.path.join(_lib.LIB_DIR, "libcail.so"))
    f = cail.cail_nvlink_auto_algorithm
    f.restype = ctypes.c_char_p
    f.argtypes = [ctypes.c_int, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
    out = []
    for p in ranks:
        row = []
        for b in SIZES:
            r = f(p, b, _lib.H[dtype], _lib.H[op])
            row.append(r.decode() if r else None)
        out.append(row)
    return out


def main(argv: Optional[List[str]] = None) -> int:
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--ranks", default="2,4,8")
    ap.add_argument("--dtype", default="MPI_FLOAT")
    ap.add_argument("--op", default="MPI_SUM")
    a = ap.parse_args(argv)
    if a.dtype not in _lib.H or a.op not in _lib.H:
        print(f"unknown handle {a.dtype if a.dtype not in _lib.H else a.op}", file=sys.stderr)
        return 2
    cail = ctypes.CDLL(os.path.join(_lib.LIB_DIR, "libcail.so"))
    cail.cail_version.restype = ctypes.c_char_p
    print(f"cail {cail.cail_version().decode()}  ({os.path.join(_lib.LIB_DIR, 'libcail.so')})")
    env = sorted((k, v) for k, v in os.environ.items() if k.startswith("CAIL_"))
    print("environment: " + (", ".join(f"{k}={v}" for k, v in env) if env else "no CAIL_* variables set"))
    ranks = [int(x) for x in a.ranks.split(",") if x]
    rows = table(ranks, a.dtype, a.op)
    print(f"\nauto mode on NVLink communicators, {a.dtype} {a.op}:")
    head = ["ranks"] + [_fmt(b) for b in SIZES]
    width = max(len(h) for h in head + [x or "-" for r in rows for x in r]) + 2
    print("".join(h.ljust(width) for h in head))
    for p, row in zip(ranks, rows):
        print("".join(c.ljust(width) for c in [str(p)] + [x or "-" for x in row]))
    return 0


if __name__ == "__main__":
    sys.exit(main())
