"""cail_reduce_sources_noalloc(): the reduction entry point for callers that
cannot allocate device memory (code running inside another allocator's
callbacks, which cannot re-enter the driver allocator it wraps, or a process
whose device memory a framework's caching allocator has already reserved).

The test calls the exported C symbol twice in a row for each of the 20
datatypes cail supports and each of SUM, PROD, MAX and MIN, on aligned
buffers and on views one element off a 16-byte boundary (counts that are
not a multiple of 16 bytes), and compares every result bit for bit with

* the existing local-reduction entry point, cail_gpu_reduce_local(), folding
  the same sources in the same order, and
* a rank-order fold on the CPU (torch for the types it has arithmetic for,
  numpy for the unsigned ones): acc = x_0; acc = op(acc, x_1); ...

It also checks that requests beyond the fixed scratch array are refused,
including a count whose byte size would overflow.  It runs in a fresh
process, so it behaves the same alone and after the other tests.
"""
import os
import subprocess
import sys

import pytest

from conftest import LIB, ROOT, gpu_count

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import ctypes, sys
import numpy as np, torch
sys.path.insert(0, %(root)r)
from cail_b200 import _lib
H = _lib.H
ctypes.CDLL(%(mpi)r, mode=ctypes.RTLD_GLOBAL)
c = ctypes.CDLL(%(cail)r)
vp = ctypes.c_void_p
c.cail_reduce_sources_noalloc.argtypes = [ctypes.POINTER(vp), ctypes.c_int, vp, ctypes.c_size_t,
                                          ctypes.c_int, ctypes.c_int, vp]
c.cail_gpu_reduce_local.argtypes = [vp, vp, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
torch.cuda.set_device(0)
# MPI datatype -> (numpy type, cail element type)
TYPES = {"MPI_CHAR": (np.int8, 0), "MPI_SHORT": (np.int16, 10), "MPI_INT": (np.int32, 1),
         "MPI_LONG": (np.int64, 2), "MPI_LONG_LONG": (np.int64, 5), "MPI_FLOAT": (np.float32, 3),
         "MPI_DOUBLE": (np.float64, 4), "MPI_UNSIGNED_CHAR": (np.uint8, 6), "MPI_UNSIGNED_SHORT": (np.uint16, 11),
         "MPI_UNSIGNED": (np.uint32, 7), "MPI_UNSIGNED_LONG": (np.uint64, 8),
         "MPI_UNSIGNED_LONG_LONG": (np.uint64, 9), "MPI_INT8_T": (np.int8, 0), "MPI_UINT8_T": (np.uint8, 6),
         "MPI_INT16_T": (np.int16, 10), "MPI_UINT16_T": (np.uint16, 11), "MPI_INT32_T": (np.int32, 1),
         "MPI_UINT32_T": (np.uint32, 7), "MPI_INT64_T": (np.int64, 5), "MPI_UINT64_T": (np.uint64, 9)}
OPS = [("MPI_SUM", 0, "sum"), ("MPI_PROD", 1, "prod"), ("MPI_MAX", 2, "max"), ("MPI_MIN", 3, "min")]
SIGNED = {np.uint8: np.int8, np.uint16: np.int16, np.uint32: np.int32, np.uint64: np.int64}
rng = np.random.default_rng(7)

def inputs(dt, op, n):
    if np.issubdtype(dt, np.floating):
        x = rng.uniform(0.999, 1.001, n) if op == "prod" else rng.standard_normal(n)
    elif op == "prod":
        x = rng.choice([1, -1], n) if np.issubdtype(dt, np.signedinteger) else rng.integers(1, 3, n)
    else:
        x = rng.integers(-8, 9, n) if np.issubdtype(dt, np.signedinteger) else rng.integers(0, 17, n)
    return np.asarray(x).astype(dt)

def cpu_fold(xs, op):
    dt = xs[0].dtype.type
    if dt in (np.uint16, np.uint32, np.uint64):
        acc = xs[0].copy()
        with np.errstate(over="ignore"):
            for x in xs[1:]:
                acc = {"sum": acc + x, "prod": acc * x, "max": np.where(acc > x, acc, x),
                       "min": np.where(acc < x, acc, x)}[op].astype(dt)
        return acc
    acc = torch.from_numpy(xs[0].copy())
    for x in xs[1:]:
        t = torch.from_numpy(x)
        acc = {"sum": acc + t, "prod": acc * t, "max": torch.where(acc > t, acc, t),
               "min": torch.where(acc < t, acc, t)}[op]
    return acc.numpy()

def device(x, offset):
    # x at `offset` elements into a fresh device buffer (offset 1: not 16-byte aligned)
    sv = SIGNED.get(x.dtype.type, x.dtype.type)
    buf = torch.zeros(x.size + offset + 16, dtype=getattr(torch, np.dtype(sv).name), device="cuda")
    buf[offset:offset + x.size] = torch.from_numpy(x.view(sv)).cuda()
    return buf, buf[offset:offset + x.size]

def host(t, dt):
    return t.cpu().numpy().view(dt)

checked = 0
for call in range(2):
    for mdt, (dt, cdt) in TYPES.items():
        esz = np.dtype(dt).itemsize
        for mop, cop, op in OPS:
            for nsrc, count, offset in ((1, 1000, 0), (4, 50003, 0), (8, 32768, 0), (3, 4097, 1), (8, 777, 1)):
                count = min(count, (256 << 10) // esz)
                xs = [inputs(dt, op, count) for _ in range(nsrc)]
                keep, srcs = zip(*[device(x, offset) for x in xs])
                obuf, out = device(np.full(count, 7, dtype=dt), offset)
                arr = (vp * nsrc)(*[s.data_ptr() for s in srcs])
                rc = c.cail_reduce_sources_noalloc(arr, nsrc, out.data_ptr(), count, H[mdt], H[mop],
                                                   torch.cuda.current_stream().cuda_stream)
                assert rc == 0, (mdt, mop, rc)
                torch.cuda.synchronize()
                # the existing entry point, folding in the same order
                rbuf, ref = device(xs[0], offset)
                for s in srcs[1:]:
                    assert c.cail_gpu_reduce_local(s.data_ptr(), ref.data_ptr(), count, cdt, cop) == 0
                torch.cuda.synchronize()
                got, via_local, want = host(out, dt), host(ref, dt), cpu_fold(xs, op)
                case = (call, mdt, mop, nsrc, count, offset)
                assert np.array_equal(got.view(np.uint8), via_local.view(np.uint8)), ("vs reduce_local",) + case
                assert np.array_equal(got.view(np.uint8), want.view(np.uint8)), ("vs cpu fold",) + case
                checked += 1
# requests beyond the scratch array are refused
big = torch.zeros(70000, device="cuda")
arr = (vp * 2)(big.data_ptr(), big.data_ptr())
assert c.cail_reduce_sources_noalloc(arr, 2, big.data_ptr(), 70000, H["MPI_FLOAT"], H["MPI_SUM"], None) == H["MPI_ERR_COUNT"]
arr9 = (vp * 9)(*([big.data_ptr()] * 9))
assert c.cail_reduce_sources_noalloc(arr9, 9, big.data_ptr(), 16, H["MPI_FLOAT"], H["MPI_SUM"], None) == H["MPI_ERR_COUNT"]
# a count whose byte size wraps around 2^64 must not pass as a small request
huge = (1 << 62) + 1
assert c.cail_reduce_sources_noalloc(arr, 2, big.data_ptr(), huge, H["MPI_FLOAT"], H["MPI_SUM"], None) == H["MPI_ERR_COUNT"]
print("NOALLOC OK", checked)
"""


def test_noalloc_entry_point_matches_reduce_local_and_cpu_fold():
    if gpu_count() < 1:
        pytest.skip("needs a GPU")
    code = SCRIPT % {"root": ROOT, "mpi": os.path.join(LIB, "libmpi.so"), "cail": os.path.join(LIB, "libcail.so")}
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "NOALLOC OK 800" in r.stdout, r.stdout
    assert "exceed the limit" in r.stderr
