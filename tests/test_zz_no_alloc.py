"""cail_reduce_sources_noalloc(): the reduction entry point for callers that
cannot allocate device memory (for example code running inside another
allocator's callbacks, or in a process whose device memory a framework's
caching allocator has already reserved).

The test calls the exported C symbol twice in a row and compares each result
with the existing local-reduction entry point, cail_gpu_reduce_local(),
folding the same sources in the same order; it also checks that a request
beyond the fixed scratch size is refused.  It runs in a fresh process, so it
behaves the same alone and after the other tests.
"""
import os
import subprocess
import sys

import pytest

from conftest import LIB, ROOT, gpu_count

pytestmark = pytest.mark.gpu

SCRIPT = r"""
import ctypes, sys, torch
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
g = torch.Generator(device="cuda").manual_seed(7)
# (torch dtype, MPI datatype, cail element type, MPI op, cail op)
CASES = [(torch.float32, "MPI_FLOAT", 3, "MPI_SUM", 0), (torch.int32, "MPI_INT", 1, "MPI_MAX", 2),
         (torch.float64, "MPI_DOUBLE", 4, "MPI_PROD", 1), (torch.uint8, "MPI_UNSIGNED_CHAR", 6, "MPI_MIN", 3)]

def make(dt, n):
    if dt.is_floating_point:
        return 1.0 + 0.001 * torch.randn(n, device="cuda", dtype=dt, generator=g)
    return torch.randint(0, 100, (n,), device="cuda", dtype=dt, generator=g)

for call in range(2):
    for dt, mdt, cdt, mop, cop in CASES:
        for nsrc, count in ((1, 1000), (4, 50003), (8, 32768)):
            count = min(count, (256 << 10) // torch.tensor([], dtype=dt).element_size())
            srcs = [make(dt, count) for _ in range(nsrc)]
            out = torch.full((count,), 7, device="cuda", dtype=dt)
            arr = (vp * nsrc)(*[s.data_ptr() for s in srcs])
            rc = c.cail_reduce_sources_noalloc(arr, nsrc, out.data_ptr(), count, H[mdt], H[mop],
                                               torch.cuda.current_stream().cuda_stream)
            assert rc == 0, rc
            torch.cuda.synchronize()
            ref = srcs[0].clone()
            for s in srcs[1:]:
                assert c.cail_gpu_reduce_local(s.data_ptr(), ref.data_ptr(), count, cdt, cop) == 0
            torch.cuda.synchronize()
            if dt.is_floating_point:
                assert torch.allclose(out, ref, rtol=1e-5, atol=1e-6), (call, mdt, mop, nsrc)
            else:
                assert torch.equal(out, ref), (call, mdt, mop, nsrc)
# requests beyond the scratch size are refused
big = torch.zeros(70000, device="cuda")
arr = (vp * 2)(big.data_ptr(), big.data_ptr())
assert c.cail_reduce_sources_noalloc(arr, 2, big.data_ptr(), 70000, H["MPI_FLOAT"], H["MPI_SUM"], None) == H["MPI_ERR_COUNT"]
arr9 = (vp * 9)(*([big.data_ptr()] * 9))
assert c.cail_reduce_sources_noalloc(arr9, 9, big.data_ptr(), 16, H["MPI_FLOAT"], H["MPI_SUM"], None) == H["MPI_ERR_COUNT"]
print("NOALLOC OK")
"""


def test_noalloc_entry_point_matches_reduce_local():
    if gpu_count() < 1:
        pytest.skip("needs a GPU")
    code = SCRIPT % {"root": ROOT, "mpi": os.path.join(LIB, "libmpi.so"), "cail": os.path.join(LIB, "libcail.so")}
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "NOALLOC OK" in r.stdout
    assert "exceed the limit" in r.stderr
