"""Python side: handle table parsed from mpi.h, dtype/op mapping, tensor
allreduce through the host-only interposer on CPU ranks."""
import os
import subprocess
import sys

import pytest
import torch

from conftest import ROOT, mpirun


def test_handles_parsed_from_mpi_h():
    from cail_b200 import _lib

    h = _lib.H
    assert h["MPI_COMM_WORLD"] == 1 and h["MPI_FLOAT"] == 14 and h["MPI_SUM"] == 3
    assert h["MPI_IN_PLACE"] == -1
    assert len({h[k] for k in h if k.startswith("MPI_INT") and k.endswith("_T")}) == 4


def test_dtype_mapping():
    from cail_b200.ops import mpi_datatype, mpi_op
    from cail_b200 import _lib

    assert mpi_datatype(torch.float32) == _lib.H["MPI_FLOAT"]
    assert mpi_datatype(torch.float64) == _lib.H["MPI_DOUBLE"]
    assert mpi_datatype(torch.int64) == _lib.H["MPI_LONG_LONG"]
    assert mpi_op("max") == _lib.H["MPI_MAX"]
    with pytest.raises(TypeError):
        mpi_datatype(torch.bfloat16)


def test_tensor_api_rejects_bad_arguments_before_any_mpi_call():
    """Argument errors surface as Python exceptions before MPI is touched
    (no cail_b200.init() here): non-contiguous tensors, size or dtype
    mismatches, counts that do not fit MPI's int, and unknown operators."""
    from cail_b200.ops import allreduce, allreduce_, mpi_op

    with pytest.raises(ValueError, match="contiguous"):
        allreduce_(torch.zeros(4, 4).t())
    with pytest.raises(ValueError):
        allreduce(torch.zeros(4), torch.zeros(5))
    with pytest.raises(ValueError):
        allreduce(torch.zeros(8)[::2], torch.zeros(4))
    with pytest.raises(TypeError, match="dtypes differ"):
        allreduce(torch.zeros(4), torch.zeros(4, dtype=torch.float64))
    big = torch.empty(2**31, dtype=torch.int8, device="meta")  # 2^31 elements, nothing allocated
    with pytest.raises(ValueError, match="int"):
        allreduce_(big)
    with pytest.raises(KeyError):
        mpi_op("xor")


def test_handle_table_maps_23_datatypes_to_12_types_and_4_ops():
    """The interposer accepts the 20 documented datatypes plus the aliases
    MPI_SIGNED_CHAR, MPI_BYTE and MPI_LONG_LONG_INT, mapped onto 12 element
    types with the reference's enum values (src/core/cail_types.c:5-40);
    anything else, and operators other than SUM/PROD/MAX/MIN, is
    unsupported (-1) and passes through to PMPI."""
    import ctypes

    from conftest import LIB, ensure_build
    from cail_b200 import _lib

    ensure_build()
    ctypes.CDLL(os.path.join(LIB, "libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    c = ctypes.CDLL(os.path.join(LIB, "libcail_host.so"))
    H = _lib.H
    want = {  # handle -> (cail element type, bytes)
        "MPI_CHAR": (0, 1), "MPI_SIGNED_CHAR": (0, 1), "MPI_INT8_T": (0, 1),
        "MPI_UNSIGNED_CHAR": (6, 1), "MPI_BYTE": (6, 1), "MPI_UINT8_T": (6, 1),
        "MPI_SHORT": (10, 2), "MPI_INT16_T": (10, 2), "MPI_UNSIGNED_SHORT": (11, 2), "MPI_UINT16_T": (11, 2),
        "MPI_INT": (1, 4), "MPI_INT32_T": (1, 4), "MPI_UNSIGNED": (7, 4), "MPI_UINT32_T": (7, 4),
        "MPI_LONG": (2, 8), "MPI_UNSIGNED_LONG": (8, 8),
        "MPI_LONG_LONG": (5, 8), "MPI_LONG_LONG_INT": (5, 8), "MPI_INT64_T": (5, 8),
        "MPI_UNSIGNED_LONG_LONG": (9, 8), "MPI_UINT64_T": (9, 8),
        "MPI_FLOAT": (3, 4), "MPI_DOUBLE": (4, 8),
    }
    assert len(want) == 23
    for name, (dt, size) in want.items():
        assert c.cail_mpi_type_to_dtype(H[name]) == dt, name
        assert c.cail_type_size(dt) == size, name
    assert len({dt for dt, _ in want.values()}) == 12
    assert c.cail_mpi_type_to_dtype(H["MPI_LONG_DOUBLE"]) == -1
    for name, op in (("MPI_SUM", 0), ("MPI_PROD", 1), ("MPI_MAX", 2), ("MPI_MIN", 3), ("MPI_BAND", -1)):
        assert c.cail_mpi_op_to_optype(H[name]) == op, name


def test_stream_ordered_toggle_returns_previous_mode():
    code = ("import ctypes; ctypes.CDLL('build/lib/libmpi.so', mode=ctypes.RTLD_GLOBAL); "
            "c = ctypes.CDLL('build/lib/libcail.so'); "
            "print(c.cail_set_stream_ordered(1), c.cail_set_stream_ordered(0), c.cail_set_stream_ordered(0))")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    assert r.stdout.split() == ["0", "1", "0"]


SCRIPT = r"""
import os, sys, torch
sys.path.insert(0, %r)
import cail_b200 as cail
r = cail.init("ours", host=True)
P = cail.world_size()
x = torch.arange(100000, dtype=torch.float64) * (r + 1)
cail.ops.allreduce_(x)
assert torch.equal(x, torch.arange(100000, dtype=torch.float64) * (P * (P + 1) / 2))
y = torch.full((70000,), r, dtype=torch.int32)
z = torch.empty_like(y)
cail.ops.allreduce(y, z, op="max")
assert int(z.min()) == P - 1
s = cail.stats()
if r == 0:
    print("API OK", cail.last_algorithm(), s.calls, s.by_algo[3])
cail.finalize()
"""


@pytest.mark.parametrize("np", [1, 3])
def test_tensor_allreduce_cpu_ranks(tmp_path, np):
    p = tmp_path / "api.py"
    p.write_text(SCRIPT % ROOT)
    r = mpirun(np, [sys.executable, str(p)], preload=None, env={"CAIL_ALGO": "rabenseifner"})
    assert r.returncode == 0, r.stdout + r.stderr
    assert "API OK" in r.stdout
    if np > 1:
        assert "API OK rabenseifner 2 2" in r.stdout


def test_bench_reference_arm_reports_unavailable_without_build(tmp_path):
    # the reference arm must print its "unavailable" line (exit 0) when the
    # reference library is absent; simulated by pointing the loader elsewhere
    code = ("import sys, runpy; sys.argv=['bench.py','--impl','reference'];"
            "import cail_b200._lib as L; L.REF_LIB_DIR='/nonexistent';"
            f"runpy.run_path({os.path.join(ROOT, 'bench.py')!r}, run_name='__main__')")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    assert '"unavailable"' in r.stdout and '"impl": "reference"' in r.stdout


def test_max_min_nan_semantics_match_pmpi_reduce_local():
    """cail's reduction template (shared by the host backend and the device
    kernels) and minimpi's PMPI_Reduce_local agree bit for bit on MAX/MIN
    over NaN and +-Inf, in both operand orders."""
    import ctypes

    import numpy as np

    from cail_b200 import _lib

    mpi = ctypes.CDLL(os.path.join(ROOT, "build", "lib", "libmpi.so"), mode=ctypes.RTLD_GLOBAL)
    host = ctypes.CDLL(os.path.join(ROOT, "build", "lib", "libcail_host.so"))
    vals = [float("nan"), float("inf"), float("-inf"), 0.0, -0.0, 1.5, -2.25]
    a = np.array([x for x in vals for _ in vals], dtype=np.float32)
    b = np.array([y for _ in vals for y in vals], dtype=np.float32)
    # cail_types.h: dtype FLOAT = 3, DOUBLE = 4; op MAX = 2, MIN = 3
    for dt_np, cail_dt, mpi_dt in ((np.float32, 3, "MPI_FLOAT"), (np.float64, 4, "MPI_DOUBLE")):
        for cail_op, mpi_op in ((2, "MPI_MAX"), (3, "MPI_MIN")):
            for x, y in ((a, b), (b, a)):
                x, y = x.astype(dt_np), y.astype(dt_np)
                io1, io2 = y.copy(), y.copy()
                rc1 = host.cail_gpu_reduce_local(x.ctypes.data_as(ctypes.c_void_p), io1.ctypes.data_as(ctypes.c_void_p),
                                                 ctypes.c_size_t(len(x)), cail_dt, cail_op)
                rc2 = mpi.PMPI_Reduce_local(x.ctypes.data_as(ctypes.c_void_p), io2.ctypes.data_as(ctypes.c_void_p),
                                            len(x), _lib.H[mpi_dt], _lib.H[mpi_op])
                assert rc1 == 0 and rc2 == 0
                assert io1.tobytes() == io2.tobytes(), (mpi_dt, mpi_op)
