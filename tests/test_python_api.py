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
