"""Data-parallel harness: bucketed gradient allreduce through the interposer
matches a single-process reference (CPU ranks; GPU variant marked gpu)."""
import os
import sys

import pytest

from conftest import ROOT, gpu_count, mpirun

WORKER = os.path.join(ROOT, "tests", "ddp_worker.py")


@pytest.fixture(scope="module")
def ext_built(build):
    from cail_b200.ops import ext

    ext.build()


@pytest.mark.parametrize("np", [2, 3])
def test_ddp_cpu_ranks(ext_built, np):
    r = mpirun(np, [sys.executable, WORKER, "cpu"], preload=None, timeout=600,
               env={"CAIL_MIN_MSG_SIZE": "0"})
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    assert f"DDP OK P={np}" in r.stdout


@pytest.mark.gpu
def test_ddp_gpu_ranks(ext_built):
    n = min(gpu_count(), 4)
    if n < 1:
        pytest.skip("needs a GPU")
    np = max(n, 2)
    env = {"CAIL_MIN_MSG_SIZE": "0"}
    if n < 2:
        env["CUDA_VISIBLE_DEVICES"] = "0"
    r = mpirun(np, [sys.executable, WORKER, "cuda"], preload=None, timeout=900, env=env)
    assert r.returncode == 0, r.stdout + r.stderr[-3000:]
    assert f"DDP OK P={np}" in r.stdout
