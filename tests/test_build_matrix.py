"""Algorithm compile-out switches (CMake CAIL_ENABLE_RING /
CAIL_ENABLE_RABENSEIFNER, the reference's configure --enable-ring /
--enable-rabenseifner, configure.ac:63-100 there).

A host-only build with ring and Rabenseifner compiled out:
* CAIL_ALGO=ring prints "[cail ERROR] CAIL_ALGO=ring forced but disabled at
  compile time, aborting" and the job aborts (cail_allreduce.c:112-117 there);
* in auto mode a large message, which would run Rabenseifner, warns
  "rabenseifner selected (...) but disabled at compile time, falling back to
  PMPI" and still gives PMPI's result;
* the algorithm that is built (recursive doubling) runs as before.
"""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

BUILD = os.path.join(ROOT, "build-noalgo")


@pytest.fixture(scope="module")
def noalgo_build():
    if not shutil.which("cmake"):
        pytest.skip("no cmake")
    if not os.path.exists(os.path.join(BUILD, "build.ninja")):
        gen = ["-G", "Ninja"] if shutil.which("ninja") else []
        r = subprocess.run(["cmake", "-S", ROOT, "-B", BUILD, *gen, "-DCAIL_HOST_PATH=ON", "-DCAIL_ENABLE_RING=OFF",
                            "-DCAIL_ENABLE_RABENSEIFNER=OFF"], capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
    r = subprocess.run(["cmake", "--build", BUILD, "--target", "mpi", "cail-mpirun", "cail_check_linked"],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return BUILD


def _run(np, args, env):
    e = {k: v for k, v in os.environ.items() if not k.startswith("CAIL_") and k != "LD_PRELOAD"}
    e.update(env)
    return subprocess.run([os.path.join(BUILD, "bin", "cail-mpirun"), "-np", str(np),
                           os.path.join(BUILD, "bin", "cail_check_linked")] + args, env=e, capture_output=True,
                          text=True, timeout=300)


def test_forced_compiled_out_algorithm_aborts(noalgo_build):
    r = _run(2, ["-m", "basic"], {"CAIL_ALGO": "ring"})
    assert r.returncode != 0
    assert "[cail ERROR] CAIL_ALGO=ring forced but disabled at compile time, aborting" in r.stderr


def test_auto_mode_falls_back_when_large_algorithm_is_compiled_out(noalgo_build):
    # config1 reduces 262144 floats (1 MiB, above the 256 KiB crossover)
    r = _run(2, ["-m", "config1"], {"CAIL_ALGO": "auto"})
    assert r.returncode == 0 and ", 0 failed" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
    assert "[cail WARN] rabenseifner selected (msg_size >= msg_small_threshold) but disabled at compile time" \
        in r.stderr


def test_built_algorithm_still_runs(noalgo_build):
    r = _run(3, ["-m", "matrix", "-c", "1003"], {"CAIL_ALGO": "recursive_doubling", "CAIL_MIN_MSG_SIZE": "0"})
    assert r.returncode == 0 and ", 0 failed" in r.stdout, r.stdout[-3000:] + r.stderr[-3000:]
    assert "disabled at compile time" not in r.stderr
