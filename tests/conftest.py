"""Shared fixtures: the in-tree build and a launcher for MPI jobs.

Tests marked ``gpu`` need a CUDA device; everything else runs on CPU ranks
(minimpi processes with host buffers and the host-only libcail).
"""
import os
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path.insert(0, ROOT)
BUILD = os.path.join(ROOT, "build")
LIB = os.path.join(BUILD, "lib")
BIN = os.path.join(BUILD, "bin")


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA GPU (B200)")
    config.addinivalue_line("markers", "multigpu: needs two or more GPUs")


_built = {"done": False}


def _stale():
    """True when a native artefact is missing or older than a source file."""
    outs = [os.path.join(LIB, n) for n in ("libmpi.so", "libcail.so", "libcail_host.so")]
    outs += [os.path.join(BIN, n) for n in ("cail-mpirun", "cail_check", "cail_check_linked", "cail_copier_check")]
    if not all(os.path.exists(p) for p in outs):
        return True
    oldest = min(os.path.getmtime(p) for p in outs)
    for d, _, files in os.walk(os.path.join(ROOT, "csrc")):
        for f in files:
            if os.path.getmtime(os.path.join(d, f)) > oldest:
                return True
    return False


def ensure_build():
    if _built["done"]:
        return
    if _stale():
        from cail_b200.build import build_native

        build_native("build")
    _built["done"] = True


@pytest.fixture(scope="session")
def build():
    ensure_build()
    return BUILD


def mpirun(np, args, env=None, preload="host", timeout=240, launcher_timeout=None):
    """Runs `cail-mpirun -np np <args>`; preload: "host", "cuda", "ref-host",
    "ref-cuda" or None (no interposer)."""
    ensure_build()
    e = dict(os.environ)
    e.pop("CAIL_ALGO", None)
    e.update({k: str(v) for k, v in (env or {}).items()})
    pre = {
        "host": os.path.join(LIB, "libcail_host.so"),
        "cuda": os.path.join(LIB, "libcail.so"),
        "ref-host": os.path.join(ROOT, "baseline", "_ref", "lib", "libcail_host.so"),
        "ref-cuda": os.path.join(ROOT, "baseline", "_ref", "lib", "libcail.so"),
        None: None,
    }[preload]
    if pre:
        e["LD_PRELOAD"] = pre
    else:
        e.pop("LD_PRELOAD", None)
    cmd = [os.path.join(BIN, "cail-mpirun"), "-np", str(np)]
    if launcher_timeout:
        cmd += ["--timeout", str(launcher_timeout)]
    if args and not os.path.isabs(args[0]):
        args = [os.path.join(BIN, args[0])] + list(args[1:])
    cmd += list(args)
    return subprocess.run(cmd, env=e, capture_output=True, text=True, timeout=timeout)


def gpu_count():
    try:
        import torch

        return torch.cuda.device_count() if torch.cuda.is_available() else 0
    except Exception:
        return 0


@pytest.fixture
def ngpus():
    return gpu_count()
