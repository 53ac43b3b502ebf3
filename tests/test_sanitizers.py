"""The host path under AddressSanitizer (with leak detection) and
UndefinedBehaviorSanitizer: a host-only build of minimpi, the interposer
(linked in, as a link-time interposition) and the checks, compiled with
-fsanitize=address,undefined.  Every rank must end with no sanitizer report:
no invalid access, no undefined arithmetic (e.g. 16-bit products promoted to
signed int) and nothing left allocated after MPI_Finalize's teardown.  A
deliberately leaking rank shows the check works under the launcher."""
import os
import shutil
import subprocess

import pytest

from conftest import ROOT

ASAN = os.path.join(ROOT, "build-sanitize")
CC, CXX = "/usr/bin/gcc", "/usr/bin/g++"
ENV_ASAN = {"ASAN_OPTIONS": "detect_leaks=1:halt_on_error=1", "UBSAN_OPTIONS": "print_stacktrace=1"}

LEAK = r"""
#include <mpi.h>
#include <stdlib.h>
int main(int argc, char **argv) {
    MPI_Init(&argc, &argv);
    void *volatile p = malloc(12345);
    p = 0;
    MPI_Finalize();
    return 0;
}
"""


def _can_sanitize(tmp):
    if not (os.path.exists(CC) and os.path.exists(CXX) and shutil.which("cmake")):
        return False
    src = os.path.join(tmp, "probe.c")
    with open(src, "w") as f:
        f.write("int main(void) { return 0; }\n")
    r = subprocess.run([CC, "-fsanitize=address,undefined", src, "-o", os.path.join(tmp, "probe")],
                       capture_output=True)
    return r.returncode == 0


@pytest.fixture(scope="module")
def asan_build(tmp_path_factory):
    if not _can_sanitize(str(tmp_path_factory.mktemp("probe"))):
        pytest.skip("no AddressSanitizer runtime for the system compiler")
    if not os.path.exists(os.path.join(ASAN, "build.ninja")):
        r = subprocess.run(["cmake", "-S", ROOT, "-B", ASAN, "-G", "Ninja", "-DCAIL_HOST_PATH=ON",
                            "-DCAIL_SANITIZE=address,undefined", f"-DCMAKE_C_COMPILER={CC}",
                            f"-DCMAKE_CXX_COMPILER={CXX}"],
                           capture_output=True, text=True, timeout=300)
        assert r.returncode == 0, r.stdout + r.stderr
    r = subprocess.run(["cmake", "--build", ASAN, "--target", "mpi", "cail-mpirun", "cail_check_linked"],
                       capture_output=True, text=True, timeout=900)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    return ASAN


def _run(build, np, args, extra_env=None, timeout=600):
    env = dict(os.environ)
    for k in list(env):
        if k.startswith("CAIL_") or k == "LD_PRELOAD":
            env.pop(k)
    env.update(ENV_ASAN)
    env.update(extra_env or {})
    return subprocess.run([os.path.join(build, "bin", "cail-mpirun"), "-np", str(np)] + args, env=env,
                          capture_output=True, text=True, timeout=timeout)


@pytest.mark.parametrize("np,mode,extra", [
    (2, ["-m", "basic"], {}),
    (3, ["-m", "matrix", "-c", "1000", "-p"], {"CAIL_MIN_MSG_SIZE": "0"}),
    (4, ["-m", "edge"], {}),
    (2, ["-m", "config1"], {}),
    (5, ["-m", "matrix", "-c", "1003"], {"CAIL_MIN_MSG_SIZE": "0", "CAIL_ALGO": "rabenseifner"}),
    (6, ["-m", "matrix", "-c", "1003"], {"CAIL_MIN_MSG_SIZE": "0", "CAIL_ALGO": "ring"}),
])
def test_host_path_is_clean_under_sanitizers(asan_build, np, mode, extra):
    r = _run(asan_build, np, [os.path.join(asan_build, "bin", "cail_check_linked")] + mode, extra)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert ", 0 failed" in r.stdout
    assert "Sanitizer" not in out and "runtime error" not in out, out[-4000:]


def test_leak_check_catches_a_leaking_rank(asan_build, tmp_path):
    src = tmp_path / "leak.c"
    src.write_text(LEAK)
    exe = tmp_path / "leak"
    lib = os.path.join(asan_build, "lib")
    r = subprocess.run([CC, "-fsanitize=address,undefined", f"-I{os.path.join(ROOT, 'csrc', 'minimpi', 'include')}",
                        str(src),
                        "-o", str(exe), f"-L{lib}", "-lmpi", f"-Wl,-rpath,{lib}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = _run(asan_build, 2, [str(exe)], timeout=120)
    assert r.returncode != 0
    assert "LeakSanitizer: detected memory leaks" in r.stderr and "12345 byte" in r.stderr


@pytest.mark.parametrize("which", ["PROBE", "PROBE2"])
def test_minimpi_probes_are_clean_under_sanitizers(asan_build, tmp_path, which):
    # minimpi's point-to-point, non-blocking, collective and communicator code
    # under ASan + UBSan (the probe programs of test_minimpi.py)
    import test_minimpi

    src = tmp_path / "probe.c"
    src.write_text(getattr(test_minimpi, which))
    exe = tmp_path / "probe"
    lib = os.path.join(asan_build, "lib")
    r = subprocess.run([CC, "-O1", "-fsanitize=address,undefined",
                        f"-I{os.path.join(ROOT, 'csrc', 'minimpi', 'include')}", str(src), "-o", str(exe),
                        f"-L{lib}", "-lmpi", f"-Wl,-rpath,{lib}"], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    r = _run(asan_build, 3, [str(exe)], timeout=300)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert " OK p=3" in r.stdout
    assert "Sanitizer" not in out and "runtime error" not in out, out[-4000:]
