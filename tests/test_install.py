"""Installation, as the reference's `make install` provides it: headers,
libraries, the launcher and a pkg-config file (`cail.pc`) that a program
builds against."""
import os
import subprocess
import textwrap

from conftest import BUILD, ensure_build

PROGRAM = textwrap.dedent("""
    #include <stdio.h>
    #include <cail.h>
    int main(void) {
        printf("version %s\\n", cail_version());
        return 0;
    }
""")


def test_install_and_build_against_pkg_config(tmp_path):
    ensure_build()
    prefix = tmp_path / "prefix"
    r = subprocess.run(["cmake", "--install", BUILD, "--prefix", str(prefix)], capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    for rel in ("include/cail.h", "include/mpi.h", "include/cail_noalloc.h", "lib/libcail.so",
                "lib/libcail_host.so", "lib/libmpi.so", "bin/cail-mpirun", "lib/pkgconfig/cail.pc"):
        assert (prefix / rel).exists(), rel
    env = dict(os.environ, PKG_CONFIG_PATH=str(prefix / "lib" / "pkgconfig"))
    flags = subprocess.run(["pkg-config", "--cflags", "--libs", "cail"], env=env, capture_output=True, text=True)
    assert flags.returncode == 0, flags.stderr
    words = flags.stdout.split()
    assert "-lcail" in words
    assert any(w.startswith("-I") and os.path.realpath(w[2:]) == os.path.realpath(prefix / "include") for w in words)
    assert any(w.startswith("-L") and os.path.realpath(w[2:]) == os.path.realpath(prefix / "lib") for w in words)
    src = tmp_path / "use_cail.c"
    src.write_text(PROGRAM)
    exe = tmp_path / "use_cail"
    cc = subprocess.run(["gcc", str(src), "-o", str(exe)] + words + ["-lmpi"], capture_output=True, text=True)
    assert cc.returncode == 0, cc.stderr
    run = subprocess.run([str(exe)], env=dict(os.environ, LD_LIBRARY_PATH=str(prefix / "lib")),
                         capture_output=True, text=True, timeout=60)
    assert run.returncode == 0, run.stderr
    assert run.stdout.startswith("version 0.1.0"), run.stdout
