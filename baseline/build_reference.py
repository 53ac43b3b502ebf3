"""Builds the unmodified reference CAIL sources as the comparison baseline.

The reference (cornelisnetworks/cail) is a C/CUDA library built with
autotools; it has no Python packaging, so `pip install` of it fails with
"Neither 'setup.py' nor 'pyproject.toml' found", and autoreconf is not
available here.  This script copies its sources (a read-only checkout: --src,
else $CAIL_REFERENCE_SRC, else a `reference` directory beside this
repository) to baseline/_ref/src without
changing a byte, and compiles them the way its configure script would with

    --with-cuda --with-cuda-arch=sm_100a     -> baseline/_ref/lib/libcail.so
    --enable-host-path                       -> baseline/_ref/lib/libcail_host.so

against this repository's bundled MPI (minimpi, build/lib/libmpi.so), the
only MPI on these machines.  cudart is linked statically, as in cail-b200's
own build, so the library does not depend on which libcudart a host
process (e.g. PyTorch) has already loaded.

Usage:  python baseline/build_reference.py [--src DIR]
"""
import argparse
import glob
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
OUT = os.path.join(ROOT, "baseline", "_ref")
CUDA = os.environ.get("CUDA_HOME", "/usr/local/cuda")


def run(cmd):
    subprocess.run(cmd, check=True)


def build(src_root: str) -> None:
    if not os.path.isdir(os.path.join(src_root, "src", "core")):
        raise SystemExit(f"reference sources not found under {src_root}")
    src = os.path.join(OUT, "src")
    if os.path.isdir(src):
        shutil.rmtree(src)
    shutil.copytree(os.path.join(src_root, "src"), src)
    for f in ("README.md", "LICENSE", "configure.ac"):
        if os.path.exists(os.path.join(src_root, f)):
            shutil.copy(os.path.join(src_root, f), OUT)
    obj = os.path.join(OUT, "obj")
    lib = os.path.join(OUT, "lib")
    os.makedirs(obj, exist_ok=True)
    os.makedirs(lib, exist_ok=True)
    mpi_inc = os.path.join(ROOT, "csrc", "minimpi", "include")
    mpi_lib = os.path.join(ROOT, "build", "lib")
    if not os.path.exists(os.path.join(mpi_lib, "libmpi.so")):
        raise SystemExit("build/lib/libmpi.so missing: build cail-b200 first")
    defs = ["-DCAIL_ENABLE_RECURSIVE_DOUBLING=1", "-DCAIL_ENABLE_RING=1", "-DCAIL_ENABLE_RABENSEIFNER=1"]
    incs = [f"-I{mpi_inc}", f"-I{src}/core", f"-I{src}/gpu", f"-I{CUDA}/include"]
    common_c = sorted(glob.glob(f"{src}/core/*.c") + glob.glob(f"{src}/coll/allreduce/*.c"))

    def compile_c(files, extra, tag):
        objs = []
        for f in files:
            o = os.path.join(obj, tag + "_" + os.path.basename(f) + ".o")
            run(["gcc", "-O2", "-fPIC", "-w", *defs, *extra, *incs, "-c", f, "-o", o])
            objs.append(o)
        return objs

    # CUDA build (sm_100a)
    objs = compile_c(common_c + [f"{src}/gpu/cuda/cail_cuda_mem.c"], [], "cuda")
    cu = os.path.join(obj, "cuda_cail_cuda_reduce.o")
    run([f"{CUDA}/bin/nvcc", "-gencode", "arch=compute_100a,code=sm_100a", "-O2", "-Xcompiler", "-fPIC",
         *defs, *incs, "-c", f"{src}/gpu/cuda/cail_cuda_reduce.cu", "-o", cu])
    run(["g++", "-shared", "-o", os.path.join(lib, "libcail.so"), *objs, cu, f"-L{mpi_lib}", "-lmpi",
         f"-Wl,-rpath,{mpi_lib}", f"-L{CUDA}/lib64", "-lcudart_static", "-lrt", "-ldl", "-lpthread"])
    # host-path build
    objs = compile_c(common_c + [f"{src}/gpu/host/cail_host_reduce.c"], ["-DCAIL_HOST_PATH=1"], "host")
    run(["g++", "-shared", "-o", os.path.join(lib, "libcail_host.so"), *objs, f"-L{mpi_lib}", "-lmpi",
         f"-Wl,-rpath,{mpi_lib}"])
    with open(os.path.join(OUT, "BUILD_INFO.txt"), "w") as f:
        f.write(f"reference sources copied unmodified from {src_root}\n"
                "libcail.so: CUDA backend, nvcc -gencode arch=compute_100a,code=sm_100a\n"
                "libcail_host.so: --enable-host-path equivalent\n"
                "algorithms: recursive_doubling, ring, rabenseifner enabled\n")
    print(f"reference built into {lib}")


def main() -> None:
    ap = argparse.ArgumentParser()
    # this script is the one place that reads the reference checkout
    sibling = os.path.normpath(os.path.join(os.path.dirname(os.path.abspath(__file__)), "..", "..", "reference"))
    ap.add_argument("--src", default=os.environ.get("CAIL_REFERENCE_SRC", sibling))
    ap.add_argument("--if-present", action="store_true",
                    help="exit quietly when the reference sources are not there")
    a = ap.parse_args()
    if a.if_present and not os.path.isdir(os.path.join(a.src, "src")):
        print(f"reference sources not found at {a.src}; baseline not rebuilt")
        return
    build(a.src)


if __name__ == "__main__":
    sys.exit(main())
