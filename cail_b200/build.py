"""Builds the native libraries in-tree (CMake + Ninja, sm_100a).

    python -m cail_b200.build            # build/ (CUDA + host-only libcail, minimpi, tests)
    python -m cail_b200.build --variant host-only --dir build-host

Device code is compiled with -gencode arch=compute_100a,code=sm_100a
-lineinfo; nvcc cross-compiles without a GPU.
"""
from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def build_native(build_dir: str = "build", options: dict | None = None, quiet: bool = True) -> str:
    """Configures (if needed) and builds the CMake project; returns the build dir."""
    bdir = build_dir if os.path.isabs(build_dir) else os.path.join(ROOT, build_dir)
    opts = {"CMAKE_BUILD_TYPE": "Release"}
    opts.update(options or {})
    gen = ["-G", "Ninja"] if shutil.which("ninja") else []
    cfg = ["cmake", "-S", ROOT, "-B", bdir, *gen] + [f"-D{k}={v}" for k, v in opts.items()]
    out = subprocess.DEVNULL if quiet else None
    subprocess.run(cfg, check=True, stdout=out)
    subprocess.run(["cmake", "--build", bdir, "-j", str(os.cpu_count() or 4)], check=True, stdout=out)
    return bdir


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--dir", default="build")
    ap.add_argument("--variant", choices=["cuda", "host-only"], default="cuda")
    ap.add_argument("-D", action="append", default=[], help="extra CMake cache entries KEY=VALUE")
    a = ap.parse_args()
    opts = dict(kv.split("=", 1) for kv in a.D)
    if a.variant == "host-only":
        opts["CAIL_HOST_PATH"] = "ON"
    print(build_native(a.dir, opts, quiet=False))


if __name__ == "__main__":
    sys.exit(main())
