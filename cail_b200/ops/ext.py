"""Builds (in-tree, under build/torch_ext) and loads the cail_torch extension."""
from __future__ import annotations

import ctypes
import os

from .. import _lib

_SRC = os.path.join(_lib.ROOT, "csrc", "torch_ext", "cail_torch.cpp")
_BUILD = os.path.join(_lib.BUILD, "torch_ext")
_mod = None


def build(verbose: bool = False):
    """Compiles the extension into build/torch_ext (no-op when up to date)."""
    from torch.utils.cpp_extension import load

    os.makedirs(_BUILD, exist_ok=True)
    return load(name="cail_torch", sources=[_SRC], build_directory=_BUILD, extra_cflags=["-O2"],
                verbose=verbose)


def get():
    """The loaded extension, wired to the interposer chosen by cail_b200.init()."""
    global _mod
    if _mod is None:
        libs = _lib.loaded()
        if libs is None:
            raise RuntimeError("cail_b200.init() must run before the extension is used")
        _mod = build()
        addr = ctypes.cast(libs.cail.MPI_Allreduce, ctypes.c_void_p).value
        _mod.set_allreduce(addr, _lib.H["MPI_IN_PLACE"])
    return _mod
