"""Auto-dispatch policy of NVLink communicators, queried on CPU through
cail_nvlink_auto_algorithm() under different environments: the one-shot /
two-shot crossover and its overrides, NVLS only when asked for and only for
(type, op) pairs multimem can reduce, the copy-engine two-shot only above
CAIL_CE_MIN."""
import json
import os
import subprocess
import sys

import pytest

from conftest import LIB, ROOT

QUERY = r"""
import ctypes, json, sys
sys.path.insert(0, %r)
from cail_b200 import _lib
H = _lib.H
ctypes.CDLL(%r, mode=ctypes.RTLD_GLOBAL)
c = ctypes.CDLL(%r)
f = c.cail_nvlink_auto_algorithm
f.restype = ctypes.c_char_p
f.argtypes = [ctypes.c_int, ctypes.c_size_t, ctypes.c_int, ctypes.c_int]
out = []
for P, b, dt, op in json.loads(sys.argv[1]):
    r = f(P, b, H[dt], H[op])
    out.append(r.decode() if r else None)
print(json.dumps(out))
"""

KIB, MIB, GIB = 1 << 10, 1 << 20, 1 << 30


def query(cases, env=None):
    e = {k: v for k, v in os.environ.items() if not k.startswith("CAIL_")}
    e.update(env or {})
    code = QUERY % (ROOT, os.path.join(LIB, "libmpi.so"), os.path.join(LIB, "libcail.so"))
    r = subprocess.run([sys.executable, "-c", code, json.dumps(cases)], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_default_crossover_is_512_kib_and_two_shot_above():
    cases = [(8, 32 * KIB, "MPI_FLOAT", "MPI_SUM"), (8, 512 * KIB, "MPI_FLOAT", "MPI_SUM"),
             (8, 512 * KIB + 4, "MPI_FLOAT", "MPI_SUM"), (8, GIB, "MPI_FLOAT", "MPI_SUM"),
             (2, GIB, "MPI_DOUBLE", "MPI_MAX"), (4, 16 * MIB, "MPI_INT", "MPI_PROD")]
    assert query(cases) == ["one_shot", "one_shot", "two_shot", "two_shot", "two_shot", "two_shot"]


def test_unsupported_type_or_op_has_no_nvlink_algorithm():
    assert query([(8, MIB, "MPI_LONG_DOUBLE", "MPI_SUM"), (8, MIB, "MPI_FLOAT", "MPI_BAND")]) == [None, None]


def test_oneshot_max_and_small_threshold_move_the_crossover():
    cases = [(8, 64 * KIB, "MPI_FLOAT", "MPI_SUM"), (8, 64 * KIB + 4, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases, {"CAIL_ONESHOT_MAX": "65536"}) == ["one_shot", "two_shot"]
    # CAIL_MSG_SMALL_THRESHOLD keeps its reference meaning: below it is "small"
    cases = [(8, 256 * KIB - 4, "MPI_FLOAT", "MPI_SUM"), (8, 256 * KIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases, {"CAIL_MSG_SMALL_THRESHOLD": "262144"}) == ["one_shot", "two_shot"]


def test_nvls_only_when_requested_and_for_multimem_pairs():
    cases = [(8, 16 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 16 * MIB - 4, "MPI_FLOAT", "MPI_SUM"),
             (4, 16 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 16 * MIB, "MPI_FLOAT", "MPI_PROD"),
             (8, 16 * MIB, "MPI_INT8_T", "MPI_SUM"), (8, 16 * MIB, "MPI_FLOAT", "MPI_MAX"),
             (8, 16 * MIB, "MPI_INT", "MPI_MAX"), (8, 16 * MIB, "MPI_DOUBLE", "MPI_SUM")]
    assert query(cases) == ["two_shot"] * 8
    assert query(cases, {"CAIL_NVLS_MIN_RANKS": "8"}) == [
        "nvls", "two_shot", "two_shot", "two_shot", "two_shot", "two_shot", "nvls", "nvls"]
    assert query(cases[:1], {"CAIL_NVLS_MIN_RANKS": "8", "CAIL_NVLS": "0"}) == ["two_shot"]
    assert query(cases[:1], {"CAIL_NVLS_MIN_RANKS": "8", "CAIL_NVLS_MIN": str(64 * MIB)}) == ["two_shot"]


def test_copy_engine_two_shot_only_above_ce_min():
    cases = [(8, 64 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 32 * MIB, "MPI_FLOAT", "MPI_SUM"),
             (8, 256 * KIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases) == ["two_shot", "two_shot", "one_shot"]
    assert query(cases, {"CAIL_CE_MIN": str(64 * MIB)}) == ["ce_two_shot", "two_shot", "one_shot"]
