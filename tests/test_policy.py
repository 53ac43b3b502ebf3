"""Auto-dispatch policy of NVLink communicators, queried on CPU through
cail_nvlink_auto_algorithm() under different environments: the one-shot /
two-shot crossover and its overrides, NVLS only when asked for and only for
(type, op) pairs multimem can reduce, the copy-engine two-shot only above
CAIL_CE_MIN."""
import json
import os
import subprocess
import sys


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


def query(cases, env=None, stderr=None):
    e = {k: v for k, v in os.environ.items() if not k.startswith("CAIL_")}
    e.update(env or {})
    code = QUERY % (ROOT, os.path.join(LIB, "libmpi.so"), os.path.join(LIB, "libcail.so"))
    r = subprocess.run([sys.executable, "-c", code, json.dumps(cases)], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    if stderr is not None:
        stderr.append(r.stderr)
    return json.loads(r.stdout.strip().splitlines()[-1])


def test_default_crossover_per_rank_count_and_two_shot_above():
    # measured: one_shot up to 64 KiB at 2 and 4 ranks, up to 256 KiB at 8
    cases = [(8, 32 * KIB, "MPI_FLOAT", "MPI_SUM"), (8, 256 * KIB, "MPI_FLOAT", "MPI_SUM"),
             (8, 256 * KIB + 4, "MPI_FLOAT", "MPI_SUM"), (8, GIB - 4, "MPI_FLOAT", "MPI_SUM"),
             (2, 64 * KIB, "MPI_FLOAT", "MPI_SUM"), (2, 64 * KIB + 4, "MPI_FLOAT", "MPI_SUM"),
             (2, GIB, "MPI_DOUBLE", "MPI_MAX"), (4, 64 * KIB, "MPI_INT", "MPI_PROD"),
             (4, 256 * KIB, "MPI_INT", "MPI_PROD")]
    assert query(cases) == ["one_shot", "one_shot", "two_shot", "two_shot", "one_shot", "two_shot", "two_shot",
                            "one_shot", "two_shot"]


def test_unsupported_type_or_op_has_no_nvlink_algorithm():
    assert query([(8, MIB, "MPI_LONG_DOUBLE", "MPI_SUM"), (8, MIB, "MPI_FLOAT", "MPI_BAND")]) == [None, None]


def test_oneshot_max_and_small_threshold_move_the_crossover():
    cases = [(8, 64 * KIB, "MPI_FLOAT", "MPI_SUM"), (8, 64 * KIB + 4, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases, {"CAIL_ONESHOT_MAX": "65536"}) == ["one_shot", "two_shot"]
    # CAIL_MSG_SMALL_THRESHOLD keeps its reference meaning: below it is "small"
    cases = [(8, 256 * KIB - 4, "MPI_FLOAT", "MPI_SUM"), (8, 256 * KIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases, {"CAIL_MSG_SMALL_THRESHOLD": "262144"}) == ["one_shot", "two_shot"]


def test_nvls_from_8_ranks_and_1_gib_and_only_for_multimem_pairs():
    # built in (measured): NVLS from 8 ranks and 1 GiB, for the pairs multimem reduces
    big = [(8, GIB, "MPI_FLOAT", "MPI_SUM"), (8, GIB - 4, "MPI_FLOAT", "MPI_SUM"),
           (4, GIB, "MPI_FLOAT", "MPI_SUM"), (8, GIB, "MPI_FLOAT", "MPI_PROD"),
           (8, GIB, "MPI_INT8_T", "MPI_SUM"), (8, GIB, "MPI_FLOAT", "MPI_MAX"),
           (8, GIB, "MPI_INT", "MPI_MAX"), (8, GIB, "MPI_DOUBLE", "MPI_SUM")]
    assert query(big) == ["nvls", "two_shot", "two_shot", "two_shot", "two_shot", "two_shot", "nvls", "nvls"]
    assert query(big[:1], {"CAIL_NVLS": "0"}) == ["two_shot"]
    assert query(big[:1], {"CAIL_NVLS_MIN_RANKS": "0"}) == ["two_shot"]
    # the environment moves both bounds
    cases = [(8, 16 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 16 * MIB - 4, "MPI_FLOAT", "MPI_SUM"),
             (4, 16 * MIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases) == ["two_shot"] * 3
    assert query(cases, {"CAIL_NVLS_MIN": str(16 * MIB)}) == ["nvls", "two_shot", "two_shot"]
    assert query(cases, {"CAIL_NVLS_MIN": str(16 * MIB), "CAIL_NVLS_MIN_RANKS": "4"}) == ["nvls", "two_shot", "nvls"]


def test_copy_engine_two_shot_only_above_ce_min():
    cases = [(8, 64 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 32 * MIB, "MPI_FLOAT", "MPI_SUM"),
             (8, 256 * KIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases) == ["two_shot", "two_shot", "one_shot"]
    assert query(cases, {"CAIL_CE_MIN": str(64 * MIB)}) == ["ce_two_shot", "two_shot", "one_shot"]


TUNE = """# crossovers measured on this box
nranks=8 oneshot_max=256K nvls_min=64M
nranks=4 oneshot_max=1M ce_min=128M   # copy engines from 128 MiB
nranks=2 bogus=1
nranks=x oneshot_max=5
"""


def test_tune_file_sets_crossovers_per_rank_count(tmp_path):
    f = tmp_path / "cail.tune"
    f.write_text(TUNE)
    cases = [(8, 256 * KIB, "MPI_FLOAT", "MPI_SUM"), (8, 256 * KIB + 4, "MPI_FLOAT", "MPI_SUM"),
             (8, 64 * MIB, "MPI_FLOAT", "MPI_SUM"), (8, 32 * MIB, "MPI_FLOAT", "MPI_SUM"),
             (8, 64 * MIB, "MPI_FLOAT", "MPI_PROD"),
             (4, MIB, "MPI_FLOAT", "MPI_SUM"), (4, MIB + 4, "MPI_FLOAT", "MPI_SUM"),
             (4, 128 * MIB, "MPI_FLOAT", "MPI_SUM"),
             (2, 64 * KIB, "MPI_FLOAT", "MPI_SUM"), (2, MIB, "MPI_FLOAT", "MPI_SUM")]
    err = []
    got = query(cases, {"CAIL_TUNE_FILE": str(f)}, stderr=err)
    assert got == ["one_shot", "two_shot", "nvls", "two_shot", "two_shot",
                   "one_shot", "two_shot", "ce_two_shot",
                   "one_shot", "two_shot"]
    # the two malformed lines are reported with their numbers and ignored
    assert "line 4:" in err[0] and "line 5:" in err[0] and "[cail ERROR] CAIL_TUNE_FILE" in err[0]


def test_environment_overrides_the_tune_file(tmp_path):
    f = tmp_path / "cail.tune"
    f.write_text(TUNE)
    env = {"CAIL_TUNE_FILE": str(f), "CAIL_ONESHOT_MAX": "65536", "CAIL_CE_MIN": str(GIB)}
    cases = [(8, 128 * KIB, "MPI_FLOAT", "MPI_SUM"), (4, 128 * MIB, "MPI_FLOAT", "MPI_SUM")]
    assert query(cases, env) == ["two_shot", "two_shot"]


def test_missing_tune_file_is_reported():
    err = []
    assert query([(8, MIB, "MPI_FLOAT", "MPI_SUM")], {"CAIL_TUNE_FILE": "/nonexistent/cail.tune"},
                 stderr=err) == ["two_shot"]
    assert "[cail ERROR] cannot open CAIL_TUNE_FILE '/nonexistent/cail.tune'" in err[0]


# ---------------------------------------------------------------- cail_b200.tune analysis
def test_tune_analysis_places_crossovers_from_sweeps():
    from cail_b200 import tune

    # p50 (us) per size in the shape measured on 8 x B200: one_shot ahead up
    # to 512 KiB, two_shot ahead above; nvls only winning from 256 MiB on,
    # with one noisy loss at 64 MiB that must not count as "lasting"
    csv_one = "bytes,algo,p50_us\n" + "\n".join(f"{32768 << i},one_shot,{23 + 2.5 * i}" for i in range(9))
    csv_two = "bytes,algo,p50_us\n" + "\n".join(f"{32768 << i},two_shot,{30 + 0.8 * i}" for i in range(9))
    one, two = tune.parse_bench(csv_one), tune.parse_bench(csv_two)
    assert tune.last_win(one, two) == 32768 << 4
    big = [1 << 20, 1 << 24, 1 << 26, 1 << 28, 1 << 30]
    two_big = dict(zip(big, [40.0, 70.0, 200.0, 740.0, 3000.0]))
    nvls = dict(zip(big, [80.0, 60.0, 210.0, 700.0, 2500.0]))
    assert tune.first_lasting_win(nvls, two_big) == 1 << 28
    assert tune.tune_line(8, one, two, nvls, two_big) == "nranks=8 oneshot_max=524288 nvls_min=268435456"
    # never winning leaves the key out (the library keeps its default)
    assert tune.tune_line(2, two, one) == "nranks=2"


def test_info_tool_prints_the_policy_table(tmp_path):
    f = tmp_path / "cail.tune"
    f.write_text("nranks=8 oneshot_max=256K nvls_min=256M\n")
    e = {k: v for k, v in os.environ.items() if not k.startswith("CAIL_")}
    e["CAIL_TUNE_FILE"] = str(f)
    r = subprocess.run([sys.executable, "-m", "cail_b200.info", "--ranks", "2,8"], cwd=ROOT, env=e,
                       capture_output=True, text=True, timeout=120)
    assert r.returncode == 0, r.stderr
    lines = r.stdout.splitlines()
    assert lines[0].startswith("cail 0.1.0")
    assert f"CAIL_TUNE_FILE={f}" in r.stdout
    row2 = next(l for l in lines if l.startswith("2 ")).split()
    row8 = next(l for l in lines if l.startswith("8 ")).split()
    # columns: 32K 256K 512K 1M 16M 256M 1G
    assert row2[1:] == ["one_shot", "two_shot", "two_shot", "two_shot", "two_shot", "two_shot", "two_shot"]
    assert row8[1:] == ["one_shot", "one_shot", "two_shot", "two_shot", "two_shot", "nvls", "nvls"]
