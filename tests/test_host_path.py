"""The interposer's contract on CPU ranks (host-only build): algorithms,
dispatch table, fallbacks, logging and environment parsing.  Mirrors the
reference's make-check programs (tests/test_allreduce_{basic,correctness,edge}.c
there, run at -np 4, 3, 1 by tests/test_runner.sh) with PMPI_Allreduce as
the oracle for seeded, position-dependent inputs."""
import os
import re

import pytest

from conftest import mpirun

ALGOS = ["recursive_doubling", "ring", "rabenseifner"]


def ok(r):
    return r.returncode == 0 and ", 0 failed" in r.stdout


@pytest.mark.parametrize("np", [1, 3, 4])
def test_basic(np):
    r = mpirun(np, ["cail_check", "-m", "basic"])
    assert ok(r), r.stdout + r.stderr


@pytest.mark.parametrize("algo", ALGOS + ["auto"])
@pytest.mark.parametrize("np", [1, 2, 3, 4, 5, 8])
def test_matrix_all_types_ops(algo, np):
    # 20 datatypes x 4 ops x {separate, in place} x counts {1,2,3,1000,1001,1003};
    # CAIL_MIN_MSG_SIZE=0 so every call runs a cail algorithm
    r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "1000", "-p"],
               env={"CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r), r.stdout[-2000:] + r.stderr[-2000:]


@pytest.mark.parametrize("np", [2, 4, 7])
def test_matrix_large_counts(np):
    r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "100003"], env={"CAIL_ALGO": "rabenseifner"})
    assert ok(r), r.stdout[-2000:]


@pytest.mark.parametrize("np", [1, 2, 3, 4])
def test_edge_cases(np):
    r = mpirun(np, ["cail_check", "-m", "edge"])
    assert ok(r), r.stdout + r.stderr


@pytest.mark.parametrize("np", [2, 3])
def test_large_ragged_and_unaligned_messages_host(np):
    # the host algorithms on the same ragged / off-boundary cases the NVLink
    # test runs (2 MiB + 12 bytes of floats here, to keep the CPU run short)
    r = mpirun(np, ["cail_check", "-m", "slots", "-c", "524291", "--tol", "1e-4"])
    assert ok(r), r.stdout + r.stderr


@pytest.mark.parametrize("algo", ALGOS)
def test_config1_host_only(algo):
    """Host-only build, np=2: FLOAT SUM 262144 uniform[-1,1) seeded seed+rank and
    INT MAX 65536 uniform [-1000,1000]; each algorithm, in place and separate;
    checked against PMPI_Allreduce; min-msg-size fallback at count 1024."""
    r = mpirun(2, ["cail_check", "-m", "config1"], env={"CAIL_ALGO": algo, "CAIL_DEBUG": "1"})
    assert ok(r), r.stdout + r.stderr
    assert f"algorithm={algo} (forced)" in r.stderr
    assert "falling back to PMPI_Allreduce: msg_size=4096 < min_msg_size=32768" in r.stderr


def test_min_msg_size_zero_disables_passthrough():
    r = mpirun(2, ["cail_check", "-m", "config1"], env={"CAIL_MIN_MSG_SIZE": "0", "CAIL_DEBUG": "1"})
    assert ok(r), r.stdout + r.stderr
    assert "min_msg_size" not in r.stderr.split("initialized:")[-1].replace("min_msg_size=0", "")


def test_link_time_interposition():
    # cail_check_linked links -lcail_host before -lmpi (no LD_PRELOAD)
    r = mpirun(2, ["cail_check_linked", "-m", "config1"], preload=None, env={"CAIL_DEBUG": "1"})
    assert ok(r), r.stdout + r.stderr
    assert "[cail] initialized:" in r.stderr


def test_without_interposer_is_plain_mpi():
    r = mpirun(2, ["cail_check", "-m", "basic"], preload=None, env={"CAIL_DEBUG": "1"})
    assert ok(r)
    assert "[cail]" not in r.stderr


# ---------------------------------------------------------------- dispatch table
def algos_used(stderr):
    return re.findall(r"algorithm=(\w+) \(([^)]*)\)", stderr)


@pytest.mark.parametrize("np,count,expect", [
    (4, 1000, "recursive_doubling"),      # 4000 B < 256 KiB
    (4, 200000, "rabenseifner"),          # 800 KB >= 256 KiB
    (3, 65536, "rabenseifner"),           # exactly 256 KiB
    (3, 65535, "recursive_doubling"),
])
def test_auto_dispatch(np, count, expect):
    r = mpirun(np, ["cail_check", "-m", "basic", "-c", str(count)],
               env={"CAIL_DEBUG": "1", "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r), r.stderr
    used = algos_used(r.stderr)
    assert used and all(a == expect for a, _ in used), used


def test_count_below_pof2_uses_small_algorithm():
    r = mpirun(5, ["cail_check", "-m", "basic", "-c", "3"],
               env={"CAIL_DEBUG": "1", "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r)
    assert ("recursive_doubling", "count < pof2") in algos_used(r.stderr)


def test_small_threshold_env():
    r = mpirun(2, ["cail_check", "-m", "basic", "-c", "20000"],
               env={"CAIL_DEBUG": "1", "CAIL_MSG_SMALL_THRESHOLD": "4096"})
    assert ok(r)
    assert all(a == "rabenseifner" for a, _ in algos_used(r.stderr))


def test_non_pof2_threshold_halving_at_17_ranks():
    # P=17 (not a power of two, >= 16): the threshold is halved to 128 KiB,
    # so a 160 KB message runs Rabenseifner; at P=8 it runs recursive doubling
    r17 = mpirun(17, ["cail_check", "-m", "basic", "-c", "40000"], env={"CAIL_DEBUG": "1"}, timeout=600)
    assert ok(r17), r17.stdout[-1000:] + r17.stderr[-1000:]
    assert all(a == "rabenseifner" for a, _ in algos_used(r17.stderr))
    r8 = mpirun(8, ["cail_check", "-m", "basic", "-c", "40000"], env={"CAIL_DEBUG": "1"})
    assert ok(r8)
    assert all(a == "recursive_doubling" for a, _ in algos_used(r8.stderr))


def test_forced_rabenseifner_count_below_pof2_warns():
    r = mpirun(4, ["cail_check", "-m", "basic", "-c", "3"],
               env={"CAIL_ALGO": "rabenseifner", "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r)
    assert "[cail WARN] forced rabenseifner but count=3 < pof2=4, falling back to PMPI" in r.stderr


def test_ring_count_below_nprocs_warns():
    r = mpirun(4, ["cail_check", "-m", "basic", "-c", "3"], env={"CAIL_ALGO": "ring", "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r)
    assert "ring: count=3 < nprocs=4, cannot distribute chunks, falling back to PMPI" in r.stderr


@pytest.mark.parametrize("algo", ["one_shot", "two_shot", "nvls", "ce_two_shot"])
def test_forced_device_algorithm_on_host_build_warns(algo):
    # the NVLink algorithms exist only in the CUDA build: the host-only build
    # names the forced algorithm, warns and forwards to PMPI_Allreduce
    r = mpirun(2, ["cail_check", "-m", "basic"], env={"CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r), r.stdout + r.stderr
    assert f"[cail WARN] forced {algo} needs the CUDA build, falling back to PMPI" in r.stderr


def test_nvtx_ranges_are_harmless_without_a_profiler():
    # CAIL_NVTX=1 wraps every call of the CUDA build in an NVTX range; with no
    # profiler attached the calls are no-ops (host buffers: passthrough here)
    r = mpirun(2, ["cail_check", "-m", "basic"], preload="cuda", env={"CAIL_NVTX": "1"})
    assert ok(r), r.stdout + r.stderr


def test_canary_zones_catch_an_overrun():
    # every cail_check buffer sits between guard zones checked after each
    # call; the self-test overruns one buffer by a byte and must fail
    r = mpirun(2, ["cail_check", "-m", "canary_selftest"])
    assert r.returncode != 0
    assert "FAIL: canary zones intact after a deliberate one-byte overrun" in r.stdout
    assert "canary byte after the buffer overwritten" in r.stderr


# ---------------------------------------------------------------- logging / env
def test_unsupported_type_warns_and_warn_zero_silences():
    r = mpirun(2, ["cail_check", "-m", "edge"])
    assert ok(r)
    assert "[cail WARN] falling back to PMPI_Allreduce: unsupported type=UNKNOWN" in r.stderr
    assert "[cail WARN] falling back to PMPI_Allreduce: unsupported op=UNKNOWN" in r.stderr
    r = mpirun(2, ["cail_check", "-m", "edge"], env={"CAIL_WARN": "0"})
    assert ok(r)
    assert "[cail WARN]" not in r.stderr


@pytest.mark.parametrize("var,val,msg", [
    ("CAIL_MSG_SMALL_THRESHOLD", "abc", "[cail ERROR] invalid CAIL_MSG_SMALL_THRESHOLD='abc', using default"),
    ("CAIL_MSG_SMALL_THRESHOLD", "0", "[cail ERROR] invalid CAIL_MSG_SMALL_THRESHOLD='0', using default"),
    ("CAIL_MIN_MSG_SIZE", "-1", "[cail ERROR] invalid CAIL_MIN_MSG_SIZE='-1', using default"),
    ("CAIL_MIN_MSG_SIZE", "12k", "[cail ERROR] invalid CAIL_MIN_MSG_SIZE='12k', using default"),
    ("CAIL_NPROCS_THRESHOLD", "0", "[cail ERROR] invalid CAIL_NPROCS_THRESHOLD='0', using default"),
    ("CAIL_NPROCS_THRESHOLD", "99999999999", "[cail ERROR] invalid CAIL_NPROCS_THRESHOLD='99999999999', using default"),
    ("CAIL_ALGO", "fastest", "[cail ERROR] unknown CAIL_ALGO='fastest', using auto"),
])
def test_env_parse_errors(var, val, msg):
    r = mpirun(1, ["cail_check", "-m", "basic", "-c", "10000"], env={var: val, "CAIL_DEBUG": "1"})
    assert ok(r)
    assert msg in r.stderr
    assert "min_msg_size=32768 msg_small_threshold=262144 nprocs_threshold=4" in r.stderr


@pytest.mark.parametrize("val,on", [("1", True), ("yes", True), ("0", False), ("", False), ("0x", False)])
def test_debug_flag_rules(val, on):
    r = mpirun(1, ["cail_check", "-m", "basic", "-c", "10"], env={"CAIL_DEBUG": val})
    assert ok(r)
    assert ("[cail] initialized:" in r.stderr) == on


def test_leading_zero_values_parse():
    r = mpirun(1, ["cail_check", "-m", "basic", "-c", "10"],
               env={"CAIL_DEBUG": "1", "CAIL_MIN_MSG_SIZE": "0100", "CAIL_MSG_SMALL_THRESHOLD": "00512"})
    assert ok(r)
    assert "min_msg_size=100 msg_small_threshold=512" in r.stderr


def test_stats_dump():
    r = mpirun(2, ["cail_check", "-m", "config1"], env={"CAIL_STATS": "1", "CAIL_ALGO": "ring"})
    assert ok(r)
    m = re.search(r"\[cail\] stats: calls=(\d+) passthrough=(\d+) rd=\d+ ring=(\d+)", r.stderr)
    assert m and int(m.group(3)) == 4 and int(m.group(2)) >= 1


@pytest.mark.parametrize("algo", ["recursive_doubling", "ring", "rabenseifner"])
def test_dispatch_error_falls_back_to_pmpi(algo):
    """An algorithm that fails (here its scratch request, injected with
    CAIL_FI_SCRATCH_FAIL=1) makes the shim retry through PMPI_Allreduce
    (the reference's cail_pmpi.c:73-77): every result still matches PMPI."""
    r = mpirun(2, ["cail_check", "-m", "basic"],
               env={"CAIL_FI_SCRATCH_FAIL": "1", "CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0", "CAIL_DEBUG": "1"})
    assert ok(r), r.stdout + r.stderr
    assert "injected by CAIL_FI_SCRATCH_FAIL" in r.stderr
    assert "falling back to PMPI" in r.stderr


def test_scratch_cache_only_grows():
    """The point-to-point algorithms' scratch buffer is reallocated only when
    a request exceeds it and is otherwise reused (the reference's grow-only
    cache, src/core/cail_buf.c:28-69): over the matrix's rising and falling
    sizes, the allocations each rank logs only grow, and every reuse serves
    a request no larger than the cached size."""
    r = mpirun(2, ["cail_check", "-m", "matrix", "-c", "1000"],
               env={"CAIL_DEBUG": "1", "CAIL_ALGO": "recursive_doubling", "CAIL_MIN_MSG_SIZE": "0"})
    assert ok(r), r.stdout + r.stderr
    allocs = [int(n) for n in re.findall(r"buf: allocated (\d+) bytes", r.stderr)]
    reuses = [(int(c), int(q)) for c, q in re.findall(r"buf: reusing cached (\d+) bytes \(requested (\d+)\)", r.stderr)]
    assert allocs and reuses
    # both ranks log the same rising sequence, interleaved: never a decrease
    assert all(a <= b for a, b in zip(allocs, allocs[1:])), allocs
    assert len(allocs) <= 2 * len(set(allocs))
    assert all(q <= c for c, q in reuses)
    assert len(reuses) > len(allocs)


def test_trace_file(tmp_path):
    path = tmp_path / "trace.csv"
    r = mpirun(2, ["cail_check", "-m", "config1"], env={"CAIL_TRACE": str(path), "CAIL_ALGO": "rabenseifner"})
    assert ok(r)
    lines = path.read_text().strip().splitlines()
    assert any(line.startswith("rabenseifner,1048576,262144,FLOAT,SUM,2,") for line in lines)
