"""GPU tests (B200).  Single-GPU tests run everywhere a GPU exists; the
NVLink-kernel tests need two or more GPUs and skip otherwise.

Oracle: minimpi's PMPI_Allreduce, which folds in rank order exactly like
the one-shot and two-shot kernels, so their float results must match it
bit for bit (--bits); NVLS reduces inside the switch in an unspecified
order and is checked with a reassociation tolerance.
"""
import ctypes
import os
import re
import subprocess
import sys

import pytest

from conftest import LIB, ROOT, gpu_count, mpirun

pytestmark = pytest.mark.gpu


def ok(r):
    return r.returncode == 0 and ", 0 failed" in r.stdout


def need_gpus(n):
    if gpu_count() < n:
        pytest.skip(f"needs {n} GPUs")


# ---------------------------------------------------------------- one GPU
def test_smoke_entry():
    need_gpus(1)
    r = subprocess.run([sys.executable, "-c", "import __graft_entry__ as g; g.smoke()"], cwd=ROOT,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "smoke ok" in r.stdout


def test_device_pointer_detection_over_memory_kinds():
    # cudaMalloc and managed buffers take the device path, pinned host and
    # malloc'd buffers pass through to PMPI; all give the PMPI result
    need_gpus(1)
    r = mpirun(1, ["cail_check", "-m", "memkinds"], preload="cuda", timeout=300)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]


def test_canary_zones_catch_an_overrun_on_the_device():
    # the guard zones around device buffers are checked the same way
    need_gpus(1)
    r = mpirun(1, ["cail_check", "-m", "canary_selftest", "-d"], preload="cuda", timeout=300)
    assert r.returncode != 0
    assert "FAIL: canary zones intact after a deliberate one-byte overrun" in r.stdout


def test_call_keeps_the_callers_current_device():
    # a buffer on cuda:1 while cuda:0 is current: the call runs on GPU 1 and
    # hands GPU 0 back as the current device
    need_gpus(2)
    code = ("import cail_b200 as c, torch; torch.cuda.set_device(0); c.init();"
            "x = torch.full((1 << 18,), 3.0, device='cuda:1'); c.ops.allreduce_(x);"
            "torch.cuda.synchronize(1); d = torch.cuda.current_device();"
            "ok = bool((x == 3.0).all()); c.finalize(); print('device', d, 'ok', ok)")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "device 0 ok True" in r.stdout, r.stdout + r.stderr


def test_native_library_loaded_in_process():
    need_gpus(1)
    code = ("import cail_b200 as c, torch; c.init(); x=torch.ones(1<<20, device='cuda');"
            "c.ops.allreduce_(x); print(open('/proc/self/maps').read()); c.finalize()")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr
    assert os.path.join(LIB, "libcail.so") in r.stdout


@pytest.mark.parametrize("copy_max", ["0", "134217728"], ids=["bulk_copy", "copy_kernel"])
def test_single_rank_copy_all_types(copy_max):
    """One rank: the allreduce is dst = src (a copy kernel below
    CAIL_COPY_KERNEL_MAX, the TMA bulk copy above); every type and op,
    separate and in place, against PMPI bit for bit."""
    need_gpus(1)
    r = mpirun(1, ["cail_check", "-m", "matrix", "-c", "100003", "-d", "-p", "--bits"], preload="cuda",
               env={"CAIL_MIN_MSG_SIZE": "0", "CAIL_COPY_KERNEL_MAX": copy_max, "CAIL_STATS": "1"})
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
    assert "copy=" in r.stderr and " copy=0 " not in r.stderr


@pytest.mark.parametrize("algo", ["recursive_doubling", "ring", "rabenseifner", "auto"])
@pytest.mark.parametrize("np", [2, 3])
def test_p2p_algorithms_device_buffers_one_gpu(algo, np):
    """Several ranks on one GPU: no NVLink path (shared GPU), so the
    point-to-point algorithms run on device buffers over minimpi's CUDA-IPC
    transport, folding with the sm_100a local reduction kernel."""
    need_gpus(1)
    r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "4099", "-d", "-p"], preload="cuda",
               env={"CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0", "CUDA_VISIBLE_DEVICES": "0"}, timeout=900)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.parametrize("copy_max", ["0", "134217728"], ids=["bulk_copy", "copy_kernel"])
def test_single_rank_copy_unaligned_views(copy_max):
    """One rank, byte buffers whose views start a few bytes off a 16-byte
    boundary and have odd lengths: the copy's plain-load head and tail run;
    the output must equal the input byte for byte, and the bytes around the
    view must stay untouched."""
    need_gpus(1)
    code = ("import cail_b200 as c, torch; c.init();"
            "ok = True\n"
            "for off, n in ((3, 1000003), (13, 65), (5, 7), (1, (3 << 20) + 11)):\n"
            "    src = torch.randint(0, 256, (n + 64,), dtype=torch.uint8, device='cuda')\n"
            "    dst = torch.full((n + 64,), 7, dtype=torch.uint8, device='cuda')\n"
            "    c.ops.allreduce(src[off:off + n], dst[off:off + n], op='max')\n"
            "    torch.cuda.synchronize()\n"
            "    ok = ok and torch.equal(dst[off:off + n], src[off:off + n])\n"
            "    ok = ok and bool((dst[:off] == 7).all()) and bool((dst[off + n:] == 7).all())\n"
            "print('views ok', ok, c.last_algorithm()); c.finalize()")
    env = dict(os.environ, CAIL_COPY_KERNEL_MAX=copy_max, CAIL_MIN_MSG_SIZE="0")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600, env=env)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "views ok True copy" in r.stdout, r.stdout + r.stderr


@pytest.mark.parametrize("np", [2, 3])
def test_zero_copy_two_shot_with_ranks_sharing_one_gpu(np):
    """CAIL_TEST_SHARED_GPU=1: 2 and 3 ranks on one GPU take the zero-copy
    two-shot (the auto path above the one-shot crossover), whose kernels
    never wait on one another: cross-process IPC of the user buffers, the
    registration cache (64 rotating buffers, in place on every other call)
    and the P > 1 slicing, bit for bit against PMPI."""
    need_gpus(1)
    env = {"CAIL_TEST_SHARED_GPU": "1", "CAIL_MIN_MSG_SIZE": "0", "CUDA_VISIBLE_DEVICES": "0", "CAIL_STATS": "1",
           "CAIL_NVLS": "0"}
    r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "4099", "-d", "-p", "--bits"], preload="cuda", env=env,
               timeout=900)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
    calls = [int(n) for n in re.findall(r"(?<![a-z_])two_shot=(\d+)", r.stderr)]
    assert len(calls) == np and all(n > 0 for n in calls), r.stderr[-2000:]
    r = mpirun(np, ["cail_check", "-m", "stress", "-c", "300000", "-r", "200", "-b", "64", "-d", "--bits"],
               preload="cuda", env=env, timeout=900)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
    hits = [int(n) for n in re.findall(r"reg_hits=(\d+)", r.stderr)]
    assert len(hits) == np and all(n > 0 for n in hits), r.stderr[-2000:]


def test_device_wait_timeout_reports_status():
    """A one-shot kernel whose peer never arrives gives up after the limit
    and reports code 1; the context stays usable afterwards."""
    need_gpus(1)
    code = ("import ctypes, time, torch; torch.cuda.init(); "
            f"lib=ctypes.CDLL('{os.path.join(LIB, 'libmpi.so')}', mode=ctypes.RTLD_GLOBAL); "
            f"c=ctypes.CDLL('{os.path.join(LIB, 'libcail.so')}'); t=time.time(); "
            "rc=c.cail_test_device_timeout(300); dt=time.time()-t; "
            "x=torch.ones(4, device='cuda'); torch.cuda.synchronize(); print(rc, dt, float(x.sum()))")
    r = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=300)
    assert r.returncode == 0, r.stderr
    rc, dt, s = r.stdout.split()
    assert int(rc) == 1 and 0.25 < float(dt) < 30 and float(s) == 4.0


def test_reference_sm100a_build_runs_on_device_buffers():
    need_gpus(1)
    if not os.path.exists(os.path.join(ROOT, "baseline", "_ref", "lib", "libcail.so")):
        pytest.skip("reference baseline not built")
    r = mpirun(2, ["cail_check", "-m", "config1", "-d"], preload="ref-cuda",
               env={"CUDA_VISIBLE_DEVICES": "0"}, timeout=600)
    assert ok(r), r.stdout[-2000:] + r.stderr[-2000:]


# ---------------------------------------------------------------- NVLink kernels
def nranks():
    """Rank counts for the NVLink tests: 2, 4, 8 (those the box has GPUs for),
    or the comma-separated list in CAIL_TEST_NRANKS."""
    want = os.environ.get("CAIL_TEST_NRANKS")
    cand = [int(x) for x in want.split(",")] if want else [2, 4, 8]
    return [n for n in cand if n <= gpu_count()]


def algo_env(algo):
    """CAIL_ALGO for a test parameter.  Blocking two_shot calls run the
    zero-copy kernel by default: two_shot_zerocopy forces it
    (CAIL_TWOSHOT_ZEROCOPY=1) and two_shot_push forces the push kernel
    over the workspace (CAIL_TWOSHOT_ZEROCOPY=0)."""
    if algo == "two_shot_zerocopy":
        return {"CAIL_ALGO": "two_shot", "CAIL_TWOSHOT_ZEROCOPY": "1"}
    if algo == "two_shot_push":
        return {"CAIL_ALGO": "two_shot", "CAIL_TWOSHOT_ZEROCOPY": "0"}
    return {"CAIL_ALGO": algo}


@pytest.mark.multigpu
@pytest.mark.parametrize("algo", ["one_shot", "two_shot_push", "two_shot_zerocopy", "ce_two_shot"])
def test_nvlink_p2p_matrix_bit_exact(algo):
    # counts {1,2,3,4099,4100,4102}: heads, tails, fewer elements than ranks;
    # separate and in place; floats bit-identical to the rank-order oracle
    need_gpus(2)
    for np in nranks():
        r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "4099", "-d", "-p", "--bits"], preload="cuda",
                   env={**algo_env(algo), "CAIL_MIN_MSG_SIZE": "0"}, timeout=1200)
        assert ok(r), f"np={np}\n" + r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
@pytest.mark.parametrize("algo", ["auto", "nvls", "two_shot_push", "two_shot_zerocopy", "ce_two_shot", "one_shot"])
def test_nvlink_config3_coverage(algo):
    """20 datatypes x SUM/PROD/MAX/MIN at counts 1,000,003 and 4,194,304 at
    every available rank count; integers bit-exact, floats within
    reassociation tolerance (NVLS) or bit-exact (the P2P kernels).  Forced
    one_shot changes its piece between these sizes and element types, so
    its host barrier before a new slot layout runs many times."""
    need_gpus(2)
    for np in nranks():
        exact = "two_shot" in algo or algo == "one_shot"
        args = ["cail_check", "-m", "config3", "-d"] + (["--bits"] if exact else ["--tol", "1e-4"])
        r = mpirun(np, args, preload="cuda", env=algo_env(algo), timeout=1200)
        assert ok(r), f"np={np} algo={algo}\n" + r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
def test_nvlink_edge_and_config1():
    need_gpus(2)
    for np in nranks():
        r = mpirun(np, ["cail_check", "-m", "edge", "-d"], preload="cuda", timeout=600)
        assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
        r = mpirun(np, ["cail_check", "-m", "config1", "-d"], preload="cuda", timeout=600)
        assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
@pytest.mark.parametrize("algo", ["nvls", "two_shot_push", "two_shot_zerocopy", "one_shot"])
def test_large_ragged_and_unaligned_messages(algo):
    """Messages of 40 MiB plus a few bytes (not a multiple of 16 bytes), on
    buffers one or three elements off a 16-byte boundary, separate and in
    place.  With 64 KiB NVLS units every CTA refills its two staging slots
    while earlier units are still being copied out; the P2P kernels run many
    rounds.  Integers bit-exact, floats bit-exact on the P2P kernels and
    within reassociation tolerance on NVLS."""
    need_gpus(2)
    env = {**algo_env(algo), "CAIL_NVLS_UNIT": "65536"}
    exact = ["--tol", "1e-4"] if algo == "nvls" else ["--bits"]
    for np in nranks():
        r = mpirun(np, ["cail_check", "-m", "slots", "-d"] + exact, preload="cuda", env=env, timeout=900)
        assert ok(r), f"np={np} algo={algo}\n" + r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
def test_registration_cache_stress():
    need_gpus(2)
    np = nranks()[-1]
    for count in (4096, 32768, 1 << 20):
        r = mpirun(np, ["cail_check", "-m", "stress", "-c", str(count), "-r", "300", "-b", "64", "-d", "--bits"],
                   preload="cuda", env={"CAIL_STATS": "1", "CAIL_NVLS": "0"}, timeout=900)
        assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
def test_nan_and_inf_max_min_bit_identical_to_pmpi():
    """Float/double MAX and MIN over data holding NaN and +-Inf, one-shot and
    two-shot sizes, separate and in place: the rank-order fold of the NVLink
    kernels gives PMPI's result bit for bit."""
    need_gpus(2)
    for np in nranks():
        r = mpirun(np, ["cail_check", "-m", "nan", "-d"], preload="cuda", timeout=900)
        assert ok(r), f"np={np}\n" + r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
@pytest.mark.parametrize("algo", ["one_shot", "two_shot", "nvls"])
def test_stream_ordered_calls(algo):
    """CAIL_STREAM_ORDERED=1: one_shot, two_shot (the push kernel, which needs
    no host barrier) and nvls calls return once queued and the legacy stream
    waits for them; results read back through the legacy stream must be the
    rank-order oracle's (NVLS: within tolerance, the switch reassociates),
    also over 64 rotating buffers with in-place calls interleaved, so that
    successive calls reuse the workspace slots while earlier kernels may
    still run."""
    need_gpus(2)
    env = {"CAIL_ALGO": algo, "CAIL_MIN_MSG_SIZE": "0", "CAIL_STREAM_ORDERED": "1", "CAIL_STATS": "1"}
    exact = ["--bits"] if algo != "nvls" else ["--tol", "1e-4"]
    for np in nranks():
        r = mpirun(np, ["cail_check", "-m", "matrix", "-c", "4099", "-d", "-p"] + exact, preload="cuda",
                   env=env, timeout=900)
        assert ok(r), f"np={np}\n" + r.stdout[-3000:] + r.stderr[-3000:]
        r = mpirun(np, ["cail_check", "-m", "stress", "-c", "300000", "-r", "300", "-b", "64", "-d"] + exact,
                   preload="cuda", env=env, timeout=900)
        assert ok(r), f"np={np}\n" + r.stdout[-3000:] + r.stderr[-3000:]


@pytest.mark.multigpu
def test_two_shot_failure_on_one_rank_reaches_every_rank():
    """Zero-copy two-shot (CAIL_TWOSHOT_ZEROCOPY=1), the path with a host
    exchange: a failure injected on the host of rank 1 (its import of the peers'
    buffers fails, as a failing cudaIpcOpenMemHandle would) must end the
    two-shot call with an error on every rank: rank 1 still passes both host
    barriers with an error bit, so rank 0 neither waits forever nor returns
    a result whose slice 1 was never reduced.  No GPU fault is involved."""
    need_gpus(2)
    r = mpirun(2, ["cail_check", "-m", "expect_error", "-d"], preload="cuda",
               env={"CAIL_ALGO": "two_shot", "CAIL_TWOSHOT_ZEROCOPY": "1", "CAIL_FI_TWOSHOT_FAIL": "1",
                    "CAIL_NVLS": "0"}, timeout=300)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
    assert "injected import failure" in r.stderr
    assert "a peer failed during the call" in r.stderr


@pytest.mark.multigpu
def test_rank_leaving_between_steps_is_detected():
    need_gpus(2)
    r = mpirun(2, ["cail_check", "-m", "leave", "-d"], preload="cuda",
               env={"CAIL_NVLS": "0", "NCCL_NVLS_ENABLE": "0", "CAIL_DEVICE_TIMEOUT_MS": "1000"}, timeout=300)
    assert r.returncode == 0, r.stdout + r.stderr
    assert "LEAVE DETECTED at step 2" in r.stdout


@pytest.mark.multigpu
def test_host_barrier_wait_is_bounded():
    """Zero-copy two-shot with a peer that stalls on the host (alive, but 3 s
    late): the waiting rank returns an error after CAIL_HOST_TIMEOUT_MS, the
    late rank sees the error bit and returns at once, and the communicator
    refuses further calls.  No GPU is involved in the stall."""
    need_gpus(2)
    r = mpirun(2, ["cail_check", "-m", "stall", "-d"], preload="cuda",
               env={"CAIL_ALGO": "two_shot", "CAIL_TWOSHOT_ZEROCOPY": "1", "CAIL_HOST_TIMEOUT_MS": "1000",
                    "CAIL_NVLS": "0"}, timeout=300)
    assert ok(r), r.stdout[-3000:] + r.stderr[-3000:]
    assert "STALL DETECTED" in r.stdout
    assert "did not reach the arrive barrier" in r.stderr
