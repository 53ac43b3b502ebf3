"""minimpi, the bundled MPI: launcher, point-to-point, collectives,
communicators, attributes and host-side fault injection (CPU ranks)."""
import os
import subprocess

import pytest

from conftest import BIN, LIB, ROOT, mpirun

PROBE = r"""
#include <mpi.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
static int deleted = 0;
static int del_cb(MPI_Comm c, int k, void *v, void *x) { (void)c; (void)k; (void)x; deleted += *(int *)v; return MPI_SUCCESS; }
int main(int argc, char **argv) {
    MPI_Init(&argc, &argv);
    int r, p, bad = 0;
    MPI_Comm_rank(MPI_COMM_WORLD, &r);
    MPI_Comm_size(MPI_COMM_WORLD, &p);
    /* ring Sendrecv with a large host message (streams through the rings) */
    int n = 3 << 20;
    int *a = malloc(n * sizeof(int)), *b = malloc(n * sizeof(int));
    for (int i = 0; i < n; i++) a[i] = r * 1000003 + i;
    MPI_Status st;
    MPI_Sendrecv(a, n, MPI_INT, (r + 1) % p, 5, b, n, MPI_INT, (r + p - 1) % p, 5, MPI_COMM_WORLD, &st);
    int left = (r + p - 1) % p, cnt = -1;
    MPI_Get_count(&st, MPI_INT, &cnt);
    for (int i = 0; i < n; i += 4099) bad |= b[i] != left * 1000003 + i;
    bad |= st.MPI_SOURCE != left || st.MPI_TAG != 5 || cnt != n;
    /* tag matching out of order + ANY_SOURCE */
    if (p > 1) {
        if (r == 0) {
            int x = -1, y = -1;
            MPI_Recv(&y, 1, MPI_INT, 1, 22, MPI_COMM_WORLD, MPI_STATUS_IGNORE);
            MPI_Recv(&x, 1, MPI_INT, MPI_ANY_SOURCE, 11, MPI_COMM_WORLD, &st);
            bad |= x != 11 || y != 22 || st.MPI_SOURCE != 1;
        } else if (r == 1) {
            int x = 11, y = 22;
            MPI_Send(&x, 1, MPI_INT, 0, 11, MPI_COMM_WORLD);
            MPI_Send(&y, 1, MPI_INT, 0, 22, MPI_COMM_WORLD);
        }
    }
    /* bcast / reduce / gather / allgather */
    double v = r == p - 1 ? 42.5 : 0;
    MPI_Bcast(&v, 1, MPI_DOUBLE, p - 1, MPI_COMM_WORLD);
    bad |= v != 42.5;
    long long s = r, tot = -1;
    MPI_Reduce(&s, &tot, 1, MPI_LONG_LONG, MPI_SUM, 0, MPI_COMM_WORLD);
    if (r == 0) bad |= tot != (long long)p * (p - 1) / 2;
    int *all = malloc(p * sizeof(int));
    MPI_Allgather(&r, 1, MPI_INT, all, 1, MPI_INT, MPI_COMM_WORLD);
    for (int q = 0; q < p; q++) bad |= all[q] != q;
    /* split + attributes with delete callback on free */
    MPI_Comm sub;
    MPI_Comm_split(MPI_COMM_WORLD, r % 2, p - r, &sub);
    int sr, ss, kv, one = 1, mx = 0;
    MPI_Comm_rank(sub, &sr);
    MPI_Comm_size(sub, &ss);
    MPI_Allreduce(&r, &mx, 1, MPI_INT, MPI_MAX, sub);
    bad |= mx != ((p - 1) % 2 == r % 2 ? p - 1 : p - 2);
    MPI_Comm_create_keyval(MPI_COMM_NULL_COPY_FN, del_cb, &kv, NULL);
    MPI_Comm_set_attr(sub, kv, &one);
    void *got; int flag;
    MPI_Comm_get_attr(sub, kv, &got, &flag);
    bad |= !flag || got != &one;
    MPI_Comm_free(&sub);
    bad |= deleted != 1;
    /* reduce_local and derived contiguous types */
    int x[4] = {1, 2, 3, 4}, y[4] = {10, 20, 30, 40};
    MPI_Datatype two;
    MPI_Type_contiguous(2, MPI_INT, &two);
    MPI_Type_commit(&two);
    MPI_Reduce_local(x, y, 2, two, MPI_PROD);
    bad |= y[3] != 160;
    int sz; MPI_Type_size(two, &sz); bad |= sz != 8;
    MPI_Type_free(&two);
    int any = 0;
    MPI_Allreduce(&bad, &any, 1, MPI_INT, MPI_LOR, MPI_COMM_WORLD);
    if (r == 0) printf("minimpi probe %s p=%d\n", any ? "FAIL" : "OK", p);
    free(a); free(b); free(all);
    MPI_Finalize();
    return any;
}
"""


@pytest.fixture(scope="module")
def probe(build, tmp_path_factory):
    d = tmp_path_factory.mktemp("mpi")
    src = d / "probe.c"
    src.write_text(PROBE)
    exe = d / "probe"
    inc = os.path.join(ROOT, "csrc", "minimpi", "include")
    subprocess.run(["gcc", "-O1", f"-I{inc}", str(src), "-o", str(exe), f"-L{LIB}", "-lmpi",
                    f"-Wl,-rpath,{LIB}"], check=True)
    return str(exe)


@pytest.mark.parametrize("np", [1, 2, 3, 4, 8])
def test_minimpi_probe(probe, np):
    r = mpirun(np, [probe], preload=None)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"minimpi probe OK p={np}" in r.stdout


def test_singleton_init(probe):
    env = {k: v for k, v in os.environ.items() if not k.startswith("CMPI_")}
    env.pop("RANK", None)
    env.pop("WORLD_SIZE", None)
    r = subprocess.run([probe], capture_output=True, text=True, env=env, timeout=60)
    assert r.returncode == 0 and "p=1" in r.stdout


def test_weak_mpi_strong_pmpi_symbols(build):
    out = subprocess.run(["nm", "-D", os.path.join(LIB, "libmpi.so")], capture_output=True, text=True).stdout
    syms = {line.split()[-1]: line.split()[-2] for line in out.splitlines() if len(line.split()) >= 2}
    for name in ("Allreduce", "Send", "Recv", "Sendrecv", "Reduce_local", "Comm_test_inter", "Finalize"):
        assert syms.get("PMPI_" + name) == "T", name
        assert syms.get("MPI_" + name) == "W", name


def test_launcher_propagates_failure(probe):
    r = mpirun(3, [probe], preload=None, env={"CMPI_FI_RANK": "1", "CMPI_FI_AT_CALL": "1",
                                               "CMPI_FI_ACTION": "exit", "CMPI_FI_EXIT_CODE": "7"})
    assert r.returncode == 7
    assert "fault injection: exit(7)" in r.stderr


def test_hung_rank_is_detected_by_timeout(probe):
    # rank 2 stalls before its first call; the others' waits time out with a
    # clean error instead of hanging (ERRORS_ARE_FATAL -> job abort)
    r = mpirun(3, [probe], preload=None, timeout=120,
               env={"CMPI_FI_RANK": "2", "CMPI_FI_ACTION": "hang", "CMPI_FI_HANG_S": "20",
                    "CMPI_TIMEOUT_S": "2"})
    assert r.returncode != 0
    assert "timed out" in r.stderr


def test_dropped_message_is_detected(probe):
    r = mpirun(2, [probe], preload=None, timeout=120,
               env={"CMPI_FI_RANK": "0", "CMPI_FI_AT_CALL": "1", "CMPI_FI_ACTION": "drop",
                    "CMPI_TIMEOUT_S": "2"})
    assert r.returncode != 0
    assert "timed out" in r.stderr


def test_launcher_timeout(probe):
    r = mpirun(2, [probe], preload=None, timeout=120, launcher_timeout=3,
               env={"CMPI_FI_RANK": "1", "CMPI_FI_ACTION": "hang", "CMPI_FI_HANG_S": "30"})
    assert r.returncode == 124


def test_dead_peer_detected(probe):
    # rank 1 exits without MPI_Finalize at its 2nd MPI call; rank 0 notices the
    # dead process through the liveness check (no timeout configured)
    r = mpirun(2, [probe], preload=None, timeout=120,
               env={"CMPI_FI_RANK": "1", "CMPI_FI_AT_CALL": "2", "CMPI_FI_ACTION": "exit",
                    "CMPI_FI_EXIT_CODE": "0"})
    assert r.returncode != 0
    assert "exited without MPI_Finalize" in r.stderr


PROBE2 = r"""
#include <mpi.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
int main(int argc, char **argv) {
    int flag = -1, provided = -1, bad = 0;
    MPI_Initialized(&flag);
    bad |= flag != 0;
    MPI_Init_thread(&argc, &argv, MPI_THREAD_FUNNELED, &provided);
    MPI_Initialized(&flag);
    bad |= flag != 1 || provided < MPI_THREAD_SINGLE;
    int q = -1;
    MPI_Query_thread(&q);
    bad |= q != provided;
    int r, p;
    MPI_Comm_rank(MPI_COMM_WORLD, &r);
    MPI_Comm_size(MPI_COMM_WORLD, &p);
    /* non-blocking ring in both directions, completed with Waitall */
    int n = 1 << 18;
    int *s0 = malloc(n * sizeof(int)), *s1 = malloc(n * sizeof(int));
    int *r0 = malloc(n * sizeof(int)), *r1 = malloc(n * sizeof(int));
    for (int i = 0; i < n; i++) { s0[i] = r * 7 + i; s1[i] = -(r * 7 + i); }
    int right = (r + 1) % p, left = (r + p - 1) % p;
    MPI_Request req[4];
    MPI_Status sts[4];
    MPI_Irecv(r0, n, MPI_INT, left, 1, MPI_COMM_WORLD, &req[0]);
    MPI_Irecv(r1, n, MPI_INT, right, 2, MPI_COMM_WORLD, &req[1]);
    MPI_Isend(s0, n, MPI_INT, right, 1, MPI_COMM_WORLD, &req[2]);
    MPI_Isend(s1, n, MPI_INT, left, 2, MPI_COMM_WORLD, &req[3]);
    MPI_Waitall(4, req, sts);
    for (int i = 0; i < n; i += 997) bad |= r0[i] != left * 7 + i || r1[i] != -(right * 7 + i);
    bad |= sts[0].MPI_SOURCE != left || sts[1].MPI_SOURCE != right;
    for (int i = 0; i < 4; i++) bad |= req[i] != MPI_REQUEST_NULL;
    /* Test until complete, then Wait on the nulled request */
    int tok = r, got = -1, done = 0;
    MPI_Request a, b;
    MPI_Irecv(&got, 1, MPI_INT, left, 3, MPI_COMM_WORLD, &a);
    MPI_Isend(&tok, 1, MPI_INT, right, 3, MPI_COMM_WORLD, &b);
    while (!done) MPI_Test(&a, &done, MPI_STATUS_IGNORE);
    MPI_Wait(&b, MPI_STATUS_IGNORE);
    bad |= got != left;
    /* gather to a non-zero root on a duplicated communicator */
    MPI_Comm dup;
    MPI_Comm_dup(MPI_COMM_WORLD, &dup);
    int root = p - 1, *all = malloc(p * sizeof(int));
    int mine = 100 + r;
    MPI_Gather(&mine, 1, MPI_INT, all, 1, MPI_INT, root, dup);
    if (r == root) for (int i = 0; i < p; i++) bad |= all[i] != 100 + i;
    MPI_Comm_free(&dup);
    /* extents, error strings, clocks, processor name */
    MPI_Datatype three;
    MPI_Type_contiguous(3, MPI_DOUBLE, &three);
    MPI_Type_commit(&three);
    MPI_Aint lb = -1, ext = -1;
    MPI_Type_get_extent(three, &lb, &ext);
    bad |= lb != 0 || ext != 24;
    MPI_Type_free(&three);
    char msg[MPI_MAX_ERROR_STRING];
    int len = 0;
    MPI_Error_string(MPI_ERR_COUNT, msg, &len);
    bad |= len <= 0 || (int)strlen(msg) != len;
    double t0 = MPI_Wtime(), t1 = MPI_Wtime();
    bad |= t1 < t0 || MPI_Wtick() <= 0.0;
    char host[MPI_MAX_PROCESSOR_NAME];
    MPI_Get_processor_name(host, &len);
    bad |= len <= 0;
    int any = 0;
    MPI_Allreduce(&bad, &any, 1, MPI_INT, MPI_LOR, MPI_COMM_WORLD);
    MPI_Finalized(&flag);
    any |= flag != 0;
    if (r == 0) printf("minimpi probe2 %s p=%d\n", any ? "FAIL" : "OK", p);
    free(s0); free(s1); free(r0); free(r1); free(all);
    MPI_Finalize();
    MPI_Finalized(&flag);
    if (r == 0 && flag != 1) printf("Finalized flag not set\n");
    return any || flag != 1;
}
"""


@pytest.fixture(scope="module")
def probe2(build, tmp_path_factory):
    d = tmp_path_factory.mktemp("mpi2")
    src = d / "probe2.c"
    src.write_text(PROBE2)
    exe = d / "probe2"
    inc = os.path.join(ROOT, "csrc", "minimpi", "include")
    subprocess.run(["gcc", "-O1", f"-I{inc}", str(src), "-o", str(exe), f"-L{LIB}", "-lmpi",
                    f"-Wl,-rpath,{LIB}"], check=True)
    return str(exe)


@pytest.mark.parametrize("np", [1, 2, 3, 5])
def test_minimpi_nonblocking_gather_dup_and_queries(probe2, np):
    r = subprocess.run([os.path.join(BIN, "cail-mpirun"), "-np", str(np), probe2], capture_output=True,
                       text=True, timeout=120)
    assert r.returncode == 0, r.stdout + r.stderr
    assert f"minimpi probe2 OK p={np}" in r.stdout
