// cmpi_api.cpp — the MPI_/PMPI_ entry points of minimpi.
//
// Every routine is defined as PMPI_x and exported under MPI_x as a weak
// alias (see the pragma list at the end), the arrangement the MPI profiling
// interface prescribes.  Internal code never calls through these symbols, so
// an interposer that overrides MPI_x (or PMPI_x) cannot recurse into itself.
#include "cmpi_internal.h"

#include <unistd.h>

#include <algorithm>
#include <cstdlib>

namespace cmpi {
int comm_copy_attrs(MPI_Comm src, MPI_Comm dst);
}

using namespace cmpi;

namespace {
int g_initialized = 0;
int g_finalized = 0;
int g_thread_level = MPI_THREAD_SINGLE;

#define CHECK_INIT() \
    do { if (!g_initialized || g_finalized) return MPI_ERR_OTHER; } while (0)

inline int fail(MPI_Comm c, int rc, const char *where) { return comm_errhandler_apply(c, rc, where); }

inline int type_bytes(MPI_Datatype dt, int count, uint64_t *bytes) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    if (count < 0) return MPI_ERR_COUNT;
    *bytes = (uint64_t)ti->size * (uint64_t)count;
    return MPI_SUCCESS;
}

int comm_rank_of_world(const Comm *c, int w) {
    for (int i = 0; i < c->size; ++i)
        if (c->world[i] == w) return i;
    return w;
}

void fix_status_source(const Comm *c, MPI_Status *st) {
    if (st && st->MPI_SOURCE >= 0) st->MPI_SOURCE = comm_rank_of_world(c, st->MPI_SOURCE);
}
}  // namespace

extern "C" {

// ------------------------------------------------------------------ init / finalize
int PMPI_Init_thread(int *argc, char ***argv, int required, int *provided) {
    (void)argc;
    (void)argv;
    if (g_initialized) return MPI_ERR_OTHER;
    int wr = 0, ws = 1;
    int rc = init_transport(&wr, &ws);
    if (rc != MPI_SUCCESS) return rc;
    std::vector<int> all(ws);
    for (int i = 0; i < ws; ++i) all[i] = i;
    MPI_Comm w = MPI_COMM_WORLD, s = MPI_COMM_SELF;
    comm_create(all, wr, 0, &w);
    comm_create(std::vector<int>{wr}, 0, 2, &s);
    g_thread_level = std::min(required, (int)MPI_THREAD_SERIALIZED);
    if (provided) *provided = g_thread_level;
    g_initialized = 1;
    return MPI_SUCCESS;
}

int PMPI_Init(int *argc, char ***argv) {
    int provided;
    return PMPI_Init_thread(argc, argv, MPI_THREAD_SINGLE, &provided);
}

int PMPI_Initialized(int *flag) { *flag = g_initialized; return MPI_SUCCESS; }
int PMPI_Finalized(int *flag) { *flag = g_finalized; return MPI_SUCCESS; }
int PMPI_Query_thread(int *provided) { *provided = g_thread_level; return MPI_SUCCESS; }

int PMPI_Finalize(void) {
    CHECK_INIT();
    Comm *w = comm_get(MPI_COMM_WORLD);
    int rc = w ? coll_barrier(w) : MPI_SUCCESS;
    comm_finalize_all();
    cuda_finalize();
    finalize_transport();
    g_finalized = 1;
    return rc;
}

int PMPI_Abort(MPI_Comm comm, int errorcode) {
    (void)comm;
    std::fprintf(stderr, "[minimpi] rank %d: MPI_Abort(errorcode=%d)\n", g_world_rank, errorcode);
    std::fflush(stdout);
    std::fflush(stderr);
    request_abort(errorcode);
    _exit(errorcode ? errorcode : 1);
}

double PMPI_Wtime(void) { return now_s(); }
double PMPI_Wtick(void) { return 1e-9; }

int PMPI_Get_processor_name(char *name, int *len) {
    gethostname(name, MPI_MAX_PROCESSOR_NAME - 1);
    name[MPI_MAX_PROCESSOR_NAME - 1] = 0;
    *len = (int)strlen(name);
    return MPI_SUCCESS;
}

int PMPI_Get_library_version(char *version, int *len) {
    const char *v = "minimpi 1.0 (cail-b200 bundled single-node MPI subset)";
    strncpy(version, v, MPI_MAX_LIBRARY_VERSION_STRING - 1);
    version[MPI_MAX_LIBRARY_VERSION_STRING - 1] = 0;
    *len = (int)strlen(version);
    return MPI_SUCCESS;
}

int PMPI_Error_string(int code, char *s, int *len) {
    snprintf(s, MPI_MAX_ERROR_STRING, "minimpi error %d", code);
    *len = (int)strlen(s);
    return MPI_SUCCESS;
}

// ------------------------------------------------------------------ communicators
int PMPI_Comm_rank(MPI_Comm comm, int *rank) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    *rank = c->rank;
    return MPI_SUCCESS;
}

int PMPI_Comm_size(MPI_Comm comm, int *size) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    *size = c->size;
    return MPI_SUCCESS;
}

int PMPI_Comm_test_inter(MPI_Comm comm, int *flag) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    *flag = c->test_inter ? 1 : 0;
    return MPI_SUCCESS;
}

int MPIX_Comm_set_test_inter(MPI_Comm comm, int flag) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    c->test_inter = flag != 0;
    return MPI_SUCCESS;
}

unsigned long long MPIX_Node_id(void) { return (unsigned long long)node_id(); }

int PMPI_Comm_split(MPI_Comm comm, int color, int key, MPI_Comm *newcomm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Comm_split");
    std::vector<int> mine = {color, key}, all(2 * c->size);
    int rc = coll_allgather_bytes(mine.data(), 2 * sizeof(int), all.data(), c);
    int ctx = 0;
    if (rc == MPI_SUCCESS) rc = comm_alloc_ctx(c, &ctx);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Comm_split");
    if (color == MPI_UNDEFINED) { *newcomm = MPI_COMM_NULL; return MPI_SUCCESS; }
    std::vector<std::pair<std::pair<int, int>, int>> members;  // ((key, parent rank), world)
    for (int q = 0; q < c->size; ++q)
        if (all[2 * q] == color) members.push_back({{all[2 * q + 1], q}, c->world[q]});
    std::sort(members.begin(), members.end());
    std::vector<int> world;
    int myrank = 0;
    for (size_t i = 0; i < members.size(); ++i) {
        if (members[i].first.second == c->rank) myrank = (int)i;
        world.push_back(members[i].second);
    }
    MPI_Comm out = MPI_COMM_NULL;
    comm_create(world, myrank, ctx, &out);
    *newcomm = out;
    return MPI_SUCCESS;
}

int PMPI_Comm_dup(MPI_Comm comm, MPI_Comm *newcomm) {
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Comm_dup");
    int rc = PMPI_Comm_split(comm, 0, c->rank, newcomm);
    if (rc == MPI_SUCCESS) {
        comm_get(*newcomm)->errh = c->errh;
        rc = comm_copy_attrs(comm, *newcomm);
    }
    return rc;
}

int PMPI_Comm_free(MPI_Comm *comm) { return comm_free(comm); }

int PMPI_Comm_set_errhandler(MPI_Comm comm, MPI_Errhandler eh) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    if (eh != MPI_ERRORS_RETURN && eh != MPI_ERRORS_ARE_FATAL) return MPI_ERR_ARG;
    c->errh = eh;
    return MPI_SUCCESS;
}

// ------------------------------------------------------------------ datatypes
int PMPI_Type_size(MPI_Datatype dt, int *size) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    *size = ti->size;
    return MPI_SUCCESS;
}

int PMPI_Type_get_extent(MPI_Datatype dt, MPI_Aint *lb, MPI_Aint *extent) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    *lb = 0;
    *extent = ti->size;
    return MPI_SUCCESS;
}

int PMPI_Type_contiguous(int count, MPI_Datatype old, MPI_Datatype *out) {
    return type_new_contiguous(count, old, out);
}

int PMPI_Type_commit(MPI_Datatype *dt) { return type_info(*dt) ? MPI_SUCCESS : MPI_ERR_TYPE; }
int PMPI_Type_free(MPI_Datatype *dt) { return type_free(dt); }

int PMPI_Get_count(const MPI_Status *st, MPI_Datatype dt, int *count) {
    const TypeInfo *ti = type_info(dt);
    if (!ti || !st) return MPI_ERR_TYPE;
    if (ti->size == 0) { *count = 0; return MPI_SUCCESS; }
    *count = st->nbytes % ti->size ? MPI_UNDEFINED : (int)(st->nbytes / ti->size);
    return MPI_SUCCESS;
}

// ------------------------------------------------------------------ point to point
int PMPI_Isend(const void *buf, int count, MPI_Datatype dt, int dest, int tag, MPI_Comm comm,
               MPI_Request *req) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Isend");
    uint64_t bytes;
    int rc = type_bytes(dt, count, &bytes);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Isend");
    int wd = comm_world_rank(c, dest);
    if (wd == -100) return fail(comm, MPI_ERR_RANK, "MPI_Isend");
    if (tag < 0) return fail(comm, MPI_ERR_TAG, "MPI_Isend");
    Request *r;
    rc = isend(buf, bytes, wd, tag, c->ctx, &r);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Isend");
    *req = req_to_handle(r);
    return MPI_SUCCESS;
}

int PMPI_Irecv(void *buf, int count, MPI_Datatype dt, int src, int tag, MPI_Comm comm,
               MPI_Request *req) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Irecv");
    uint64_t bytes;
    int rc = type_bytes(dt, count, &bytes);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Irecv");
    int ws = comm_world_rank(c, src);
    if (ws == -100) return fail(comm, MPI_ERR_RANK, "MPI_Irecv");
    Request *r;
    rc = irecv(buf, bytes, ws, tag, c->ctx, &r);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Irecv");
    *req = req_to_handle(r);
    return MPI_SUCCESS;
}

int PMPI_Wait(MPI_Request *req, MPI_Status *st) {
    if (!req || *req == MPI_REQUEST_NULL) return MPI_SUCCESS;
    Request *r = handle_to_req(*req);
    if (!r) return MPI_ERR_REQUEST;
    int rc = wait(r, st);
    handle_release(*req);
    *req = MPI_REQUEST_NULL;
    return fail(MPI_COMM_WORLD, rc, "MPI_Wait");
}

int PMPI_Waitall(int n, MPI_Request reqs[], MPI_Status sts[]) {
    int first = MPI_SUCCESS;
    for (int i = 0; i < n; ++i) {
        int rc = PMPI_Wait(&reqs[i], sts ? &sts[i] : nullptr);
        if (rc != MPI_SUCCESS && first == MPI_SUCCESS) first = rc;
    }
    return first;
}

int PMPI_Test(MPI_Request *req, int *flag, MPI_Status *st) {
    if (!req || *req == MPI_REQUEST_NULL) { *flag = 1; return MPI_SUCCESS; }
    Request *r = handle_to_req(*req);
    if (!r) return MPI_ERR_REQUEST;
    *flag = test(r) ? 1 : 0;
    if (*flag) return PMPI_Wait(req, st);
    return MPI_SUCCESS;
}

int PMPI_Send(const void *buf, int count, MPI_Datatype dt, int dest, int tag, MPI_Comm comm) {
    MPI_Request r;
    int rc = PMPI_Isend(buf, count, dt, dest, tag, comm, &r);
    if (rc != MPI_SUCCESS) return rc;
    Request *q = handle_to_req(r);
    rc = wait(q, nullptr);
    handle_release(r);
    return fail(comm, rc, "MPI_Send");
}

int PMPI_Recv(void *buf, int count, MPI_Datatype dt, int src, int tag, MPI_Comm comm,
              MPI_Status *st) {
    MPI_Request r;
    int rc = PMPI_Irecv(buf, count, dt, src, tag, comm, &r);
    if (rc != MPI_SUCCESS) return rc;
    Request *q = handle_to_req(r);
    rc = wait(q, st);
    handle_release(r);
    fix_status_source(comm_get(comm), st);
    return fail(comm, rc, "MPI_Recv");
}

int PMPI_Sendrecv(const void *sbuf, int scount, MPI_Datatype stype, int dest, int stag, void *rbuf,
                  int rcount, MPI_Datatype rtype, int src, int rtag, MPI_Comm comm, MPI_Status *st) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Sendrecv");
    uint64_t sb, rb;
    int rc = type_bytes(stype, scount, &sb);
    if (rc == MPI_SUCCESS) rc = type_bytes(rtype, rcount, &rb);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Sendrecv");
    int wd = comm_world_rank(c, dest), ws = comm_world_rank(c, src);
    if (wd == -100 || ws == -100) return fail(comm, MPI_ERR_RANK, "MPI_Sendrecv");
    Request *q[2];
    rc = irecv(rbuf, rb, ws, rtag, c->ctx, &q[1]);
    if (rc == MPI_SUCCESS) rc = isend(sbuf, sb, wd, stag, c->ctx, &q[0]);
    if (rc != MPI_SUCCESS) return fail(comm, rc, "MPI_Sendrecv");
    MPI_Status sts[2];
    rc = waitall(2, q, sts);
    if (st) { *st = sts[1]; fix_status_source(c, st); }
    return fail(comm, rc, "MPI_Sendrecv");
}

// ------------------------------------------------------------------ collectives
int PMPI_Barrier(MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Barrier");
    return fail(comm, coll_barrier(c), "MPI_Barrier");
}

int PMPI_Bcast(void *buf, int count, MPI_Datatype dt, int root, MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Bcast");
    uint64_t bytes;
    int rc = type_bytes(dt, count, &bytes);
    if (rc == MPI_SUCCESS && (root < 0 || root >= c->size)) rc = MPI_ERR_ROOT;
    if (rc == MPI_SUCCESS) rc = coll_bcast(buf, bytes, root, c);
    return fail(comm, rc, "MPI_Bcast");
}

int PMPI_Allreduce(const void *sendbuf, void *recvbuf, int count, MPI_Datatype dt, MPI_Op op,
                   MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Allreduce");
    if (!op_valid(op)) return fail(comm, MPI_ERR_OP, "MPI_Allreduce");
    return fail(comm, coll_allreduce(sendbuf, recvbuf, count, dt, op, c), "MPI_Allreduce");
}

int PMPI_Reduce(const void *sendbuf, void *recvbuf, int count, MPI_Datatype dt, MPI_Op op,
                int root, MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Reduce");
    if (!op_valid(op)) return fail(comm, MPI_ERR_OP, "MPI_Reduce");
    if (root < 0 || root >= c->size) return fail(comm, MPI_ERR_ROOT, "MPI_Reduce");
    return fail(comm, coll_reduce(sendbuf, recvbuf, count, dt, op, root, c), "MPI_Reduce");
}

int PMPI_Reduce_local(const void *inbuf, void *inoutbuf, int count, MPI_Datatype dt, MPI_Op op) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    if (count < 0) return MPI_ERR_COUNT;
    if (!op_valid(op)) return MPI_ERR_OP;
    long long n = (long long)count * ti->base_count;
    uint64_t bytes = (uint64_t)count * (uint64_t)ti->size;
    int oi = -1, oo = -1;
    bool din = bytes && is_device_ptr(inbuf, &oi), dout = bytes && is_device_ptr(inoutbuf, &oo);
    if (!din && !dout) return reduce_host(inbuf, inoutbuf, n, ti->kind, op);
    // Device operands: stage through host memory.
    std::vector<char> a(bytes), b(bytes);
    int rc = din ? cuda_copy(a.data(), inbuf, bytes, oi) : (memcpy(a.data(), inbuf, bytes), MPI_SUCCESS);
    if (rc == MPI_SUCCESS)
        rc = dout ? cuda_copy(b.data(), inoutbuf, bytes, oo) : (memcpy(b.data(), inoutbuf, bytes), MPI_SUCCESS);
    if (rc == MPI_SUCCESS) rc = reduce_host(a.data(), b.data(), n, ti->kind, op);
    if (rc == MPI_SUCCESS)
        rc = dout ? cuda_copy(inoutbuf, b.data(), bytes, oo) : (memcpy(inoutbuf, b.data(), bytes), MPI_SUCCESS);
    return rc;
}

int PMPI_Allgather(const void *sendbuf, int scount, MPI_Datatype stype, void *recvbuf, int rcount,
                   MPI_Datatype rtype, MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Allgather");
    uint64_t rb;
    int rc = type_bytes(rtype, rcount, &rb);
    if (rc == MPI_SUCCESS && sendbuf != MPI_IN_PLACE) {
        uint64_t sb;
        rc = type_bytes(stype, scount, &sb);
        if (rc == MPI_SUCCESS && sb != rb) rc = MPI_ERR_TRUNCATE;
    }
    if (rc == MPI_SUCCESS) rc = coll_allgather_bytes(sendbuf, rb, recvbuf, c);
    return fail(comm, rc, "MPI_Allgather");
}

int PMPI_Gather(const void *sendbuf, int scount, MPI_Datatype stype, void *recvbuf, int rcount,
                MPI_Datatype rtype, int root, MPI_Comm comm) {
    CHECK_INIT();
    note_call();
    Comm *c = comm_get(comm);
    if (!c) return fail(comm, MPI_ERR_COMM, "MPI_Gather");
    uint64_t sb = 0;
    int rc = MPI_SUCCESS;
    if (c->rank == root) rc = type_bytes(rtype, rcount, &sb);
    else rc = type_bytes(stype, scount, &sb);
    if (rc == MPI_SUCCESS) rc = coll_gather_bytes(sendbuf, sb, recvbuf, root, c);
    return fail(comm, rc, "MPI_Gather");
}

}  // extern "C"

// ------------------------------------------------------------------ weak MPI_ aliases
#pragma weak MPI_Init = PMPI_Init
#pragma weak MPI_Init_thread = PMPI_Init_thread
#pragma weak MPI_Initialized = PMPI_Initialized
#pragma weak MPI_Finalized = PMPI_Finalized
#pragma weak MPI_Finalize = PMPI_Finalize
#pragma weak MPI_Query_thread = PMPI_Query_thread
#pragma weak MPI_Abort = PMPI_Abort
#pragma weak MPI_Wtime = PMPI_Wtime
#pragma weak MPI_Wtick = PMPI_Wtick
#pragma weak MPI_Get_processor_name = PMPI_Get_processor_name
#pragma weak MPI_Get_library_version = PMPI_Get_library_version
#pragma weak MPI_Error_string = PMPI_Error_string
#pragma weak MPI_Comm_rank = PMPI_Comm_rank
#pragma weak MPI_Comm_size = PMPI_Comm_size
#pragma weak MPI_Comm_test_inter = PMPI_Comm_test_inter
#pragma weak MPI_Comm_dup = PMPI_Comm_dup
#pragma weak MPI_Comm_split = PMPI_Comm_split
#pragma weak MPI_Comm_free = PMPI_Comm_free
#pragma weak MPI_Comm_set_errhandler = PMPI_Comm_set_errhandler
#pragma weak MPI_Type_size = PMPI_Type_size
#pragma weak MPI_Type_get_extent = PMPI_Type_get_extent
#pragma weak MPI_Type_contiguous = PMPI_Type_contiguous
#pragma weak MPI_Type_commit = PMPI_Type_commit
#pragma weak MPI_Type_free = PMPI_Type_free
#pragma weak MPI_Get_count = PMPI_Get_count
#pragma weak MPI_Send = PMPI_Send
#pragma weak MPI_Recv = PMPI_Recv
#pragma weak MPI_Sendrecv = PMPI_Sendrecv
#pragma weak MPI_Isend = PMPI_Isend
#pragma weak MPI_Irecv = PMPI_Irecv
#pragma weak MPI_Wait = PMPI_Wait
#pragma weak MPI_Waitall = PMPI_Waitall
#pragma weak MPI_Test = PMPI_Test
#pragma weak MPI_Barrier = PMPI_Barrier
#pragma weak MPI_Bcast = PMPI_Bcast
#pragma weak MPI_Reduce = PMPI_Reduce
#pragma weak MPI_Allreduce = PMPI_Allreduce
#pragma weak MPI_Reduce_local = PMPI_Reduce_local
#pragma weak MPI_Allgather = PMPI_Allgather
#pragma weak MPI_Gather = PMPI_Gather
