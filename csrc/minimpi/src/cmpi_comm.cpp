// cmpi_comm.cpp — communicators, context ids and attribute caching.
//
// A communicator is a rank translation table plus a context id; its
// point-to-point traffic is matched on ctx and its collectives on ctx + 1, so
// the two never mix.  New context ids are agreed with an allreduce(MAX) over
// the parent of every process' next free id, which keeps ids unique within
// each process and equal among a new communicator's members.
//
// Attribute caching follows MPI-3: delete callbacks run on MPI_Comm_free, on
// MPI_Comm_delete_attr, when an attribute is overwritten, and at
// MPI_Finalize (MPI_COMM_SELF first), which is how layered libraries release
// per-communicator state.
#include "cmpi_internal.h"

#include <unistd.h>

#include <algorithm>

namespace cmpi {

namespace {
std::vector<std::unique_ptr<Comm>> g_comms;
int g_next_ctx = 4;

struct Keyval {
    bool valid = false;
    MPI_Comm_copy_attr_function *copy_fn = nullptr;
    MPI_Comm_delete_attr_function *delete_fn = nullptr;
    void *extra = nullptr;
};
std::vector<Keyval> g_keyvals;
}  // namespace

Comm *comm_get(MPI_Comm c) {
    if (c <= 0 || (size_t)c >= g_comms.size()) return nullptr;
    return g_comms[c].get();
}

int comm_world_rank(const Comm *c, int r) {
    if (r == MPI_ANY_SOURCE || r == MPI_PROC_NULL) return r;
    if (r < 0 || r >= c->size) return -100;
    return c->world[r];
}

int comm_create(const std::vector<int> &world_ranks, int my_rank, int ctx, MPI_Comm *out) {
    auto c = std::make_unique<Comm>();
    c->ctx = ctx;
    c->rank = my_rank;
    c->size = (int)world_ranks.size();
    c->world = world_ranks;
    if (g_comms.empty()) g_comms.resize(1);  // handle 0 is MPI_COMM_NULL
    size_t slot = 0;
    for (size_t i = 3; i < g_comms.size(); ++i)
        if (!g_comms[i]) { slot = i; break; }
    if (*out == MPI_COMM_WORLD || *out == MPI_COMM_SELF) {
        slot = (size_t)*out;
        if (g_comms.size() <= slot) g_comms.resize(slot + 1);
    } else if (slot == 0) {
        if (g_comms.size() < 3) g_comms.resize(3);
        slot = g_comms.size();
        g_comms.resize(slot + 1);
    }
    c->handle = (MPI_Comm)slot;
    g_comms[slot] = std::move(c);
    *out = (MPI_Comm)slot;
    return MPI_SUCCESS;
}

int comm_alloc_ctx(Comm *parent, int *ctx) {
    int mine = g_next_ctx, agreed = 0;
    int rc = coll_allreduce(&mine, &agreed, 1, MPI_INT, MPI_MAX, parent);
    if (rc != MPI_SUCCESS) return rc;
    *ctx = agreed;
    g_next_ctx = agreed + 2;
    return MPI_SUCCESS;
}

static int delete_attr(Comm *c, MPI_Comm h, int keyval) {
    auto it = c->attrs.find(keyval);
    if (it == c->attrs.end()) return MPI_ERR_KEYVAL;
    void *v = it->second;
    c->attrs.erase(it);
    if (keyval >= 0 && (size_t)keyval < g_keyvals.size() && g_keyvals[keyval].delete_fn)
        return g_keyvals[keyval].delete_fn(h, keyval, v, g_keyvals[keyval].extra);
    return MPI_SUCCESS;
}

int comm_delete_all_attrs(MPI_Comm h) {
    Comm *c = comm_get(h);
    if (!c) return MPI_ERR_COMM;
    std::vector<int> keys;
    for (auto &kv : c->attrs) keys.push_back(kv.first);
    for (int k : keys) delete_attr(c, h, k);
    return MPI_SUCCESS;
}

int comm_free(MPI_Comm *h) {
    if (!h || *h == MPI_COMM_WORLD || *h == MPI_COMM_SELF) return MPI_ERR_COMM;
    Comm *c = comm_get(*h);
    if (!c) return MPI_ERR_COMM;
    comm_delete_all_attrs(*h);
    g_comms[*h].reset();
    *h = MPI_COMM_NULL;
    return MPI_SUCCESS;
}

void comm_finalize_all() {
    comm_delete_all_attrs(MPI_COMM_SELF);
    comm_delete_all_attrs(MPI_COMM_WORLD);
    for (size_t i = 3; i < g_comms.size(); ++i)
        if (g_comms[i]) comm_delete_all_attrs((MPI_Comm)i);
    g_comms.clear();
}

int comm_errhandler_apply(MPI_Comm h, int rc, const char *where) {
    if (rc == MPI_SUCCESS) return rc;
    Comm *c = comm_get(h);
    MPI_Errhandler eh = c ? c->errh : MPI_ERRORS_ARE_FATAL;
    if (eh == MPI_ERRORS_RETURN) return rc;
    std::fprintf(stderr, "[minimpi] rank %d: %s failed with error %d; aborting job\n", g_world_rank,
                 where, rc);
    std::fflush(stderr);
    request_abort(rc);
    _exit(rc);
}

// ------------------------------------------------------------------ attributes
}  // namespace cmpi

using namespace cmpi;

extern "C" {

int PMPI_Comm_create_keyval(MPI_Comm_copy_attr_function *copy_fn,
                            MPI_Comm_delete_attr_function *delete_fn, int *keyval,
                            void *extra_state) {
    if (!keyval) return MPI_ERR_ARG;
    Keyval k;
    k.valid = true;
    k.copy_fn = copy_fn;
    k.delete_fn = delete_fn;
    k.extra = extra_state;
    for (size_t i = 0; i < g_keyvals.size(); ++i) {
        if (!g_keyvals[i].valid) { g_keyvals[i] = k; *keyval = (int)i; return MPI_SUCCESS; }
    }
    g_keyvals.push_back(k);
    *keyval = (int)g_keyvals.size() - 1;
    return MPI_SUCCESS;
}

int PMPI_Comm_free_keyval(int *keyval) {
    if (!keyval || *keyval < 0 || (size_t)*keyval >= g_keyvals.size()) return MPI_ERR_KEYVAL;
    g_keyvals[*keyval].valid = false;
    *keyval = MPI_KEYVAL_INVALID;
    return MPI_SUCCESS;
}

int PMPI_Comm_set_attr(MPI_Comm comm, int keyval, void *value) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    if (keyval < 0 || (size_t)keyval >= g_keyvals.size() || !g_keyvals[keyval].valid)
        return MPI_ERR_KEYVAL;
    if (c->attrs.count(keyval)) delete_attr(c, comm, keyval);
    c->attrs[keyval] = value;
    return MPI_SUCCESS;
}

int PMPI_Comm_get_attr(MPI_Comm comm, int keyval, void *value, int *flag) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    if (keyval == MPI_TAG_UB) {
        static int tag_ub = MPI_TAG_UB_VALUE;
        *(void **)value = &tag_ub;
        *flag = 1;
        return MPI_SUCCESS;
    }
    auto it = c->attrs.find(keyval);
    *flag = it != c->attrs.end();
    if (*flag) *(void **)value = it->second;
    return MPI_SUCCESS;
}

int PMPI_Comm_delete_attr(MPI_Comm comm, int keyval) {
    Comm *c = comm_get(comm);
    if (!c) return MPI_ERR_COMM;
    return delete_attr(c, comm, keyval);
}

}  // extern "C"

#pragma weak MPI_Comm_create_keyval = PMPI_Comm_create_keyval
#pragma weak MPI_Comm_free_keyval = PMPI_Comm_free_keyval
#pragma weak MPI_Comm_set_attr = PMPI_Comm_set_attr
#pragma weak MPI_Comm_get_attr = PMPI_Comm_get_attr
#pragma weak MPI_Comm_delete_attr = PMPI_Comm_delete_attr

namespace cmpi {
// Copies attributes from src to the freshly created dst using copy callbacks.
int comm_copy_attrs(MPI_Comm src, MPI_Comm dst) {
    Comm *s = comm_get(src), *d = comm_get(dst);
    if (!s || !d) return MPI_ERR_COMM;
    for (auto &kv : s->attrs) {
        int k = kv.first;
        if (k < 0 || (size_t)k >= g_keyvals.size() || !g_keyvals[k].copy_fn) continue;
        void *out = nullptr;
        int flag = 0;
        int rc = g_keyvals[k].copy_fn(src, k, g_keyvals[k].extra, kv.second, &out, &flag);
        if (rc != MPI_SUCCESS) return rc;
        if (flag) d->attrs[k] = out;
    }
    return MPI_SUCCESS;
}
}  // namespace cmpi
