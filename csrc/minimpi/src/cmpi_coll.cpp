// cmpi_coll.cpp — collectives of minimpi, built on the point-to-point engine.
//
// MPI_Allreduce is the oracle and the "no interposer" baseline of this
// repository, so it is deterministic: every element is reduced in rank order
//     acc = x_0;  acc = op(acc, x_1);  ...;  acc = op(acc, x_{P-1})
// and every rank receives the same bits.  The algorithm is a direct
// reduce-scatter (rank r gathers block r from all ranks and reduces it in
// rank order) followed by a direct allgather, segmented so that temporary
// memory stays bounded.  Device buffers are staged through host memory, as
// an MPI without GPU collectives would do.
#include "cmpi_internal.h"

#include <algorithm>

namespace cmpi {

namespace {
inline int coll_ctx(const Comm *c) { return c->ctx + 1; }
constexpr int kTagBarrier = 1, kTagBcast = 2, kTagGather = 3, kTagAllgather = 4, kTagRS = 5,
              kTagAG = 6;
constexpr uint64_t kSegmentBytes = 32ull << 20;
}  // namespace

int coll_barrier(Comm *c) {
    int P = c->size, r = c->rank;
    char dummy = 0;
    for (int k = 1; k < P; k <<= 1) {
        Request *rq[2];
        int rc = isend(&dummy, 0, c->world[(r + k) % P], kTagBarrier, coll_ctx(c), &rq[0]);
        if (rc == MPI_SUCCESS) rc = irecv(&dummy, 0, c->world[(r - k + P) % P], kTagBarrier, coll_ctx(c), &rq[1]);
        if (rc == MPI_SUCCESS) rc = waitall(2, rq, nullptr);
        if (rc != MPI_SUCCESS) return rc;
    }
    return MPI_SUCCESS;
}

int coll_bcast(void *buf, uint64_t bytes, int root, Comm *c) {
    int P = c->size;
    if (P == 1) return MPI_SUCCESS;
    int vr = (c->rank - root + P) % P;  // virtual rank, root = 0
    int mask = 1;
    while (mask < P) {
        if (vr & mask) {
            int src = (vr - mask + root) % P;
            Request *q;
            int rc = irecv(buf, bytes, c->world[src], kTagBcast, coll_ctx(c), &q);
            if (rc == MPI_SUCCESS) rc = wait(q, nullptr);
            if (rc != MPI_SUCCESS) return rc;
            break;
        }
        mask <<= 1;
    }
    mask >>= 1;
    while (mask > 0) {
        if (vr + mask < P) {
            int dst = (vr + mask + root) % P;
            Request *q;
            int rc = isend(buf, bytes, c->world[dst], kTagBcast, coll_ctx(c), &q);
            if (rc == MPI_SUCCESS) rc = wait(q, nullptr);
            if (rc != MPI_SUCCESS) return rc;
        }
        mask >>= 1;
    }
    return MPI_SUCCESS;
}

int coll_allgather_bytes(const void *send, uint64_t bytes, void *recv, Comm *c) {
    int P = c->size, r = c->rank;
    char *out = (char *)recv;
    if (send != MPI_IN_PLACE && bytes) {
        int ord = -1;
        bool dev = is_device_ptr(out, &ord) || is_device_ptr(send, &ord);
        if (dev) cuda_copy(out + (uint64_t)r * bytes, send, bytes, ord);
        else memcpy(out + (uint64_t)r * bytes, send, bytes);
    }
    std::vector<Request *> rq;
    rq.reserve(2 * P);
    for (int q = 0; q < P; ++q) {
        if (q == r) continue;
        Request *a;
        int rc = irecv(out + (uint64_t)q * bytes, bytes, c->world[q], kTagAllgather, coll_ctx(c), &a);
        if (rc != MPI_SUCCESS) return rc;
        rq.push_back(a);
    }
    for (int q = 0; q < P; ++q) {
        if (q == r) continue;
        Request *a;
        int rc = isend(out + (uint64_t)r * bytes, bytes, c->world[q], kTagAllgather, coll_ctx(c), &a);
        if (rc != MPI_SUCCESS) return rc;
        rq.push_back(a);
    }
    return waitall((int)rq.size(), rq.data(), nullptr);
}

int coll_gather_bytes(const void *send, uint64_t bytes, void *recv, int root, Comm *c) {
    int P = c->size, r = c->rank;
    if (r != root) {
        Request *a;
        int rc = isend(send, bytes, c->world[root], kTagGather, coll_ctx(c), &a);
        return rc == MPI_SUCCESS ? wait(a, nullptr) : rc;
    }
    char *out = (char *)recv;
    if (send != MPI_IN_PLACE && bytes) {
        int ord = -1;
        if (is_device_ptr(out, &ord) || is_device_ptr(send, &ord))
            cuda_copy(out + (uint64_t)r * bytes, send, bytes, ord);
        else
            memcpy(out + (uint64_t)r * bytes, send, bytes);
    }
    std::vector<Request *> rq;
    for (int q = 0; q < P; ++q) {
        if (q == r) continue;
        Request *a;
        int rc = irecv(out + (uint64_t)q * bytes, bytes, c->world[q], kTagGather, coll_ctx(c), &a);
        if (rc != MPI_SUCCESS) return rc;
        rq.push_back(a);
    }
    return waitall((int)rq.size(), rq.data(), nullptr);
}

// Host allreduce of n base elements of size esz, in place on `buf`.
static int allreduce_host_inplace(char *buf, uint64_t n, int esz, Kind kind, MPI_Op op, Comm *c) {
    int P = c->size, r = c->rank;
    if (P == 1 || n == 0) return MPI_SUCCESS;
    uint64_t seg_elems = std::max<uint64_t>(kSegmentBytes / (uint64_t)esz, (uint64_t)P);
    std::vector<char> tmp, acc;
    for (uint64_t s0 = 0; s0 < n; s0 += seg_elems) {
        uint64_t sn = std::min<uint64_t>(seg_elems, n - s0);
        char *seg = buf + s0 * esz;
        uint64_t base = sn / P, rem = sn % P;
        auto blk_off = [&](int q) { return (uint64_t)q * base + std::min<uint64_t>((uint64_t)q, rem); };
        auto blk_len = [&](int q) { return base + ((uint64_t)q < rem ? 1 : 0); };
        uint64_t my_off = blk_off(r), my_len = blk_len(r);
        tmp.resize((size_t)P * my_len * esz);
        std::vector<Request *> rq;
        rq.reserve(2 * P);
        int rc = MPI_SUCCESS;
        for (int q = 0; q < P && rc == MPI_SUCCESS; ++q) {
            if (q == r) continue;
            Request *a;
            rc = irecv(tmp.data() + (uint64_t)q * my_len * esz, my_len * esz, c->world[q], kTagRS,
                       coll_ctx(c), &a);
            if (rc == MPI_SUCCESS) rq.push_back(a);
        }
        for (int q = 0; q < P && rc == MPI_SUCCESS; ++q) {
            if (q == r) continue;
            Request *a;
            rc = isend(seg + blk_off(q) * esz, blk_len(q) * esz, c->world[q], kTagRS, coll_ctx(c), &a);
            if (rc == MPI_SUCCESS) rq.push_back(a);
        }
        if (rc == MPI_SUCCESS) rc = waitall((int)rq.size(), rq.data(), nullptr);
        if (rc != MPI_SUCCESS) return rc;
        // own contribution into its slot, then reduce in rank order
        if (my_len) memcpy(tmp.data() + (uint64_t)r * my_len * esz, seg + my_off * esz, my_len * esz);
        acc.assign(tmp.data(), tmp.data() + my_len * esz);
        for (int q = 1; q < P; ++q) {
            rc = reduce_host(tmp.data() + (uint64_t)q * my_len * esz, acc.data(), (long long)my_len, kind, op);
            if (rc != MPI_SUCCESS) return rc;
        }
        if (my_len) memcpy(seg + my_off * esz, acc.data(), my_len * esz);
        rq.clear();
        for (int q = 0; q < P && rc == MPI_SUCCESS; ++q) {
            if (q == r) continue;
            Request *a;
            rc = irecv(seg + blk_off(q) * esz, blk_len(q) * esz, c->world[q], kTagAG, coll_ctx(c), &a);
            if (rc == MPI_SUCCESS) rq.push_back(a);
        }
        for (int q = 0; q < P && rc == MPI_SUCCESS; ++q) {
            if (q == r) continue;
            Request *a;
            rc = isend(seg + my_off * esz, my_len * esz, c->world[q], kTagAG, coll_ctx(c), &a);
            if (rc == MPI_SUCCESS) rq.push_back(a);
        }
        if (rc == MPI_SUCCESS) rc = waitall((int)rq.size(), rq.data(), nullptr);
        if (rc != MPI_SUCCESS) return rc;
    }
    return MPI_SUCCESS;
}

int coll_allreduce(const void *send, void *recv, int count, MPI_Datatype dt, MPI_Op op, Comm *c) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    if (count < 0) return MPI_ERR_COUNT;
    const TypeInfo *bi = type_info(ti->base);
    int esz = bi ? bi->size : ti->size;
    uint64_t n = (uint64_t)count * (uint64_t)ti->base_count;
    uint64_t bytes = n * (uint64_t)esz;
    if (reduce_host(nullptr, nullptr, 0, ti->kind, op) != MPI_SUCCESS) return MPI_ERR_OP;
    if (count == 0) return MPI_SUCCESS;
    int ord = -1;
    bool rdev = is_device_ptr(recv, &ord);
    bool sdev = send != MPI_IN_PLACE && is_device_ptr(send, rdev ? nullptr : &ord);
    if (!rdev && !sdev) {
        if (send != MPI_IN_PLACE && send != recv) memcpy(recv, send, bytes);
        return allreduce_host_inplace((char *)recv, n, esz, ti->kind, op, c);
    }
    // Stage device data through host memory.
    std::vector<char> host(bytes);
    const void *src = send == MPI_IN_PLACE ? recv : send;
    int rc = (send == MPI_IN_PLACE ? rdev : sdev) ? cuda_copy(host.data(), src, bytes, ord)
                                                  : (memcpy(host.data(), src, bytes), MPI_SUCCESS);
    if (rc != MPI_SUCCESS) return rc;
    rc = allreduce_host_inplace(host.data(), n, esz, ti->kind, op, c);
    if (rc != MPI_SUCCESS) return rc;
    if (rdev) return cuda_copy(recv, host.data(), bytes, ord);
    memcpy(recv, host.data(), bytes);
    return MPI_SUCCESS;
}

int coll_reduce(const void *send, void *recv, int count, MPI_Datatype dt, MPI_Op op, int root,
                Comm *c) {
    const TypeInfo *ti = type_info(dt);
    if (!ti) return MPI_ERR_TYPE;
    uint64_t bytes = (uint64_t)count * (uint64_t)ti->size;
    const void *src = send;
    if (send == MPI_IN_PLACE) {
        if (c->rank != root) return MPI_ERR_BUFFER;
        src = recv;
    }
    std::vector<char> tmp(bytes);
    int ord = -1;
    if (bytes && is_device_ptr(src, &ord)) cuda_copy(tmp.data(), src, bytes, ord);
    else if (bytes) memcpy(tmp.data(), src, bytes);
    int rc = coll_allreduce(MPI_IN_PLACE, tmp.data(), count, dt, op, c);
    if (rc != MPI_SUCCESS || c->rank != root || !bytes) return rc;
    if (is_device_ptr(recv, &ord)) return cuda_copy(recv, tmp.data(), bytes, ord);
    memcpy(recv, tmp.data(), bytes);
    return MPI_SUCCESS;
}

}  // namespace cmpi
