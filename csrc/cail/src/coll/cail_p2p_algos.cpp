// cail_p2p_algos.cpp — host-driven allreduce algorithms over PMPI
// point-to-point: recursive doubling, ring and Rabenseifner.
//
// These are the reference's three algorithms (src/coll/allreduce/
// cail_allreduce_{recursive_doubling,ring,rabenseifner}.c there), kept as the
// path for communicators whose GPUs cannot reach each other over NVLink
// (several nodes, no peer access) and for the host-only build.  Data moves
// with PMPI_Sendrecv (device buffers need a CUDA-aware MPI, which minimpi
// is); every received block is folded into the result with
// cail_gpu_reduce_local, i.e. result = op(result, received).
//
// Shared structure:
//   * copy-in: sendbuf -> recvbuf unless MPI_IN_PLACE; the algorithms then
//     work in place on recvbuf, with one scratch buffer (cail_buf);
//   * non-power-of-two P: the first 2*rem ranks pair up, each even rank
//     hands its vector to the odd neighbour and sits out ("fold"), and gets
//     the result back at the end ("unfold"); the remaining pof2 ranks run
//     the power-of-two core under virtual ranks 0..pof2-1.
//
// Rabenseifner is written with explicit block ranges: the vector is cut into
// pof2 blocks; in reduce-scatter step k (distance pof2/2^(k+1)) a rank keeps
// the half of its current range selected by its own virtual-rank bit and
// sends the other half, so after log2(pof2) steps virtual rank v owns block
// v; the allgather retraces the steps in reverse.  This also removes the
// reference's read of uninitialised pointers on its early error exits
// (cail_allreduce_rabenseifner.c:82-122,265-271 there).
#include <stdlib.h>

#include <vector>

#include "../core/cail_internal.h"
#include "../gpu/cail_gpu.h"
#include "cail_p2p_algos.h"

namespace {

constexpr int kTag = 0;

struct Call {
    const void *send;
    void *recv;
    int count;
    MPI_Datatype dt;
    MPI_Op op;
    MPI_Comm comm;
    int rank = 0, P = 1;
    cail_datatype_t dtype = CAIL_INVALID;
    cail_op_t optype = CAIL_OP_INVALID;
    size_t esz = 0;
    size_t bytes = 0;
    char *rb() const { return (char *)recv; }
};

int setup(Call &c) {
    int rc = PMPI_Comm_rank(c.comm, &c.rank);
    CAIL_CHECK(rc);
    rc = PMPI_Comm_size(c.comm, &c.P);
    CAIL_CHECK(rc);
    c.dtype = cail_mpi_type_to_dtype(c.dt);
    c.optype = cail_mpi_op_to_optype(c.op);
    c.esz = (size_t)cail_type_size(c.dtype);
    if (c.dtype == CAIL_INVALID || c.optype == CAIL_OP_INVALID || c.esz == 0) return MPI_ERR_OP;
    c.bytes = (size_t)c.count * c.esz;
    return MPI_SUCCESS;
}

int copy_in(const Call &c) {
    const void *src = c.send == MPI_IN_PLACE ? c.recv : c.send;
    if (src == c.recv || c.bytes == 0) return MPI_SUCCESS;
    return cail_gpu_memcpy(c.recv, src, c.bytes) == 0 ? MPI_SUCCESS : MPI_ERR_INTERN;
}

// Folds received data into the result: dst = op(dst, tmp).
int fold_in(const Call &c, const void *tmp, void *dst, size_t n) {
    if (n == 0) return MPI_SUCCESS;
    cail_gpu_flush_recv_buf(tmp, n * c.esz);
    return cail_gpu_reduce_local(tmp, dst, n, c.dtype, c.optype) == 0 ? MPI_SUCCESS : MPI_ERR_INTERN;
}

// Non-power-of-two pairing.  Returns the virtual rank, or -1 for a rank that
// handed its data over and sits out the core algorithm.
int fold(const Call &c, int pof2, void *tmp, int *vrank) {
    int rem = c.P - pof2;
    *vrank = c.rank >= 2 * rem ? c.rank - rem : (c.rank % 2 ? c.rank / 2 : -1);
    if (c.rank >= 2 * rem) return MPI_SUCCESS;
    if (c.rank % 2 == 0) return PMPI_Send(c.recv, c.count, c.dt, c.rank + 1, kTag, c.comm);
    int rc = PMPI_Recv(tmp, c.count, c.dt, c.rank - 1, kTag, c.comm, MPI_STATUS_IGNORE);
    CAIL_CHECK(rc);
    return fold_in(c, tmp, c.recv, (size_t)c.count);
}

int unfold(const Call &c, int pof2) {
    int rem = c.P - pof2;
    if (c.rank >= 2 * rem) return MPI_SUCCESS;
    if (c.rank % 2 == 0)
        return PMPI_Recv(c.recv, c.count, c.dt, c.rank + 1, kTag, c.comm, MPI_STATUS_IGNORE);
    return PMPI_Send(c.recv, c.count, c.dt, c.rank - 1, kTag, c.comm);
}

// Real rank of virtual rank v.
inline int real_rank(int v, int rem) { return v < rem ? 2 * v + 1 : v + rem; }

int single_rank(const Call &c) { return copy_in(c); }

}  // namespace

extern "C" {

int cail_allreduce_recursive_doubling(const void *sendbuf, void *recvbuf, int count,
                                      MPI_Datatype datatype, MPI_Op op, MPI_Comm comm) {
    Call c{sendbuf, recvbuf, count, datatype, op, comm};
    int rc = setup(c);
    CAIL_CHECK(rc);
    if (count == 0) return MPI_SUCCESS;
    if (c.P == 1) return single_rank(c);
    void *tmp = nullptr;
    rc = cail_buf_get_tmp(&tmp, c.bytes);
    CAIL_CHECK(rc);
    rc = copy_in(c);
    CAIL_CHECK(rc);
    int pof2 = cail_pof2(c.P), rem = c.P - pof2, v;
    rc = fold(c, pof2, tmp, &v);
    CAIL_CHECK(rc);
    for (int mask = 1; v >= 0 && mask < pof2; mask <<= 1) {
        int peer = real_rank(v ^ mask, rem);
        rc = PMPI_Sendrecv(c.recv, count, datatype, peer, kTag, tmp, count, datatype, peer, kTag,
                           comm, MPI_STATUS_IGNORE);
        CAIL_CHECK(rc);
        rc = fold_in(c, tmp, c.recv, (size_t)count);
        CAIL_CHECK(rc);
    }
    rc = unfold(c, pof2);
    cail_buf_release_tmp(tmp);
    return rc;
}

int cail_allreduce_ring(const void *sendbuf, void *recvbuf, int count, MPI_Datatype datatype,
                        MPI_Op op, MPI_Comm comm) {
    Call c{sendbuf, recvbuf, count, datatype, op, comm};
    int rc = setup(c);
    CAIL_CHECK(rc);
    if (count == 0) return MPI_SUCCESS;
    if (c.P == 1) return single_rank(c);
    if (count < c.P) {
        CAIL_WARN("ring: count=%d < nprocs=%d, cannot distribute chunks, falling back to PMPI",
                  count, c.P);
        return PMPI_Allreduce(sendbuf, recvbuf, count, datatype, op, comm);
    }
    rc = copy_in(c);
    CAIL_CHECK(rc);
    // Chunk i covers [off[i], off[i] + len[i]); the first count % P chunks get
    // one extra element.
    std::vector<int> len(c.P);
    std::vector<size_t> off(c.P + 1, 0);
    for (int i = 0; i < c.P; ++i) {
        len[i] = count / c.P + (i < count % c.P ? 1 : 0);
        off[i + 1] = off[i] + (size_t)len[i];
    }
    void *tmp = nullptr;
    rc = cail_buf_get_tmp(&tmp, (size_t)len[0] * c.esz);
    CAIL_CHECK(rc);
    int right = (c.rank + 1) % c.P, left = (c.rank + c.P - 1) % c.P;
    auto chunk = [&](int i) { return c.rb() + off[((i % c.P) + c.P) % c.P] * c.esz; };
    auto clen = [&](int i) { return len[((i % c.P) + c.P) % c.P]; };
    // Reduce-scatter: in step s a rank forwards its partial chunk (rank - s)
    // and folds the incoming chunk (rank - s - 1); after P-1 steps chunk
    // (rank + 1) mod P is complete here.
    for (int s = 0; s < c.P - 1; ++s) {
        int out = c.rank - s, in = c.rank - s - 1;
        rc = PMPI_Sendrecv(chunk(out), clen(out), datatype, right, kTag, tmp, clen(in), datatype,
                           left, kTag, comm, MPI_STATUS_IGNORE);
        CAIL_CHECK(rc);
        rc = fold_in(c, tmp, chunk(in), (size_t)clen(in));
        CAIL_CHECK(rc);
    }
    // Allgather: circulate the completed chunks.
    for (int s = 0; s < c.P - 1; ++s) {
        int out = c.rank + 1 - s, in = c.rank - s;
        rc = PMPI_Sendrecv(chunk(out), clen(out), datatype, right, kTag, chunk(in), clen(in),
                           datatype, left, kTag, comm, MPI_STATUS_IGNORE);
        CAIL_CHECK(rc);
        cail_gpu_flush_recv_buf(chunk(in), (size_t)clen(in) * c.esz);
    }
    cail_buf_release_tmp(tmp);
    return MPI_SUCCESS;
}

int cail_allreduce_rabenseifner(const void *sendbuf, void *recvbuf, int count,
                                MPI_Datatype datatype, MPI_Op op, MPI_Comm comm) {
    Call c{sendbuf, recvbuf, count, datatype, op, comm};
    int rc = setup(c);
    CAIL_CHECK(rc);
    if (count == 0) return MPI_SUCCESS;
    if (c.P == 1) return single_rank(c);
    int pof2 = cail_pof2(c.P), rem = c.P - pof2;
    if (count < pof2) {
        CAIL_ERR("rabenseifner: count=%d < pof2=%d (nprocs=%d), cannot distribute in "
                 "reduce-scatter", count, pof2, c.P);
        return MPI_ERR_COUNT;
    }
    void *tmp = nullptr;
    rc = cail_buf_get_tmp(&tmp, c.bytes);
    CAIL_CHECK(rc);
    rc = copy_in(c);
    CAIL_CHECK(rc);
    int v;
    rc = fold(c, pof2, tmp, &v);
    CAIL_CHECK(rc);
    if (v >= 0) {
        // Block b covers [off[b], off[b+1]); the first count % pof2 blocks get
        // one extra element.
        std::vector<size_t> off(pof2 + 1, 0);
        for (int b = 0; b < pof2; ++b)
            off[b + 1] = off[b] + (size_t)(count / pof2 + (b < count % pof2 ? 1 : 0));
        auto elems = [&](int lo, int hi) { return (int)(off[hi] - off[lo]); };
        auto at = [&](char *base, int blk) { return base + off[blk] * c.esz; };
        int lo = 0, hi = pof2;
        // Reduce-scatter by recursive halving.
        for (int mask = pof2 >> 1; mask >= 1; mask >>= 1) {
            int peer = real_rank(v ^ mask, rem);
            int mid = lo + (hi - lo) / 2;
            int keep_lo = (v & mask) ? mid : lo, keep_hi = (v & mask) ? hi : mid;
            int send_lo = (v & mask) ? lo : mid, send_hi = (v & mask) ? mid : hi;
            rc = PMPI_Sendrecv(at(c.rb(), send_lo), elems(send_lo, send_hi), datatype, peer, kTag,
                               at((char *)tmp, keep_lo), elems(keep_lo, keep_hi), datatype, peer,
                               kTag, comm, MPI_STATUS_IGNORE);
            CAIL_CHECK(rc);
            rc = fold_in(c, at((char *)tmp, keep_lo), at(c.rb(), keep_lo),
                         (size_t)elems(keep_lo, keep_hi));
            CAIL_CHECK(rc);
            lo = keep_lo;
            hi = keep_hi;
        }
        // Allgather by recursive doubling, retracing the halving steps.
        for (int mask = 1; mask < pof2; mask <<= 1) {
            int peer = real_rank(v ^ mask, rem);
            int width = hi - lo;
            int plo = (v & mask) ? lo - width : hi, phi = plo + width;
            rc = PMPI_Sendrecv(at(c.rb(), lo), elems(lo, hi), datatype, peer, kTag, at(c.rb(), plo),
                               elems(plo, phi), datatype, peer, kTag, comm, MPI_STATUS_IGNORE);
            CAIL_CHECK(rc);
            cail_gpu_flush_recv_buf(at(c.rb(), plo), (size_t)elems(plo, phi) * c.esz);
            lo = lo < plo ? lo : plo;
            hi = hi > phi ? hi : phi;
        }
    }
    rc = unfold(c, pof2);
    cail_buf_release_tmp(tmp);
    return rc;
}

}  // extern "C"
