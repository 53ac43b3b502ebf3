// cmpi_internal.h — internal state of minimpi, the bundled single-node MPI.
//
// Layout of a job:
//   * one POSIX shared-memory segment per job (created by cail-mpirun, or by
//     rank 0 when the job was started by torchrun) holding a header, one slot
//     per rank and a P x P matrix of single-producer/single-consumer byte
//     rings ("channels"); channel (s, d) carries every packet from s to d;
//   * a per-process progress engine that streams packets into the outgoing
//     rings and drains the incoming ones, matching them against posted
//     receives (MPI ordering: per (source, communicator) non-overtaking);
//   * host buffers travel eagerly through the rings; device buffers use a
//     rendezvous: the sender ships a CUDA-IPC descriptor, the receiver copies
//     directly from the sender's allocation and returns an ACK packet.
#pragma once

#include <mpi.h>

#include <atomic>
#include <cstdint>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <deque>
#include <list>
#include <map>
#include <memory>
#include <string>
#include <vector>

namespace cmpi {

// ---------------------------------------------------------------- logging
#define CMPI_ERR(fmt, ...) \
    std::fprintf(stderr, "[minimpi] rank %d: " fmt "\n", ::cmpi::g_world_rank, ##__VA_ARGS__)
extern int g_world_rank;

// ---------------------------------------------------------------- datatypes
// Element kinds used by the reduction table.
enum Kind : int {
    K_NONE = 0, K_I8, K_U8, K_I16, K_U16, K_I32, K_U32, K_I64, K_U64,
    K_F32, K_F64, K_LD, K_BOOL, K_WCHAR, K_2INT, K_NUM
};

struct TypeInfo {
    bool valid = false;
    bool predefined = false;
    bool committed = false;
    int size = 0;          // bytes per element of this type
    Kind kind = K_NONE;    // element kind of the base type
    int base_count = 1;    // derived contiguous: number of base elements
    MPI_Datatype base = MPI_DATATYPE_NULL;
};
const TypeInfo *type_info(MPI_Datatype dt);
int type_new_contiguous(int count, MPI_Datatype old, MPI_Datatype *out);
int type_free(MPI_Datatype *dt);

// Element-wise reduction inout[i] = inout[i] (op) in[i] on host memory.
// Returns MPI_SUCCESS or MPI_ERR_OP when (op, type) has no definition.
int reduce_host(const void *in, void *inout, long long nelem_base, Kind kind, MPI_Op op);
bool op_valid(MPI_Op op);

// ---------------------------------------------------------------- shm layout
constexpr uint64_t kMagic = 0x31534d4950434d43ull;  // "CMPCIPMS1" tag
constexpr size_t kPktHdr = 32;

struct alignas(64) SegHeader {
    std::atomic<uint64_t> magic;
    uint32_t nranks;
    uint32_t ring_bytes;
    uint64_t nonce;
    std::atomic<uint32_t> joined;
    std::atomic<uint32_t> abort_flag;
    std::atomic<int32_t> abort_code;
    std::atomic<int32_t> abort_rank;
};

struct alignas(64) RankSlot {
    std::atomic<int32_t> pid;
    std::atomic<uint32_t> state;  // 0 empty, 1 joined, 2 finalized
    uint64_t node_id;
};

struct alignas(64) ChanCtl {
    std::atomic<uint64_t> head;  // bytes produced (written by the sender)
    char pad0[56];
    std::atomic<uint64_t> tail;  // bytes consumed (written by the receiver)
    char pad1[56];
};

inline size_t segment_bytes(uint32_t n, uint32_t ring) {
    return sizeof(SegHeader) + sizeof(RankSlot) * n + sizeof(ChanCtl) * (size_t)n * n +
           (size_t)ring * n * n;
}

// Ring capacity per channel: 64 MiB of ring memory per job, each ring between
// 64 KiB and 1 MiB (CMPI_RING_BYTES overrides).
inline uint32_t default_ring_bytes(uint32_t n) {
    if (const char *e = getenv("CMPI_RING_BYTES")) {
        long v = strtol(e, nullptr, 10);
        if (v >= 4096) return (uint32_t)((v + 4095) & ~4095L);
    }
    size_t r = ((size_t)64 << 20) / ((size_t)n * n);
    if (r < ((size_t)64 << 10)) r = (size_t)64 << 10;
    if (r > ((size_t)1 << 20)) r = (size_t)1 << 20;
    return (uint32_t)(r & ~(size_t)4095);
}

// Packet header: every message on a channel starts with one of these.
enum PktType : uint32_t { PKT_EAGER = 1, PKT_RNDV = 2, PKT_ACK = 3 };
struct PktHdr {
    uint32_t type;
    int32_t ctx;
    int32_t tag;
    int32_t src;      // world rank of the sender
    uint64_t len;     // payload bytes that follow (EAGER: data, RNDV: descriptor)
    uint64_t rid;     // sender request id (RNDV) / acknowledged id (ACK)
};
static_assert(sizeof(PktHdr) == kPktHdr, "packet header must be 32 bytes");

// CUDA-IPC rendezvous descriptor (payload of a PKT_RNDV packet).
struct RndvDesc {
    unsigned char handle[64];  // cudaIpcMemHandle_t of the sender's allocation
    uint64_t buffer_id;        // CU_POINTER_ATTRIBUTE_BUFFER_ID of that allocation
    uint64_t offset;           // byte offset of the message inside the allocation
    uint64_t bytes;            // message size
    int32_t device;
    int32_t pad;
};

// ---------------------------------------------------------------- requests
enum ReqKind { REQ_SEND = 1, REQ_RECV = 2 };

struct Unexpected;

struct Request {
    ReqKind kind;
    bool done = false;
    int err = MPI_SUCCESS;
    int ctx = 0, tag = 0;
    int peer = 0;               // world rank: destination (send) or source filter (recv)
    char *buf = nullptr;
    uint64_t bytes = 0;
    bool dev = false;           // buf is device memory
    int dev_ordinal = -1;
    // send side
    bool hdr_sent = false;
    uint64_t sent = 0;
    uint32_t proto = PKT_EAGER;
    uint64_t rid = 0;
    RndvDesc desc{};
    std::vector<char> stage;    // host copy of a device buffer that could not be exported
    const char *src_ptr = nullptr;
    // recv side
    MPI_Status status{};
    Unexpected *bound = nullptr;
};

struct Unexpected {
    int src, ctx, tag;
    uint32_t type;
    uint64_t len;
    uint64_t got = 0;
    bool complete = false;
    std::vector<char> data;     // eager payload or RndvDesc bytes
    uint64_t rid = 0;
    Request *bound = nullptr;   // receive that matched before the payload completed
};

// ---------------------------------------------------------------- comms
struct Comm {
    MPI_Comm handle = MPI_COMM_NULL;
    int ctx = 0;                // p2p context; ctx+1 is used by collectives
    int rank = 0;
    int size = 0;
    std::vector<int> world;     // comm rank -> world rank
    bool test_inter = false;
    MPI_Errhandler errh = MPI_ERRORS_ARE_FATAL;
    std::map<int, void *> attrs;
};
Comm *comm_get(MPI_Comm c);
int comm_world_rank(const Comm *c, int r);
int comm_create(const std::vector<int> &world_ranks, int my_rank, int ctx, MPI_Comm *out);
int comm_free(MPI_Comm *c);
int comm_alloc_ctx(Comm *parent, int *ctx);
int comm_delete_all_attrs(MPI_Comm c);
void comm_finalize_all();
int comm_errhandler_apply(MPI_Comm c, int rc, const char *where);

// ---------------------------------------------------------------- engine
struct Engine;
Engine &engine();

int init_transport(int *world_rank, int *world_size);
void finalize_transport();
bool transport_up();
int world_size();

// Nonblocking point-to-point (ranks are WORLD ranks here).
int isend(const void *buf, uint64_t bytes, int dest, int tag, int ctx, Request **out);
int irecv(void *buf, uint64_t bytes, int src, int tag, int ctx, Request **out);
int wait(Request *r, MPI_Status *st);            // frees r
int waitall(int n, Request **rs, MPI_Status *st); // frees all
bool test(Request *r);
void progress();
int check_health();     // abort flag, dead peers, timeout -> error code
void note_call();       // fault-injection hook, counts calls
void request_abort(int code);

// Handle table for MPI_Request.
MPI_Request req_to_handle(Request *r);
Request *handle_to_req(MPI_Request h);
void handle_release(MPI_Request h);

// ---------------------------------------------------------------- CUDA
// All CUDA use is optional: when no driver or no device is present every
// buffer is treated as host memory.
bool cuda_available();
bool is_device_ptr(const void *p, int *ordinal);
int cuda_copy(void *dst, const void *src, uint64_t bytes, int ordinal_hint);
// Builds an IPC descriptor for [p, p+bytes); false when the allocation cannot
// be exported (e.g. not from cudaMalloc).
bool ipc_describe(const void *p, uint64_t bytes, int ordinal, RndvDesc *d);
// Copies the rendezvous payload described by d (sent by world rank src) into dst.
int ipc_pull(int src, const RndvDesc &d, void *dst, bool dst_dev, int dst_ordinal);
void cuda_finalize();

// ---------------------------------------------------------------- collectives
int coll_barrier(Comm *c);
int coll_bcast(void *buf, uint64_t bytes, int root, Comm *c);
int coll_allgather_bytes(const void *send, uint64_t bytes, void *recv, Comm *c);
int coll_gather_bytes(const void *send, uint64_t bytes, void *recv, int root, Comm *c);
int coll_allreduce(const void *send, void *recv, int count, MPI_Datatype dt, MPI_Op op, Comm *c);
int coll_reduce(const void *send, void *recv, int count, MPI_Datatype dt, MPI_Op op, int root,
                Comm *c);

double now_s();
uint64_t node_id();

}  // namespace cmpi
