// cail_dev_comm.cpp — per-communicator device runtime of the NVLink path.
//
// Setup (collective, at the first device MPI_Allreduce on a communicator):
//   1. topology probe: PMPI_Allgather of {host id, pid, GPU UUID}; the path
//      is used only if all ranks share a node, every rank has its own GPU,
//      every peer GPU is visible and peer-accessible, and P <= 8;
//   2. workspace: one cudaMalloc per rank (arrival flags + two one-shot
//      scratch halves), exported with cudaIpcGetMemHandle, exchanged with
//      PMPI_Allgather and opened by every peer;
//   3. host exchange segment: POSIX shared memory with one cache-line slot
//      per rank, used by the two-shot path to publish the IPC descriptors of
//      the user buffers of each call and as a host barrier;
//   4. NVLS (when every GPU reports CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED
//      and CAIL_NVLS != 0): rank 0 creates a multicast object, passes its
//      POSIX file descriptor to the other ranks over a Unix-domain socket
//      (SCM_RIGHTS); each rank adds its GPU, binds its own physical memory
//      and maps both the unicast and the multicast view.
// Every step ends with an agreement (PMPI_Allreduce MIN of a success flag),
// so all ranks take the same path.  The context is cached on the
// communicator as an MPI attribute and destroyed by its delete callback.
//
// Registration cache: the user buffers of two-shot calls are exported once
// per allocation (keyed by CU_POINTER_ATTRIBUTE_BUFFER_ID, which is never
// reused) and each peer allocation is opened once (LRU of 1024 mappings).
#include "cail_dev.h"

#include <cuda.h>
#include <cuda_runtime.h>
#include <errno.h>
#include <fcntl.h>
#include <sched.h>
#include <signal.h>
#include <string.h>
#include <sys/mman.h>
#include <sys/socket.h>
#include <sys/stat.h>
#include <sys/un.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <list>
#include <string>
#include <unordered_map>
#include <vector>

#include "../core/cail_internal.h"
#include "cail_dev_kernels.cuh"

using cail::DevStatus;
using cail::kMaxBlocks;
using cail::kMaxRanks;

namespace {

// ---------------------------------------------------------------- driver API
struct Driver {
    bool loaded = false;
    CUresult (*pointerGetAttribute)(void *, CUpointer_attribute, CUdeviceptr) = nullptr;
    CUresult (*memGetAddressRange)(CUdeviceptr *, size_t *, CUdeviceptr) = nullptr;
    CUresult (*deviceGet)(CUdevice *, int) = nullptr;
    CUresult (*deviceGetAttribute)(int *, CUdevice_attribute, CUdevice) = nullptr;
    CUresult (*memCreate)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *,
                          unsigned long long) = nullptr;
    CUresult (*memRelease)(CUmemGenericAllocationHandle) = nullptr;
    CUresult (*memAddressReserve)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long) = nullptr;
    CUresult (*memAddressFree)(CUdeviceptr, size_t) = nullptr;
    CUresult (*memMap)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long) = nullptr;
    CUresult (*memUnmap)(CUdeviceptr, size_t) = nullptr;
    CUresult (*memSetAccess)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t) = nullptr;
    CUresult (*memGetAllocationGranularity)(size_t *, const CUmemAllocationProp *,
                                            CUmemAllocationGranularity_flags) = nullptr;
    CUresult (*memExportToShareableHandle)(void *, CUmemGenericAllocationHandle,
                                           CUmemAllocationHandleType, unsigned long long) = nullptr;
    CUresult (*memImportFromShareableHandle)(CUmemGenericAllocationHandle *, void *,
                                             CUmemAllocationHandleType) = nullptr;
    CUresult (*multicastCreate)(CUmemGenericAllocationHandle *, const CUmulticastObjectProp *) = nullptr;
    CUresult (*multicastAddDevice)(CUmemGenericAllocationHandle, CUdevice) = nullptr;
    CUresult (*multicastBindMem)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle,
                                 size_t, size_t, unsigned long long) = nullptr;
    CUresult (*multicastBindAddr)(CUmemGenericAllocationHandle, size_t, CUdeviceptr, size_t,
                                  unsigned long long) = nullptr;
    CUresult (*multicastUnbind)(CUmemGenericAllocationHandle, CUdevice, size_t, size_t) = nullptr;
    CUresult (*multicastGetGranularity)(size_t *, const CUmulticastObjectProp *,
                                        CUmulticastGranularity_flags) = nullptr;
};
Driver g_drv;

template <typename F>
void load_sym(const char *name, F &fn) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        fn = reinterpret_cast<F>(p);
}

void load_driver() {
    if (g_drv.loaded) return;
    g_drv.loaded = true;
    load_sym("cuPointerGetAttribute", g_drv.pointerGetAttribute);
    load_sym("cuMemGetAddressRange", g_drv.memGetAddressRange);
    load_sym("cuDeviceGet", g_drv.deviceGet);
    load_sym("cuDeviceGetAttribute", g_drv.deviceGetAttribute);
    load_sym("cuMemCreate", g_drv.memCreate);
    load_sym("cuMemRelease", g_drv.memRelease);
    load_sym("cuMemAddressReserve", g_drv.memAddressReserve);
    load_sym("cuMemAddressFree", g_drv.memAddressFree);
    load_sym("cuMemMap", g_drv.memMap);
    load_sym("cuMemUnmap", g_drv.memUnmap);
    load_sym("cuMemSetAccess", g_drv.memSetAccess);
    load_sym("cuMemGetAllocationGranularity", g_drv.memGetAllocationGranularity);
    load_sym("cuMemExportToShareableHandle", g_drv.memExportToShareableHandle);
    load_sym("cuMemImportFromShareableHandle", g_drv.memImportFromShareableHandle);
    load_sym("cuMulticastCreate", g_drv.multicastCreate);
    load_sym("cuMulticastAddDevice", g_drv.multicastAddDevice);
    load_sym("cuMulticastBindMem", g_drv.multicastBindMem);
    load_sym("cuMulticastBindAddr", g_drv.multicastBindAddr);
    load_sym("cuMulticastUnbind", g_drv.multicastUnbind);
    load_sym("cuMulticastGetGranularity", g_drv.multicastGetGranularity);
}

// ---------------------------------------------------------------- constants
// Workspace of a rank (IPC-exported): [flag area | one-shot area | push RS
// area | push AG area].  The flag area holds the one-shot, RS and AG flags
// (one word per source rank and CTA each) and the per-CTA round / step
// counters of the one-shot and NVLS kernels.
constexpr size_t kFlagBytes = 64 << 10;
static_assert(cail::kFlagAreaWords * sizeof(uint32_t) <= kFlagBytes, "flag arrays exceed the flag area");
constexpr size_t kOsOff = kFlagBytes;
constexpr size_t kDefaultPieceMin = 4 << 10;             // push two-shot: smallest piece
constexpr size_t kOsPieceMin = 8 << 10;                  // one-shot: smallest piece
constexpr size_t kNvlsStepsOff = cail::kNvlsStepsBase * sizeof(uint32_t);
constexpr size_t kNvlsCtrRegion = (cail::kNvlsCtrBytes + 65535) / 65536 * 65536;  // counters, then staging
constexpr size_t kDefaultNvlsUnit = 1 << 20;            // NVLS: largest bytes per CTA and step

// ---------------------------------------------------------------- host exchange
struct BufDesc {
    cudaIpcMemHandle_t handle;
    uint64_t id;
    uint64_t offset;
    int32_t ok;
    int32_t pad;
};

// arrive / depart hold the call sequence number; a rank that failed sets
// kXErr as well, so its peers stop waiting and report the error too.
constexpr uint64_t kXErr = 1ull << 63;

struct alignas(128) XSlot {
    std::atomic<uint64_t> arrive;
    char pad0[56];
    std::atomic<uint64_t> depart;
    char pad1[56];
    BufDesc send, recv;
    int32_t pid;
};

struct ProbeInfo {
    unsigned long long host;
    int pid;
    int ordinal;
    char uuid[16];
    int nvls_capable;
    int sms;
};

struct Export {
    cudaIpcMemHandle_t handle;
    uintptr_t base;
    bool ok;
};

struct ImportKey {
    int peer;
    uint64_t id;
    bool operator==(const ImportKey &o) const { return peer == o.peer && id == o.id; }
};
struct ImportKeyHash {
    size_t operator()(const ImportKey &k) const { return std::hash<uint64_t>()(k.id * 31 + (uint64_t)k.peer); }
};
struct Import {
    char *base;
    std::list<ImportKey>::iterator lru;
};
constexpr size_t kMaxImports = 1024;

// A process counts as gone when it no longer exists or is a zombie (it
// exited and its parent has not reaped it yet).
bool process_gone(int pid) {
    if (pid <= 0) return false;
    if (kill(pid, 0) != 0) return errno == ESRCH;
    char path[64], buf[256];
    snprintf(path, sizeof(path), "/proc/%d/stat", pid);
    int fd = open(path, O_RDONLY);
    if (fd < 0) return false;
    ssize_t n = read(fd, buf, sizeof(buf) - 1);
    close(fd);
    if (n <= 0) return false;
    buf[n] = 0;
    const char *rp = strrchr(buf, ')');
    return rp && rp[1] == ' ' && (rp[2] == 'Z' || rp[2] == 'X');
}

unsigned long long host_id() {
    char h[256] = {0};
    gethostname(h, sizeof(h) - 1);
    unsigned long long x = 1469598103934665603ull;
    for (const char *p = h; *p; ++p) { x ^= (unsigned char)*p; x *= 1099511628211ull; }
    return x;
}

}  // namespace

// ---------------------------------------------------------------- context
struct cail_dev_comm {
    MPI_Comm comm = MPI_COMM_NULL;
    bool ok = false;
    bool broken = false;
    bool shared_gpu = false;  // test mode: ranks share a GPU (zero-copy two-shot only)
    int rank = 0, P = 1, dev = -1, sms = 148;
    cudaStream_t stream = nullptr;
    // workspace
    char *ws = nullptr;
    char *peer_ws[kMaxRanks] = {};
    uint32_t epoch = 0;
    // push two-shot: CTAs per rank, largest piece, bytes per area, round epoch
    int push_gmax = 0;
    size_t push_piece_max = 0, push_area = 0;
    uint32_t push_epoch = 0;
    // one-shot: largest piece and bytes of its area; piece of the last call
    size_t os_piece_max = 0, os_area = 0, os_piece_last = 0;
    DevStatus *status_h = nullptr, *status_d = nullptr;
    // host exchange
    XSlot *xs = nullptr;
    size_t xs_bytes = 0;
    uint64_t xseq = 0;
    int peer_pid[kMaxRanks] = {};
    // registration cache
    std::unordered_map<uint64_t, Export> exports;
    std::unordered_map<ImportKey, Import, ImportKeyHash> imports;
    std::list<ImportKey> lru;
    // NVLS
    bool nvls = false;
    size_t nvls_unit = 0, nvls_size = 0;
    CUmemGenericAllocationHandle mc_handle = 0, phys_handle = 0;
    CUdeviceptr uc_va = 0, mc_va = 0;
    bool mc_bound = false;
    int nvls_blocks = 0;
    double last_live_check = 0.0;
    cudaEvent_t legacy_ev = nullptr;  // marks the legacy stream's queue at call entry
    cudaEvent_t done_ev = nullptr;    // end of a stream-ordered call, waited for by the legacy stream
    bool pending = false;             // a stream-ordered call has not been checked yet
    // copy-engine two-shot: pull / fold / push streams, per-buffer events and
    // a scratch of kCeMaxBufs x (P-1) chunks (created on first use)
    cudaStream_t ce_pull = nullptr, ce_fold = nullptr, ce_push = nullptr;
    cudaEvent_t ce_pulled[4] = {}, ce_folded[4] = {}, ce_start = nullptr, ce_end = nullptr;
    char *ce_scratch = nullptr;
    size_t ce_scratch_bytes = 0;
};

namespace {

int g_keyval = MPI_KEYVAL_INVALID;
std::vector<cail_dev_comm *> g_contexts;
int g_shm_serial = 0;

void destroy_context(cail_dev_comm *dc);

int delete_cb(MPI_Comm, int, void *val, void *) {
    auto *dc = static_cast<cail_dev_comm *>(val);
    for (auto it = g_contexts.begin(); it != g_contexts.end(); ++it)
        if (*it == dc) { g_contexts.erase(it); break; }
    destroy_context(dc);
    return MPI_SUCCESS;
}

bool agree(MPI_Comm comm, bool mine) {
    int v = mine ? 1 : 0, all = 0;
    if (PMPI_Allreduce(&v, &all, 1, MPI_INT, MPI_MIN, comm) != MPI_SUCCESS) return false;
    return all == 1;
}

int find_ordinal(const char uuid[16]) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) return -1;
    for (int d = 0; d < n; ++d) {
        cudaDeviceProp p;
        if (cudaGetDeviceProperties(&p, d) == cudaSuccess && memcmp(p.uuid.bytes, uuid, 16) == 0) return d;
    }
    return -1;
}

// ---- host barrier over the exchange segment
// Waits until every rank's arrive (depart) word reaches seq.  Bounded: a peer
// that has exited fails the wait at once, and a live peer that does not
// arrive within CAIL_HOST_TIMEOUT_MS (default: the device timeout) fails it
// at the deadline.  On failure this rank's own word is switched to
// seq | kXErr (unless it already moved on), so that a peer arriving late
// sees the failure instead of starting the collective, and
// MPI_ERR_OTHER is returned; the caller marks the communicator broken.
long host_timeout_ms() {
    static const long v = [] {
        const char *e = getenv("CAIL_HOST_TIMEOUT_MS");
        long t = e && *e ? atol(e) : 0;
        return t > 0 ? t : 0;
    }();
    return v > 0 ? v : cail_global_state.device_timeout_ms;
}

int host_wait(cail_dev_comm *dc, bool depart, uint64_t seq) {
    unsigned spins = 0;
    const double deadline = cail_now_us() + 1000.0 * (double)host_timeout_ms();
    std::atomic<uint64_t> &mine = depart ? dc->xs[dc->rank].depart : dc->xs[dc->rank].arrive;
    for (int q = 0; q < dc->P; ++q) {
        // a peer that gave up at this call's arrive barrier never departs
        if (depart && dc->xs[q].arrive.load(std::memory_order_acquire) == (seq | kXErr)) continue;
        std::atomic<uint64_t> &a = depart ? dc->xs[q].depart : dc->xs[q].arrive;
        while ((a.load(std::memory_order_acquire) & ~kXErr) < seq) {
            if (++spins % 4096 == 0) {
                const bool gone = process_gone(dc->peer_pid[q]);
                if (gone || cail_now_us() > deadline) {
                    if (gone)
                        CAIL_ERR("rank %d: peer rank %d (pid %d) is gone", dc->rank, q, dc->peer_pid[q]);
                    else
                        CAIL_ERR("rank %d: peer rank %d did not reach the %s barrier of call %llu within %ld ms "
                                 "(CAIL_HOST_TIMEOUT_MS)",
                                 dc->rank, q, depart ? "depart" : "arrive", (unsigned long long)seq, host_timeout_ms());
                    uint64_t cur = seq;
                    mine.compare_exchange_strong(cur, seq | kXErr, std::memory_order_acq_rel);
                    return MPI_ERR_OTHER;
                }
                if (spins > (1u << 20)) sched_yield();
            }
        }
    }
    return MPI_SUCCESS;
}

// ---- registration cache
bool describe(cail_dev_comm *dc, const void *p, BufDesc *d) {
    memset(d, 0, sizeof(*d));
    if (!g_drv.pointerGetAttribute || !g_drv.memGetAddressRange) return false;
    unsigned long long id = 0;
    if (g_drv.pointerGetAttribute(&id, CU_POINTER_ATTRIBUTE_BUFFER_ID, (CUdeviceptr)p) != CUDA_SUCCESS)
        return false;
    auto it = dc->exports.find(id);
    if (it == dc->exports.end()) {
        Export ex{};
        CUdeviceptr base = 0;
        size_t size = 0;
        ex.ok = g_drv.memGetAddressRange(&base, &size, (CUdeviceptr)p) == CUDA_SUCCESS &&
                cudaIpcGetMemHandle(&ex.handle, (void *)base) == cudaSuccess;
        if (!ex.ok) cudaGetLastError();
        ex.base = (uintptr_t)base;
        it = dc->exports.emplace(id, ex).first;
    }
    if (!it->second.ok) return false;
    d->handle = it->second.handle;
    d->id = id;
    d->offset = (uint64_t)((uintptr_t)p - it->second.base);
    d->ok = 1;
    return true;
}

char *import_buf(cail_dev_comm *dc, int q, const BufDesc &d) {
    ImportKey k{q, d.id};
    auto it = dc->imports.find(k);
    if (it != dc->imports.end()) {
        dc->lru.splice(dc->lru.begin(), dc->lru, it->second.lru);
        cail_counters.reg_hits++;
        return it->second.base + d.offset;
    }
    void *base = nullptr;
    cudaError_t e = cudaIpcOpenMemHandle(&base, d.handle, cudaIpcMemLazyEnablePeerAccess);
    if (e == cudaErrorAlreadyMapped) {
        // The peer freed an allocation that is still mapped here and reused
        // its memory: drop this peer's mappings and open again.
        cudaGetLastError();
        for (auto i = dc->imports.begin(); i != dc->imports.end();) {
            if (i->first.peer == q) {
                cudaIpcCloseMemHandle(i->second.base);
                dc->lru.erase(i->second.lru);
                i = dc->imports.erase(i);
            } else {
                ++i;
            }
        }
        e = cudaIpcOpenMemHandle(&base, d.handle, cudaIpcMemLazyEnablePeerAccess);
    }
    if (e != cudaSuccess) {
        CAIL_ERR("rank %d: cannot open rank %d's buffer: %s", dc->rank, q, cudaGetErrorString(e));
        cudaGetLastError();
        return nullptr;
    }
    cail_counters.reg_misses++;
    if (dc->imports.size() >= kMaxImports) {
        ImportKey old = dc->lru.back();
        dc->lru.pop_back();
        auto o = dc->imports.find(old);
        if (o != dc->imports.end()) {
            cudaIpcCloseMemHandle(o->second.base);
            dc->imports.erase(o);
        }
    }
    dc->lru.push_front(k);
    dc->imports[k] = Import{(char *)base, dc->lru.begin()};
    return (char *)base + d.offset;
}

// ---- Unix-socket file descriptor passing (NVLS handle exchange)
bool send_fd(int sock, int fd) {
    char byte = 0;
    struct iovec iov = {&byte, 1};
    char ctrl[CMSG_SPACE(sizeof(int))];
    memset(ctrl, 0, sizeof(ctrl));
    struct msghdr m;
    memset(&m, 0, sizeof(m));
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    m.msg_control = ctrl;
    m.msg_controllen = sizeof(ctrl);
    struct cmsghdr *c = CMSG_FIRSTHDR(&m);
    c->cmsg_level = SOL_SOCKET;
    c->cmsg_type = SCM_RIGHTS;
    c->cmsg_len = CMSG_LEN(sizeof(int));
    memcpy(CMSG_DATA(c), &fd, sizeof(int));
    return sendmsg(sock, &m, 0) == 1;
}

int recv_fd(int sock) {
    char byte;
    struct iovec iov = {&byte, 1};
    char ctrl[CMSG_SPACE(sizeof(int))];
    struct msghdr m;
    memset(&m, 0, sizeof(m));
    m.msg_iov = &iov;
    m.msg_iovlen = 1;
    m.msg_control = ctrl;
    m.msg_controllen = sizeof(ctrl);
    if (recvmsg(sock, &m, 0) != 1) return -1;
    struct cmsghdr *c = CMSG_FIRSTHDR(&m);
    if (!c || c->cmsg_type != SCM_RIGHTS) return -1;
    int fd;
    memcpy(&fd, CMSG_DATA(c), sizeof(int));
    return fd;
}

// Shares rank 0's file descriptor with every rank.  Returns the local fd
// (rank 0: its own) or -1.  Collective.
int share_fd(cail_dev_comm *dc, int fd0) {
    char name[108] = {0};
    int lsock = -1;
    if (dc->rank == 0) {
        snprintf(name + 1, sizeof(name) - 2, "cail-nvls-%d-%d", (int)getpid(), ++g_shm_serial);
        lsock = socket(AF_UNIX, SOCK_STREAM, 0);
        struct sockaddr_un a;
        memset(&a, 0, sizeof(a));
        a.sun_family = AF_UNIX;
        memcpy(a.sun_path, name, sizeof(a.sun_path));
        socklen_t len = (socklen_t)(offsetof(struct sockaddr_un, sun_path) + 1 + strlen(name + 1));
        if (lsock < 0 || bind(lsock, (struct sockaddr *)&a, len) != 0 || listen(lsock, 64) != 0) {
            if (lsock >= 0) close(lsock);
            lsock = -1;
            name[1] = 0;
        }
    }
    PMPI_Bcast(name, sizeof(name), MPI_CHAR, 0, dc->comm);
    if (name[1] == 0) return -1;
    int fd = -1;
    if (dc->rank == 0) {
        bool ok = true;
        for (int i = 1; i < dc->P; ++i) {
            int c = accept(lsock, nullptr, nullptr);
            if (c < 0 || !send_fd(c, fd0)) ok = false;
            if (c >= 0) close(c);
        }
        close(lsock);
        fd = ok ? fd0 : -1;
    } else {
        int s = socket(AF_UNIX, SOCK_STREAM, 0);
        struct sockaddr_un a;
        memset(&a, 0, sizeof(a));
        a.sun_family = AF_UNIX;
        memcpy(a.sun_path, name, sizeof(a.sun_path));
        socklen_t len = (socklen_t)(offsetof(struct sockaddr_un, sun_path) + 1 + strlen(name + 1));
        if (s >= 0 && connect(s, (struct sockaddr *)&a, len) == 0) fd = recv_fd(s);
        if (s >= 0) close(s);
    }
    return fd;
}

void nvls_teardown(cail_dev_comm *dc) {
    if (dc->mc_va) {
        g_drv.memUnmap(dc->mc_va, dc->nvls_size);
        g_drv.memAddressFree(dc->mc_va, dc->nvls_size);
        dc->mc_va = 0;
    }
    if (dc->mc_bound) {
        CUdevice cd;
        g_drv.deviceGet(&cd, dc->dev);
        g_drv.multicastUnbind(dc->mc_handle, cd, 0, dc->nvls_size);
        dc->mc_bound = false;
    }
    if (dc->uc_va) {
        g_drv.memUnmap(dc->uc_va, dc->nvls_size);
        g_drv.memAddressFree(dc->uc_va, dc->nvls_size);
        dc->uc_va = 0;
    }
    if (dc->phys_handle) { g_drv.memRelease(dc->phys_handle); dc->phys_handle = 0; }
    if (dc->mc_handle) { g_drv.memRelease(dc->mc_handle); dc->mc_handle = 0; }
    dc->nvls = false;
}

// Collective NVLS setup.  Leaves dc->nvls false (on every rank) on failure;
// with CAIL_DEBUG the failing step and its CUresult are printed.
bool nvls_step(cail_dev_comm *dc, bool ok, CUresult r, const char *what) {
    if (ok && r != CUDA_SUCCESS) {
        CAIL_DBG("nvls: rank %d: %s failed (CUresult %d)", dc->rank, what, (int)r);
        return false;
    }
    return ok;
}

int nvls_min_ranks();
int nvls_min_ranks_env();

// The multicast region (2 staging slots per CTA, ~592 MiB per GPU with 1 MiB
// units) is created only where it can be used: CAIL_ALGO=nvls, or auto mode
// from the built-in 8 ranks (or CAIL_NVLS_MIN_RANKS), or a CAIL_TUNE_FILE
// line for P that gives nvls_min.
bool nvls_wanted(int P) {
    if (!cail_global_state.nvls || P < 2) return false;
    if (cail_global_state.force_algo == CAIL_ALGO_NVLS) return true;
    const cail_tune_t *t = cail_tune_for(P);
    if (nvls_min_ranks_env() < 0 && t) return t->nvls_min >= 0;
    return nvls_min_ranks() > 0 && P >= nvls_min_ranks();
}

void nvls_setup(cail_dev_comm *dc, bool all_capable) {
    // (cuMulticastCreate refuses a one-device object: INVALID_VALUE on B200)
    if (!nvls_wanted(dc->P)) return;
    if (!all_capable) {
        CAIL_DBG("nvls: not every GPU reports CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED");
        return;
    }
    if (!g_drv.multicastCreate || !g_drv.multicastBindMem || !g_drv.memCreate) {
        CAIL_DBG("nvls: driver entry points missing");
        return;
    }
    // CAIL_NVLS_UNIT: largest bytes per CTA and step (a multiple of 64 KiB)
    size_t unit = kDefaultNvlsUnit;
    if (const char *e = getenv("CAIL_NVLS_UNIT")) {
        long v = atol(e);
        if (v >= (64 << 10) && v <= (64 << 20)) unit = (size_t)v / 65536 * 65536;
    }
    const int blocks = cail::nvls_max_ctas(dc->sms);
    CUdevice cd = 0;
    bool ok = nvls_step(dc, true, g_drv.deviceGet(&cd, dc->dev), "cuDeviceGet");
    CUmulticastObjectProp mp;
    memset(&mp, 0, sizeof(mp));
    mp.numDevices = (unsigned)dc->P;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    CUmemAllocationProp ap;
    memset(&ap, 0, sizeof(ap));
    ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
    ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    ap.location.id = cd;
    ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;  // as the multicast object
    size_t g1 = 0, g2 = 0;
    const size_t want = kNvlsCtrRegion + (size_t)blocks * 2 * unit;  // two staging slots per CTA
    mp.size = want;
    ok = nvls_step(dc, ok, g_drv.multicastGetGranularity(&g1, &mp, CU_MULTICAST_GRANULARITY_MINIMUM),
                   "cuMulticastGetGranularity");
    ok = nvls_step(dc, ok, g_drv.memGetAllocationGranularity(&g2, &ap, CU_MEM_ALLOC_GRANULARITY_MINIMUM),
                   "cuMemGetAllocationGranularity");
    size_t gran = g1 > g2 ? g1 : g2;
    if (gran == 0) gran = 2 << 20;
    size_t size = (want + gran - 1) / gran * gran;
    mp.size = size;
    dc->nvls_size = size;
    dc->nvls_unit = unit;
    if (!agree(dc->comm, ok)) return;

    int fd = -1;
    if (dc->rank == 0) {
        ok = nvls_step(dc, true, g_drv.multicastCreate(&dc->mc_handle, &mp), "cuMulticastCreate");
        ok = nvls_step(dc, ok,
                       g_drv.memExportToShareableHandle(&fd, dc->mc_handle,
                                                        CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR, 0),
                       "cuMemExportToShareableHandle");
    }
    if (!agree(dc->comm, ok)) { nvls_teardown(dc); return; }
    int myfd = share_fd(dc, fd);
    ok = myfd >= 0;
    if (!ok) CAIL_DBG("nvls: rank %d: file descriptor exchange failed", dc->rank);
    if (ok && dc->rank != 0)
        ok = nvls_step(dc, ok,
                       g_drv.memImportFromShareableHandle(&dc->mc_handle, (void *)(uintptr_t)myfd,
                                                          CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR),
                       "cuMemImportFromShareableHandle");
    if (myfd >= 0) close(myfd);
    if (!agree(dc->comm, ok)) { nvls_teardown(dc); return; }
    ok = nvls_step(dc, ok, g_drv.multicastAddDevice(dc->mc_handle, cd), "cuMulticastAddDevice");
    if (!agree(dc->comm, ok)) { nvls_teardown(dc); return; }  // every device added before binding
    ok = nvls_step(dc, ok, g_drv.memCreate(&dc->phys_handle, size, &ap, 0), "cuMemCreate");
    CUmemAccessDesc acc;
    memset(&acc, 0, sizeof(acc));
    acc.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
    acc.location.id = cd;
    acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
    ok = nvls_step(dc, ok, g_drv.memAddressReserve(&dc->uc_va, size, gran, 0, 0), "cuMemAddressReserve(uc)");
    ok = nvls_step(dc, ok, g_drv.memMap(dc->uc_va, size, 0, dc->phys_handle, 0), "cuMemMap(uc)");
    ok = nvls_step(dc, ok, g_drv.memSetAccess(dc->uc_va, size, &acc, 1), "cuMemSetAccess(uc)");
    if (ok) {
        CUresult r = g_drv.multicastBindMem(dc->mc_handle, 0, dc->phys_handle, 0, size, 0);
        if (r != CUDA_SUCCESS && g_drv.multicastBindAddr) {
            CAIL_DBG("nvls: rank %d: cuMulticastBindMem returned %d, trying cuMulticastBindAddr", dc->rank, (int)r);
            r = g_drv.multicastBindAddr(dc->mc_handle, 0, dc->uc_va, size, 0);
        }
        ok = nvls_step(dc, ok, r, "cuMulticastBind");
        dc->mc_bound = ok;
    }
    ok = nvls_step(dc, ok, g_drv.memAddressReserve(&dc->mc_va, size, gran, 0, 0), "cuMemAddressReserve(mc)");
    ok = nvls_step(dc, ok, g_drv.memMap(dc->mc_va, size, 0, dc->mc_handle, 0), "cuMemMap(mc)");
    ok = nvls_step(dc, ok, g_drv.memSetAccess(dc->mc_va, size, &acc, 1), "cuMemSetAccess(mc)");
    if (ok && (cudaMemset((void *)dc->uc_va, 0, kNvlsCtrRegion) != cudaSuccess ||
               cudaDeviceSynchronize() != cudaSuccess)) {
        CAIL_DBG("nvls: rank %d: clearing the counters failed", dc->rank);
        ok = false;
    }
    if (!agree(dc->comm, ok)) { nvls_teardown(dc); return; }
    dc->nvls_blocks = blocks;
    dc->nvls = true;
    CAIL_DBG("nvls: multicast region of %zu bytes (granularity %zu), %d CTAs x 2 slots of %zu bytes", size, gran,
             blocks, unit);
}

void ce_teardown(cail_dev_comm *dc) {
    for (cudaStream_t *s : {&dc->ce_pull, &dc->ce_fold, &dc->ce_push})
        if (*s) { cudaStreamSynchronize(*s); cudaStreamDestroy(*s); *s = nullptr; }
    for (int i = 0; i < 4; ++i) {
        if (dc->ce_pulled[i]) cudaEventDestroy(dc->ce_pulled[i]);
        if (dc->ce_folded[i]) cudaEventDestroy(dc->ce_folded[i]);
        dc->ce_pulled[i] = dc->ce_folded[i] = nullptr;
    }
    if (dc->ce_start) cudaEventDestroy(dc->ce_start);
    if (dc->ce_end) cudaEventDestroy(dc->ce_end);
    dc->ce_start = dc->ce_end = nullptr;
    if (dc->ce_scratch) cudaFree(dc->ce_scratch);
    dc->ce_scratch = nullptr;
    dc->ce_scratch_bytes = 0;
}

void destroy_context(cail_dev_comm *dc) {
    if (!dc) return;
    if (dc->ok) {
        int prev = -1;
        cudaGetDevice(&prev);
        if (dc->dev >= 0) cudaSetDevice(dc->dev);
        if (dc->stream) cudaStreamSynchronize(dc->stream);
        nvls_teardown(dc);
        ce_teardown(dc);
        for (auto &kv : dc->imports) cudaIpcCloseMemHandle(kv.second.base);
        dc->imports.clear();
        for (int q = 0; q < dc->P; ++q)
            if (q != dc->rank && dc->peer_ws[q]) cudaIpcCloseMemHandle(dc->peer_ws[q]);
        if (dc->ws) cudaFree(dc->ws);
        // the last stream-ordered call's status is read before the pinned
        // block that holds it is released (the stream was synchronised above)
        if (dc->pending && dc->status_h && dc->status_h->code != 0)
            CAIL_ERR("a stream-ordered MPI_Allreduce on this communicator failed: rank %d gave up "
                     "waiting (block %d, epoch %u)", dc->status_h->rank, dc->status_h->block, dc->status_h->epoch);
        dc->pending = false;
        if (dc->status_h) cudaFreeHost(dc->status_h);
        dc->status_h = nullptr;
        dc->status_d = nullptr;
        if (dc->stream) cudaStreamDestroy(dc->stream);
        if (dc->legacy_ev) cudaEventDestroy(dc->legacy_ev);
        if (dc->done_ev) cudaEventDestroy(dc->done_ev);
        if (dc->xs) munmap(dc->xs, dc->xs_bytes);
        if (prev >= 0) cudaSetDevice(prev);
    }
    delete dc;
}

// CAIL_TWOSHOT_PIECE_MAX / CAIL_TWOSHOT_PIECE_MIN (bytes, multiples of 16):
// the largest and smallest piece a CTA of the push two-shot moves per round
// and slice.  The largest one sizes the workspace (2 x 2 x G x P x piece).
size_t env_bytes(const char *name, size_t dflt, size_t lo, size_t hi) {
    const char *e = getenv(name);
    if (!e || !*e) return dflt;
    size_t v = (size_t)strtoull(e, nullptr, 10);
    v = v / 16 * 16;
    return v < lo ? lo : (v > hi ? hi : v);
}
size_t push_piece_max_env() {
    static const size_t v = env_bytes("CAIL_TWOSHOT_PIECE_MAX", 0, 1024, (size_t)1 << 20);
    return v;
}
size_t push_piece_min_env() {
    static const size_t v = env_bytes("CAIL_TWOSHOT_PIECE_MIN", kDefaultPieceMin, 256, (size_t)1 << 20);
    return v;
}

// CAIL_TEST_SHARED_GPU=1 (tests only): a communicator whose ranks share a
// GPU still gets the NVLink runtime, so that a one-GPU test run exercises
// the cross-process IPC, the registration cache and the P > 1 slicing of
// the zero-copy two-shot.  Only that path (and the copy-engine two-shot)
// then runs: its kernels never wait on another rank's kernel, the ranks
// meet on the host.  The one-shot, push and NVLS kernels wait on their
// peers' flags and must not run as separate processes on one GPU (nothing
// makes such kernels run at the same time), so they are replaced by it.
bool test_shared_gpu() {
    static const bool v = [] {
        const char *e = getenv("CAIL_TEST_SHARED_GPU");
        return e && *e && *e != '0';
    }();
    return v;
}

// Workspace sizing, the same on every rank.  Push two-shot: the largest
// piece keeps its two areas (2 parities x G CTAs x P sources x piece each)
// near 296 MiB (128 KiB at 2 ranks, 64 KiB at 4, 32 KiB at 8; larger pieces
// amortise the flag round trips of each round) unless
// CAIL_TWOSHOT_PIECE_MAX sets it.  One-shot: 3 slots x G x P x piece, about
// 112 MiB (64 KiB pieces at 2 ranks, 16 KiB at 8).
size_t push_piece_max_for(int P, int gmax) {
    if (push_piece_max_env()) return push_piece_max_env();
    size_t pm = ((size_t)296 << 20) / ((size_t)4 * gmax * P);
    pm = pm / (16 << 10) * (16 << 10);
    return std::min(std::max(pm, (size_t)16 << 10), (size_t)256 << 10);
}
size_t push_area_for(int P, int gmax, size_t piece_max) {
    return ((size_t)2 * gmax * P * piece_max + 255) / 256 * 256;
}
size_t os_piece_max_for(int P, int gmax) {
    size_t pm = ((size_t)112 << 20) / ((size_t)cail::kOsSlots * gmax * P);
    pm = pm / (8 << 10) * (8 << 10);
    return std::min(std::max(pm, kOsPieceMin), (size_t)256 << 10);
}
size_t os_area_for(int P, int gmax, size_t piece_max) {
    return ((size_t)cail::kOsSlots * gmax * P * piece_max + 255) / 256 * 256;
}

// One-shot launch shape: pieces of at least 8 KiB so that small messages use
// few CTAs (one vector per thread), at most the area's piece.
void oneshot_shape(size_t bytes, int gmax, size_t piece_max, size_t *piece, int *G) {
    size_t p = (bytes + gmax - 1) / gmax;
    p = (p + 15) / 16 * 16;
    p = std::min(std::max(p, kOsPieceMin), piece_max);
    *piece = p;
    *G = (int)std::max<size_t>(1, std::min<size_t>((bytes + p - 1) / p, (size_t)gmax));
}

// NVLS launch shape: units of at most unit_max bytes (16 KiB to 64 KiB
// steps for small messages, so that every CTA has work), and as few CTAs as
// still give every CTA the same number of units (1 GiB of 1 MiB units: 256
// CTAs of 4 units, not 296 CTAs of 3 or 4).
void nvls_shape(size_t bytes, int gmax, size_t unit_max, size_t *unit, int *blocks) {
    size_t u = (bytes + gmax - 1) / gmax;
    u = u <= (16 << 10) ? (16 << 10) : (u + 65535) / 65536 * 65536;
    if (u > unit_max) u = unit_max;
    const size_t units = (bytes + u - 1) / u;
    const size_t per = (units + gmax - 1) / gmax;
    *unit = u;
    *blocks = (int)((units + per - 1) / per);
}

cail_dev_comm *create_context(MPI_Comm comm) {
    auto *dc = new cail_dev_comm();
    dc->comm = comm;
    PMPI_Comm_rank(comm, &dc->rank);
    PMPI_Comm_size(comm, &dc->P);
    load_driver();
    cudaGetDevice(&dc->dev);
    cudaFree(0);  // make the device's primary context current for driver calls

    // 1. topology probe
    ProbeInfo me;
    memset(&me, 0, sizeof(me));
    me.host = host_id();
    me.pid = (int)getpid();
    me.ordinal = dc->dev;
    cudaDeviceProp prop;
    bool ok = cudaGetDeviceProperties(&prop, dc->dev) == cudaSuccess;
    if (ok) {
        memcpy(me.uuid, prop.uuid.bytes, 16);
        me.sms = prop.multiProcessorCount;
    }
    int mc = 0;
    CUdevice cd;
    if (g_drv.deviceGet && g_drv.deviceGetAttribute && g_drv.deviceGet(&cd, dc->dev) == CUDA_SUCCESS)
        g_drv.deviceGetAttribute(&mc, CU_DEVICE_ATTRIBUTE_MULTICAST_SUPPORTED, cd);
    me.nvls_capable = mc && nvls_wanted(dc->P);  // every rank must want it, or none sets it up
    std::vector<ProbeInfo> all(dc->P);
    if (PMPI_Allgather(&me, sizeof(me), MPI_BYTE, all.data(), sizeof(me), MPI_BYTE, comm) != MPI_SUCCESS)
        ok = false;
    bool all_nvls = true;
    ok = ok && dc->P <= kMaxRanks;
    const bool shared_ok = test_shared_gpu();
    for (int q = 0; ok && q < dc->P; ++q) {
        dc->peer_pid[q] = all[q].pid;
        if (all[q].host != me.host) ok = false;
        if (!all[q].nvls_capable) all_nvls = false;
        for (int r = 0; r < q; ++r)
            if (memcmp(all[q].uuid, all[r].uuid, 16) == 0) {  // shared GPU
                if (shared_ok) dc->shared_gpu = true;
                else ok = false;
            }
        if (q == dc->rank) continue;
        int o = find_ordinal(all[q].uuid), can = 0;
        if (o == dc->dev && shared_ok) continue;  // same device: reached through IPC without peer access
        if (o < 0 || cudaDeviceCanAccessPeer(&can, dc->dev, o) != cudaSuccess || !can) ok = false;
    }
    if (dc->shared_gpu) all_nvls = false;
    // Launch shapes and workspace layouts derive from the SM count and must
    // be the same on every rank: take the smallest over the ranks.
    dc->sms = me.sms > 0 ? me.sms : 148;
    for (int q = 0; ok && q < dc->P; ++q)
        if (all[q].sms > 0 && all[q].sms < dc->sms) dc->sms = all[q].sms;
    if (!agree(comm, ok)) {
        CAIL_DBG("nvlink path unavailable on this communicator (probe)");
        return dc;  // ok == false
    }

    // 2. workspace
    ok = cudaStreamCreateWithFlags(&dc->stream, cudaStreamNonBlocking) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&dc->legacy_ev, cudaEventDisableTiming) == cudaSuccess;
    ok = ok && cudaEventCreateWithFlags(&dc->done_ev, cudaEventDisableTiming) == cudaSuccess;
    // push two-shot areas: 2 parities x G CTAs x P sources x the largest piece;
    // by default the piece keeps the two areas near 296 MiB (128 KiB at 2
    // ranks, 64 KiB at 4, 32 KiB at 8): larger pieces amortise the flag
    // round trips of each round
    dc->push_gmax = cail::push_max_ctas(1, dc->sms);
    dc->push_piece_max = push_piece_max_for(dc->P, dc->push_gmax);
    dc->push_area = push_area_for(dc->P, dc->push_gmax, dc->push_piece_max);
    dc->os_piece_max = os_piece_max_for(dc->P, dc->push_gmax);
    dc->os_area = os_area_for(dc->P, dc->push_gmax, dc->os_piece_max);
    ok = ok && cudaMalloc(&dc->ws, kOsOff + dc->os_area + 2 * dc->push_area) == cudaSuccess;
    ok = ok && cudaMemset(dc->ws, 0, kFlagBytes) == cudaSuccess && cudaDeviceSynchronize() == cudaSuccess;
    ok = ok && cudaHostAlloc((void **)&dc->status_h, sizeof(DevStatus), cudaHostAllocMapped) == cudaSuccess;
    ok = ok && cudaHostGetDevicePointer((void **)&dc->status_d, dc->status_h, 0) == cudaSuccess;
    if (ok) memset(dc->status_h, 0, sizeof(DevStatus));
    cudaIpcMemHandle_t h;
    memset(&h, 0, sizeof(h));
    ok = ok && cudaIpcGetMemHandle(&h, dc->ws) == cudaSuccess;
    std::vector<cudaIpcMemHandle_t> hs(dc->P);
    int ag = PMPI_Allgather(&h, sizeof(h), MPI_BYTE, hs.data(), sizeof(h), MPI_BYTE, comm);
    ok = ok && ag == MPI_SUCCESS;
    for (int q = 0; ok && q < dc->P; ++q) {
        if (q == dc->rank) { dc->peer_ws[q] = dc->ws; continue; }
        void *p = nullptr;
        if (cudaIpcOpenMemHandle(&p, hs[q], cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) ok = false;
        dc->peer_ws[q] = (char *)p;
    }
    if (!ok) cudaGetLastError();

    // 3. host exchange segment
    char name[64] = {0};
    dc->xs_bytes = sizeof(XSlot) * kMaxRanks;
    if (dc->rank == 0) {
        snprintf(name, sizeof(name), "/cail_x%d_%d", (int)getpid(), ++g_shm_serial);
        shm_unlink(name);
        int fd = shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600);
        if (fd < 0 || ftruncate(fd, (off_t)dc->xs_bytes) != 0) name[0] = 0;
        if (fd >= 0) close(fd);
    }
    PMPI_Bcast(name, sizeof(name), MPI_CHAR, 0, comm);
    if (name[0]) {
        int fd = shm_open(name, O_RDWR, 0600);
        void *m = fd >= 0 ? mmap(nullptr, dc->xs_bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0) : MAP_FAILED;
        if (fd >= 0) close(fd);
        if (m == MAP_FAILED) ok = false;
        else dc->xs = (XSlot *)m;
    } else {
        ok = false;
    }
    PMPI_Barrier(comm);
    if (dc->rank == 0 && name[0]) shm_unlink(name);
    if (dc->xs) dc->xs[dc->rank].pid = (int32_t)getpid();
    dc->ok = agree(comm, ok);
    if (!dc->ok) {
        CAIL_DBG("nvlink path unavailable on this communicator (workspace setup)");
        dc->ok = true;  // let destroy_context release what was created
        destroy_context(dc);
        dc = new cail_dev_comm();
        dc->comm = comm;
        return dc;
    }

    // 4. NVLS
    nvls_setup(dc, all_nvls);
    CAIL_DBG("nvlink path: P=%d device=%d sms=%d nvls=%d", dc->P, dc->dev, dc->sms, (int)dc->nvls);
    return dc;
}

int check_status(cail_dev_comm *dc, const char *what) {
    const double t0 = cail_global_state.profile ? cail_now_us() : 0.0;
    cudaError_t e = cudaStreamSynchronize(dc->stream);
    cail_prof_mark(CAIL_PH_WAIT, t0);
    if (e != cudaSuccess) {
        CAIL_ERR("%s: CUDA error %s", what, cudaGetErrorString(e));
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    if (dc->status_h->code != 0) {
        const DevStatus &s = *dc->status_h;
        if (s.code == 2)
            CAIL_ERR("%s: rank %d: device argument check %d failed (CAIL_DEVICE_CHECKS); the kernel did not run",
                     what, s.rank, s.waited_on);
        else
            CAIL_ERR("%s: rank %d gave up after %ld ms waiting for %s %d (block %d, epoch %u, saw %u)",
                     what, s.rank, cail_global_state.device_timeout_ms,
                     s.waited_on >= 0 ? "rank" : "barrier", s.waited_on >= 0 ? s.waited_on : -1 - s.waited_on,
                     s.block, s.epoch, s.seen);
        memset(dc->status_h, 0, sizeof(DevStatus));
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    return MPI_SUCCESS;
}

unsigned long long timeout_ns() { return (unsigned long long)cail_global_state.device_timeout_ms * 1000000ull; }

// ---- one-shot
// One launch for any size: pieces of at least 8 KiB so that small messages
// use few CTAs (one vector per thread), at most the area's piece.
int run_oneshot(cail_dev_comm *dc, const char *src, char *dst, size_t count, size_t esz, int op, int ec,
                bool allow_ordered);

// Stream-ordered completion (cail_set_stream_ordered): the legacy stream
// waits for the call's kernels and the host returns at once.  This is safe
// for the one-shot, push two-shot and NVLS kernels, which need no host
// exchange: each touches only its own workspace slots and its own user
// buffers, and their per-CTA flag protocols order every reuse of a slot
// across calls as within one call (successive calls run in stream order on
// each GPU).
bool stream_ordered_ok(const cail_dev_comm *dc) {
    return cail_global_state.stream_ordered && cail_global_state.stream_sync && dc->done_ev;
}

int finish_stream_ordered(cail_dev_comm *dc, const char *what) {
    if (cudaEventRecord(dc->done_ev, dc->stream) != cudaSuccess ||
        cudaStreamWaitEvent(cudaStreamLegacy, dc->done_ev, 0) != cudaSuccess) {
        CAIL_ERR("%s: ordering the legacy stream after the call failed", what);
        return check_status(dc, what);
    }
    dc->pending = true;
    return MPI_SUCCESS;
}

// Reports a device-side timeout of an earlier stream-ordered call (without
// waiting for the device).
int poll_pending(cail_dev_comm *dc) {
    if (!dc->pending || dc->status_h->code == 0) return MPI_SUCCESS;
    const DevStatus &s = *dc->status_h;
    CAIL_ERR("an earlier stream-ordered call failed: rank %d gave up after %ld ms waiting for %s %d "
             "(block %d, epoch %u, saw %u)", s.rank, cail_global_state.device_timeout_ms,
             s.waited_on >= 0 ? "rank" : "barrier", s.waited_on >= 0 ? s.waited_on : -1 - s.waited_on, s.block,
             s.epoch, s.seen);
    memset(dc->status_h, 0, sizeof(DevStatus));
    dc->broken = true;
    return MPI_ERR_OTHER;
}

// A one-shot call whose piece differs from the previous one-shot call's lays
// its slots out differently (the kernel's slot offsets scale with the
// piece), so it must not push while a peer still folds the previous call's
// last rounds.  Every rank waits for its own queued work, then all meet at
// a host barrier on the exchange segment.  Messages up to push_gmax x 8 KiB
// all have the 8 KiB piece and never come here.
bool peer_failed(const cail_dev_comm *dc, bool depart);

int oneshot_relayout(cail_dev_comm *dc) {
    if (cudaStreamSynchronize(dc->stream) != cudaSuccess) {
        CAIL_ERR("one_shot: waiting for the previous call failed");
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    if (dc->status_h->code != 0) return check_status(dc, "one_shot");  // reports an earlier timeout
    dc->pending = false;
    XSlot &me = dc->xs[dc->rank];
    const uint64_t seq = ++dc->xseq;
    me.arrive.store(seq, std::memory_order_release);
    int rc = host_wait(dc, false, seq);
    if (rc == MPI_SUCCESS && peer_failed(dc, false)) {
        // a peer gave up at this barrier: nobody may launch into its slots
        CAIL_ERR("one_shot: a peer failed at the barrier before a new slot layout; not launching");
        rc = MPI_ERR_OTHER;
    }
    me.depart.store(rc == MPI_SUCCESS ? seq : (seq | kXErr), std::memory_order_release);
    if (rc != MPI_SUCCESS) dc->broken = true;
    return rc;
}

int run_oneshot(cail_dev_comm *dc, const char *src, char *dst, size_t count, size_t esz, int op, int ec,
                bool allow_ordered) {
    const size_t bytes = count * esz;
    cail::OneShotArgs a;
    memset(&a, 0, sizeof(a));
    size_t piece = 0;
    oneshot_shape(bytes, dc->push_gmax, dc->os_piece_max, &piece, &a.G);
    if (dc->os_piece_last && piece != dc->os_piece_last) {
        const int rc = oneshot_relayout(dc);
        if (rc != MPI_SUCCESS) return rc;
    }
    dc->os_piece_last = piece;
    a.piece = piece;
    a.sg = dc->push_gmax;  // the area holds 3 x push_gmax x P x os_piece_max
    a.bytes = bytes;
    a.area = dc->os_area;
    a.P = dc->P;
    a.rank0 = dc->rank;
    a.vec = (((uintptr_t)src | (uintptr_t)dst) & 15) == 0 ? 1 : 0;
    a.src[dc->rank] = src;
    a.dst[dc->rank] = dst;
    a.rounds_done[dc->rank] = (uint32_t *)dc->ws + cail::kOsRoundsBase;
    for (int q = 0; q < dc->P; ++q) {
        a.slots[q] = dc->peer_ws[q] + kOsOff;
        a.flags[q] = (uint32_t *)dc->peer_ws[q];
    }
    a.timeout_ns = timeout_ns();
    a.status = dc->status_d;
    a.checks = cail_global_state.device_checks;
    double t = cail_global_state.profile ? cail_now_us() : 0.0;
    cudaError_t e = cail::launch_oneshot(op, ec, a, 1, false, dc->stream);
    cail_prof_mark(CAIL_PH_LAUNCH, t);
    cail_counters.launches++;
    if (e != cudaSuccess) {
        CAIL_ERR("one_shot launch failed: %s", cudaGetErrorString(e));
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    if (allow_ordered && stream_ordered_ok(dc)) return finish_stream_ordered(dc, "one_shot");
    return check_status(dc, "one_shot");
}

// ---- push two-shot over the IPC workspace (no host exchange)
// Fills the slice table and the launch shape of a push two-shot of `count`
// elements: slices cut at 16-byte units when every buffer is 16-byte
// aligned (the last slice takes the ragged tail), else at elements; pieces
// of at least CAIL_TWOSHOT_PIECE_MIN bytes so that small messages use few
// CTAs, at most the workspace's piece; G CTAs; rounds to cover the longest
// slice.  The same on every rank.
void push_shape(cail::PushArgs &a, int P, size_t count, size_t esz, bool vec, int gmax, size_t piece_max,
                size_t piece_min) {
    const size_t bytes = count * esz;
    const size_t unit = vec ? 16 : esz;
    const size_t nunits = bytes / unit;
    for (int q = 0; q < P; ++q) a.slice_off[q] = nunits * q / P * unit;
    a.slice_off[P] = bytes;
    size_t mx = 0;
    for (int q = 0; q < P; ++q) mx = std::max(mx, a.slice_off[q + 1] - a.slice_off[q]);
    a.max_slice = mx;
    size_t piece = (mx + gmax - 1) / gmax;
    piece = (piece + 15) / 16 * 16;
    piece = std::min(std::max(piece, piece_min), piece_max);
    a.piece = piece;
    size_t g = (mx + piece - 1) / piece;
    a.G = (int)std::max<size_t>(1, std::min<size_t>(g, (size_t)gmax));
    a.rounds = (int)((mx + (size_t)a.G * piece - 1) / ((size_t)a.G * piece));
    if (a.rounds < 1) a.rounds = 1;
    a.P = P;
    a.vec = vec ? 1 : 0;
}

int run_push(cail_dev_comm *dc, const char *src, char *dst, size_t count, size_t esz, int op, int ec,
             bool allow_ordered) {
    cail::PushArgs a;
    memset(&a, 0, sizeof(a));
    const bool vec = (((uintptr_t)src | (uintptr_t)dst) & 15) == 0;
    push_shape(a, dc->P, count, esz, vec, dc->push_gmax, dc->push_piece_max, push_piece_min_env());
    a.rank0 = dc->rank;
    a.src[dc->rank] = src;
    a.dst[dc->rank] = dst;
    for (int q = 0; q < dc->P; ++q) {
        a.rs[q] = dc->peer_ws[q] + kOsOff + dc->os_area;
        a.ag[q] = dc->peer_ws[q] + kOsOff + dc->os_area + dc->push_area;
        a.flags[q] = (uint32_t *)dc->peer_ws[q];
    }
    a.epoch0 = dc->push_epoch + 1;
    dc->push_epoch += (uint32_t)a.rounds;
    a.timeout_ns = timeout_ns();
    a.status = dc->status_d;
    a.area = dc->push_area;
    a.checks = cail_global_state.device_checks;
    double t = cail_global_state.profile ? cail_now_us() : 0.0;
    cudaError_t e = cail::launch_push(op, ec, a, 1, false, dc->stream);
    cail_prof_mark(CAIL_PH_LAUNCH, t);
    cail_counters.launches++;
    if (e != cudaSuccess) {
        CAIL_ERR("two_shot launch failed: %s", cudaGetErrorString(e));
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    if (allow_ordered && stream_ordered_ok(dc)) return finish_stream_ordered(dc, "two_shot");
    return check_status(dc, "two_shot");
}

// ---- two-shot over registered user buffers (zero-copy; host exchange of
// the buffers' IPC handles and host barriers around the kernel)
// ---- copy-engine two-shot
// Rank r owns slice r of the message (cut at 16-byte units).  For each chunk
// of its slice the copy engine pulls the P-1 peers' parts into local scratch
// (stream ce_pull), a fold kernel reduces them with the local part in rank
// order into this rank's output (ce_fold), and the copy engine pushes the
// result into every peer's output (ce_push); the three stages of successive
// chunks overlap.  Chunks rotate through CAIL_CE_BUFFERS (2..4, default 4)
// scratch buffers, and the pulls into a buffer wait for the fold that last
// read it.  Only copy engines touch NVLink: with both directions busy they
// move 773 GB/s per direction between two B200s, against 704 for SM stores
// and 664 for SM loads.  Each chunk costs 2(P-1) serial copies per engine,
// so the path loses to the SM two-shot as P grows (350 vs 655 GB/s at 8).
constexpr size_t kCeScratchMax = (size_t)512 << 20;

int ce_buffers() {
    static const int v = [] {
        const char *e = getenv("CAIL_CE_BUFFERS");
        int b = e ? atoi(e) : 4;
        return b >= 2 && b <= 4 ? b : 4;
    }();
    return v;
}

bool ce_ensure(cail_dev_comm *dc, size_t scratch) {
    bool ok = true;
    for (cudaStream_t *s : {&dc->ce_pull, &dc->ce_fold, &dc->ce_push})
        if (!*s) ok = ok && cudaStreamCreateWithFlags(s, cudaStreamNonBlocking) == cudaSuccess;
    for (int i = 0; i < 4; ++i) {
        if (!dc->ce_pulled[i]) ok = ok && cudaEventCreateWithFlags(&dc->ce_pulled[i], cudaEventDisableTiming) == cudaSuccess;
        if (!dc->ce_folded[i]) ok = ok && cudaEventCreateWithFlags(&dc->ce_folded[i], cudaEventDisableTiming) == cudaSuccess;
    }
    if (!dc->ce_start) ok = ok && cudaEventCreateWithFlags(&dc->ce_start, cudaEventDisableTiming) == cudaSuccess;
    if (!dc->ce_end) ok = ok && cudaEventCreateWithFlags(&dc->ce_end, cudaEventDisableTiming) == cudaSuccess;
    if (ok && dc->ce_scratch_bytes < scratch) {
        if (dc->ce_scratch) cudaFree(dc->ce_scratch);
        dc->ce_scratch = nullptr;
        dc->ce_scratch_bytes = 0;
        ok = cudaMalloc(&dc->ce_scratch, scratch) == cudaSuccess;
        if (ok) dc->ce_scratch_bytes = scratch;
    }
    return ok;
}

size_t ce_chunk_bytes(size_t slice_bytes, int P) {
    // CAIL_CE_CHUNK (bytes) overrides: a sixteenth of the slice, 2..32 MiB,
    // and at most the scratch bound over all buffers
    static const size_t env = [] {
        const char *e = getenv("CAIL_CE_CHUNK");
        return e ? (size_t)atoll(e) : (size_t)0;
    }();
    size_t c = env ? env : slice_bytes / 16;
    if (!env) c = c < ((size_t)2 << 20) ? ((size_t)2 << 20) : (c > ((size_t)32 << 20) ? ((size_t)32 << 20) : c);
    const size_t nb = (size_t)ce_buffers();
    if (P > 1 && c > kCeScratchMax / (nb * (size_t)(P - 1))) c = kCeScratchMax / (nb * (size_t)(P - 1));
    c = (c + (1 << 16) - 1) >> 16 << 16;  // 64 KiB units
    return c ? c : (size_t)1 << 16;
}

int ce_body(cail_dev_comm *dc, const char *const *srcs, char *const *dsts, size_t count, size_t esz, int op,
            int ec) {
    const int P = dc->P, r = dc->rank;
    const size_t unit = 16 / esz;
    const size_t nunits = count / unit;
    const size_t lo = nunits * r / P * unit;
    const size_t hi = r == P - 1 ? count : nunits * (r + 1) / P * unit;
    const size_t chunk = ce_chunk_bytes((hi - lo) * esz, P);
    const size_t celems = chunk / esz;
    const int nb = ce_buffers();
    const size_t scratch = P > 1 ? (size_t)nb * (size_t)(P - 1) * chunk : 16;
    if (!ce_ensure(dc, scratch)) {
        CAIL_ERR("ce_two_shot: cannot create streams, events or %zu bytes of scratch", scratch);
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    double tl = cail_global_state.profile ? cail_now_us() : 0.0;
    bool ok = cudaEventRecord(dc->ce_start, dc->stream) == cudaSuccess;
    for (cudaStream_t s : {dc->ce_pull, dc->ce_fold, dc->ce_push})
        ok = ok && cudaStreamWaitEvent(s, dc->ce_start, 0) == cudaSuccess;
    size_t c = 0;
    for (size_t off = lo; ok && off < hi; off += celems, ++c) {
        const size_t n = hi - off < celems ? hi - off : celems;
        const int buf = (int)(c % (size_t)nb);
        char *base = P > 1 ? dc->ce_scratch + (size_t)buf * (size_t)(P - 1) * chunk : dc->ce_scratch;
        if (c >= (size_t)nb) ok = ok && cudaStreamWaitEvent(dc->ce_pull, dc->ce_folded[buf], 0) == cudaSuccess;
        cail::FoldArgs f;
        memset(&f, 0, sizeof(f));
        f.P = P;
        f.count = n;
        f.dst = dsts[r] + off * esz;
        for (int q = 0, s = 0; q < P; ++q) {
            if (q == r) {
                f.src[q] = srcs[r] + off * esz;
                continue;
            }
            char *slot = base + (size_t)s++ * chunk;
            f.src[q] = slot;
            ok = ok && cudaMemcpyAsync(slot, srcs[q] + off * esz, n * esz, cudaMemcpyDefault, dc->ce_pull) == cudaSuccess;
        }
        ok = ok && cudaEventRecord(dc->ce_pulled[buf], dc->ce_pull) == cudaSuccess;
        ok = ok && cudaStreamWaitEvent(dc->ce_fold, dc->ce_pulled[buf], 0) == cudaSuccess;
        const size_t want = (n * esz / 16 + 1023) / 1024;
        const int blocks = (int)(want < 1 ? 1 : (want > (size_t)dc->sms * 2 ? (size_t)dc->sms * 2 : want));
        ok = ok && cail::launch_fold(op, ec, f, blocks, 512, dc->ce_fold) == cudaSuccess;
        cail_counters.launches++;
        ok = ok && cudaEventRecord(dc->ce_folded[buf], dc->ce_fold) == cudaSuccess;
        ok = ok && cudaStreamWaitEvent(dc->ce_push, dc->ce_folded[buf], 0) == cudaSuccess;
        for (int q = 0; q < P; ++q)
            if (q != r)
                ok = ok && cudaMemcpyAsync(dsts[q] + off * esz, dsts[r] + off * esz, n * esz, cudaMemcpyDefault,
                                           dc->ce_push) == cudaSuccess;
    }
    ok = ok && cudaEventRecord(dc->ce_end, dc->ce_push) == cudaSuccess;
    ok = ok && cudaStreamWaitEvent(dc->stream, dc->ce_end, 0) == cudaSuccess;
    cail_prof_mark(CAIL_PH_LAUNCH, tl);
    if (!ok) {
        CAIL_ERR("ce_two_shot: enqueue failed: %s", cudaGetErrorString(cudaGetLastError()));
        cudaStreamSynchronize(dc->ce_push);
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    return check_status(dc, "ce_two_shot");
}

// A datatype of storage class ec (the reduction depends only on the class).
cail_datatype_t dtype_of_class(int ec) {
    static const cail_datatype_t t[CAIL_EC_NUM] = {CAIL_CHAR, CAIL_UCHAR, CAIL_SHORT, CAIL_USHORT, CAIL_INT,
                                                   CAIL_UINT, CAIL_LONG_LONG, CAIL_ULONGLONG, CAIL_FLOAT, CAIL_DOUBLE};
    return ec >= 0 && ec < CAIL_EC_NUM ? t[ec] : CAIL_INVALID;
}

// 1 if a peer published kXErr in its arrive (depart) word for this call.
bool peer_failed(const cail_dev_comm *dc, bool depart) {
    for (int q = 0; q < dc->P; ++q) {
        const std::atomic<uint64_t> &a = depart ? dc->xs[q].depart : dc->xs[q].arrive;
        if (a.load(std::memory_order_acquire) & kXErr) return true;
    }
    return false;
}

// Host-side fault injection (tests only): CAIL_FI_TWOSHOT_FAIL=<rank> makes
// that rank's import of its peers' buffers fail, as a failing
// cudaIpcOpenMemHandle would.
int fi_twoshot_fail_rank() {
    static const int v = [] {
        const char *e = getenv("CAIL_FI_TWOSHOT_FAIL");
        return e && *e ? atoi(e) : -1;
    }();
    return v;
}

// A rank that fails between the host barriers still takes part in both, with
// kXErr set, so no peer waits forever and no peer reports a result whose
// slice of the failed rank was never reduced.
int run_twoshot(cail_dev_comm *dc, const char *src, char *dst, size_t count, size_t esz, int op, int ec,
                bool ce = false) {
    XSlot &me = dc->xs[dc->rank];
    // Peers read this rank's buffers as soon as it arrives, so its pending
    // legacy-stream writes must have landed first.
    bool pre_ok = true;
    if (cail_global_state.stream_sync && cudaEventSynchronize(dc->legacy_ev) != cudaSuccess) {
        CAIL_ERR("two_shot: waiting for the legacy stream failed");
        pre_ok = false;
    }
    describe(dc, src, &me.send);
    describe(dc, dst, &me.recv);
    uint64_t seq = ++dc->xseq;
    me.arrive.store(pre_ok ? seq : (seq | kXErr), std::memory_order_release);
    double th = cail_global_state.profile ? cail_now_us() : 0.0;
    int rc = host_wait(dc, false, seq);
    th = cail_prof_mark(CAIL_PH_HOSTSYNC, th);
    if (rc != MPI_SUCCESS) {
        dc->broken = true;
        return rc;
    }
    bool all_ok = true;
    for (int q = 0; q < dc->P; ++q) all_ok = all_ok && dc->xs[q].send.ok && dc->xs[q].recv.ok;
    if (!pre_ok || peer_failed(dc, false)) {
        if (pre_ok) CAIL_ERR("two_shot: a peer failed before the exchange; not launching");
        rc = MPI_ERR_OTHER;
        goto depart;
    }
    if (!all_ok) {
        // some rank's buffer cannot be exported: every rank sees the same
        // descriptors and takes the copy-in path instead
        if (dc->shared_gpu) {
            // (test mode, ranks on one GPU: no kernel that waits on peers)
            rc = PMPI_Allreduce(src == dst ? MPI_IN_PLACE : src, dst, (int)count,
                                cail_dtype_to_mpi_type(dtype_of_class(ec)),
                                cail_optype_to_mpi_op((cail_op_t)op), dc->comm);
        } else {
            rc = run_oneshot(dc, src, dst, count, esz, op, ec, false);
        }
    } else {
        cail::TwoShotArgs a;
        memset(&a, 0, sizeof(a));
        a.P = dc->P;
        a.rank = dc->rank;
        a.count = count;
        bool bad = false;
        for (int q = 0; q < dc->P; ++q) {
            if (q == dc->rank) {
                a.src[q] = src;
                a.dst[q] = dst;
                continue;
            }
            a.src[q] = import_buf(dc, q, dc->xs[q].send);
            a.dst[q] = import_buf(dc, q, dc->xs[q].recv);
            if (!a.src[q] || !a.dst[q]) bad = true;
        }
        if (dc->rank == fi_twoshot_fail_rank()) {
            CAIL_ERR("two_shot: injected import failure (CAIL_FI_TWOSHOT_FAIL)");
            bad = true;
        }
        if (bad) {
            rc = MPI_ERR_OTHER;
            goto depart;
        }
        if (ce) {
            rc = ce_body(dc, a.src, a.dst, count, esz, op, ec);
            goto depart;
        }
        {
        uint64_t mis = (uint64_t)(uintptr_t)src & 15;
        bool vec_ok = true;
        for (int q = 0; q < dc->P; ++q)
            if (((uintptr_t)a.src[q] & 15) != mis || ((uintptr_t)a.dst[q] & 15) != mis) vec_ok = false;
        a.vector_ok = vec_ok ? 1 : 0;
        if (vec_ok) {
            size_t head = ((16 - mis) & 15) / esz;
            if (head > count) head = count;
            a.head = head;
            a.nvec = (count - head) * esz / 16;
        }
        size_t work = vec_ok ? a.nvec / dc->P + 1 : count / dc->P + 1;
        int threads = 512;
        size_t want = (work + threads - 1) / threads;
        // Measured on B200 (1 GiB): at 2 ranks two vectors per iteration with
        // one 512-thread CTA per SM moves ~5% more than one vector with two
        // CTAs per SM; at 8 ranks (8 loads per vector already) it moves 8%
        // less (604 vs 655 GB/s), and for one rank (a local copy) 7% less
        // (0.473 vs 0.441 ms).  Below 128 MiB the plain loop is as fast or
        // faster.  CAIL_TWOSHOT_CTAS_PER_SM / CAIL_TWOSHOT_UNROLL (1 or 2)
        // override.
        static const int env_per_sm = [] {
            const char *e = getenv("CAIL_TWOSHOT_CTAS_PER_SM");
            int v = e ? atoi(e) : 0;
            return v >= 1 && v <= 4 ? v : 0;
        }();
        static const int env_unroll = [] {
            const char *e = getenv("CAIL_TWOSHOT_UNROLL");
            return e ? atoi(e) : 0;
        }();
        const bool big = count * esz >= ((size_t)128 << 20) && dc->P >= 2 && dc->P <= 4;
        a.unroll2 = env_unroll ? (env_unroll >= 2 ? 1 : 0) : (big ? 1 : 0);
        int per_sm = env_per_sm ? env_per_sm : (a.unroll2 ? 1 : 2);
        int maxb = dc->sms * per_sm;
        int blocks = (int)(want < 1 ? 1 : (want > (size_t)maxb ? maxb : want));
        double tl = cail_global_state.profile ? cail_now_us() : 0.0;
        cudaError_t e = cail::launch_twoshot(op, ec, a, blocks, threads, dc->stream);
        cail_prof_mark(CAIL_PH_LAUNCH, tl);
        cail_counters.launches++;
        if (e != cudaSuccess) {
            CAIL_ERR("two_shot launch failed: %s", cudaGetErrorString(e));
            rc = MPI_ERR_OTHER;
        } else {
            rc = check_status(dc, "two_shot");
        }
        }
    }
depart:
    // depart: peers may only return (and reuse their buffers) once every
    // rank's kernel has finished reading and writing them
    me.depart.store(rc == MPI_SUCCESS ? seq : (seq | kXErr), std::memory_order_release);
    th = cail_global_state.profile ? cail_now_us() : 0.0;
    int rc2 = host_wait(dc, true, seq);
    cail_prof_mark(CAIL_PH_HOSTSYNC, th);
    if (rc == MPI_SUCCESS && rc2 == MPI_SUCCESS && peer_failed(dc, true)) {
        CAIL_ERR("two_shot: a peer failed during the call; the result is incomplete");
        rc2 = MPI_ERR_OTHER;
    }
    if (rc != MPI_SUCCESS || rc2 != MPI_SUCCESS) dc->broken = true;
    return rc != MPI_SUCCESS ? rc : rc2;
}

// ---- NVLS
// One launch; every CTA runs its own pipeline over units of at most
// CAIL_NVLS_UNIT bytes (see NvlsArgs).  The unit shrinks for small messages
// so that every CTA has work, in 64 KiB steps down to 16 KiB.
int run_nvls(cail_dev_comm *dc, const char *src, char *dst, size_t count, size_t esz, int op, int ec,
             bool allow_ordered) {
    const size_t bytes = count * esz;
    size_t unit = 0;
    int blocks = 0;
    nvls_shape(bytes, dc->nvls_blocks, dc->nvls_unit, &unit, &blocks);
    cail::NvlsArgs a;
    memset(&a, 0, sizeof(a));
    a.src = src;
    a.dst = dst;
    a.uc = (char *)dc->uc_va + kNvlsCtrRegion;
    a.mc = (char *)dc->mc_va + kNvlsCtrRegion;
    a.mc_ctr = (char *)dc->mc_va;
    a.uc_ctr = (const char *)dc->uc_va;
    a.steps = (uint32_t *)(dc->ws + kNvlsStepsOff);
    a.bytes = bytes;
    a.unit = unit;
    a.area = dc->nvls_size - kNvlsCtrRegion;
    a.P = dc->P;
    a.rank = dc->rank;
    a.timeout_ns = timeout_ns();
    a.status = dc->status_d;
    a.checks = cail_global_state.device_checks;
    double t = cail_global_state.profile ? cail_now_us() : 0.0;
    cudaError_t e = cail::launch_nvls(op, ec, a, blocks, dc->stream);
    cail_prof_mark(CAIL_PH_LAUNCH, t);
    cail_counters.launches++;
    if (e != cudaSuccess) {
        CAIL_ERR("nvls launch failed: %s", cudaGetErrorString(e));
        dc->broken = true;
        return MPI_ERR_OTHER;
    }
    if (allow_ordered && stream_ordered_ok(dc)) return finish_stream_ordered(dc, "nvls");
    return check_status(dc, "nvls");
}

// Which two-shot kernel runs for P ranks: the zero-copy kernel over the user
// buffers (host exchange of their IPC handles, host barriers) or the push
// kernel over the workspace (no host step).  CAIL_TWOSHOT_ZEROCOPY=1 / =0
// forces one.  Measured on B200 (blocking calls, float sum), the zero-copy
// kernel leads at every size from 128 KiB: at 2 ranks 20.2 vs 29.7 us at
// 1 MiB and 659 vs 662 GB/s at 1 GiB; at 8 ranks 30.2 vs 38.5 us at 1 MiB,
// 74.8 vs 102.6 us at 16 MiB and 650 vs 557 GB/s at 1 GiB.  Its host
// barrier costs a few microseconds even with 8 processes, and it moves about
// 2N bytes through HBM per rank against about 6N for the push kernel (which
// stages through the workspace).  The push kernel runs when calls complete
// in stream order (cail_set_stream_ordered), which a host barrier cannot.
int twoshot_zero_copy_env() {
    static const int v = [] {
        const char *e = getenv("CAIL_TWOSHOT_ZEROCOPY");
        return e && *e ? (*e != '0' ? 1 : 0) : -1;
    }();
    return v;
}

bool twoshot_zero_copy(const cail_dev_comm *dc) {
    const int env = twoshot_zero_copy_env();
    if (env >= 0) return env == 1;
    return !stream_ordered_ok(dc);
}

// Built-in one_shot / two_shot crossover per rank count, measured on B200
// (blocking calls, float sum): 2 ranks, one-shot and zero-copy two-shot
// equal up to 64 KiB (20.2 us), two-shot ahead from 128 KiB; 4 ranks, equal
// at 64 KiB (23.6 vs 23.9 us), two-shot ahead from 128 KiB (24.4 vs 26.1 us
// at 256 KiB); 8 ranks, one-shot ahead up to 256 KiB (28.2 vs 29.0 us),
// two-shot from 512 KiB (27.8 vs 31.8 us).  CAIL_TUNE_FILE lines replace it
// per rank count.
size_t default_oneshot_max(int P) {
    if (P <= 4) return 64 << 10;
    return 256 << 10;
}

// NVLS moves about N(1 + 1/P) bytes per GPU and direction plus a local
// copy-in and copy-out, against 2N(P-1)/P for two-shot: it can only win at
// large P and large messages.  Measured on B200 (float sum, 1 MiB units):
// 8 ranks, 713 GB/s bus bandwidth at 1 GiB against 650 for the zero-copy
// two-shot, but 637 vs 656 at 512 MiB and 550 vs 641 at 256 MiB; 2 ranks,
// 354 vs 659 at 1 GiB.  Built in: NVLS from 8 ranks and 1 GiB.
// CAIL_NVLS_MIN_RANKS (0: never) and CAIL_NVLS_MIN (bytes) replace both
// bounds; a CAIL_TUNE_FILE line for P replaces them for that rank count.
constexpr int kNvlsDefaultMinRanks = 8;
constexpr size_t kNvlsDefaultMinBytes = (size_t)1 << 30;

size_t nvls_min_bytes() {
    static const size_t v = [] {
        const char *e = getenv("CAIL_NVLS_MIN");
        return e && *e ? (size_t)atoll(e) : kNvlsDefaultMinBytes;
    }();
    return v;
}

// Auto mode hands messages of at least CAIL_CE_MIN bytes to the
// copy-engine two-shot (~0 when unset).
size_t ce_min_bytes() {
    static const size_t v = [] {
        const char *e = getenv("CAIL_CE_MIN");
        return e ? (size_t)atoll(e) : ~(size_t)0;
    }();
    return v;
}

// CAIL_NVLS_MIN_RANKS, or -1 when it is not set.
int nvls_min_ranks_env() {
    static const int v = [] {
        const char *e = getenv("CAIL_NVLS_MIN_RANKS");
        return e && *e ? atoi(e) : -1;
    }();
    return v;
}

// Smallest rank count for which auto mode uses NVLS (0: never) on a
// communicator of P ranks without a tune-file line.
int nvls_min_ranks() {
    const int e = nvls_min_ranks_env();
    return e >= 0 ? e : kNvlsDefaultMinRanks;
}

// Auto mode on an NVLink communicator of P ranks; nvls_pair: NVLS is set up
// and multimem can reduce the call's (type, op).  Depends only on its
// arguments and the environment.
// Precedence for each crossover: its environment variable, then the
// CAIL_TUNE_FILE line for P, then the built-in default.
int pick_nvlink(int P, size_t bytes, bool nvls_pair) {
    const cail_state_t &s = cail_global_state;
    const cail_tune_t *t = cail_tune_for(P);
    size_t one_max = s.oneshot_max ? s.oneshot_max
                     : s.msg_small_threshold_set ? s.msg_small_threshold - 1
                     : (t && t->oneshot_max >= 0) ? (size_t)t->oneshot_max
                                                  : default_oneshot_max(P);
    if (bytes <= one_max) return CAIL_ALGO_ONE_SHOT;
    if (nvls_pair) {
        if (nvls_min_ranks_env() < 0 && t) {
            if (t->nvls_min >= 0 && bytes >= (size_t)t->nvls_min) return CAIL_ALGO_NVLS;
        } else if (nvls_min_ranks() > 0 && P >= nvls_min_ranks() && bytes >= nvls_min_bytes()) {
            return CAIL_ALGO_NVLS;
        }
    }
    if (ce_min_bytes() != ~(size_t)0) {
        if (bytes >= ce_min_bytes()) return CAIL_ALGO_CE_TWO_SHOT;
    } else if (t && t->ce_min >= 0 && bytes >= (size_t)t->ce_min) {
        return CAIL_ALGO_CE_TWO_SHOT;
    }
    return CAIL_ALGO_TWO_SHOT;
}

}  // namespace

// ---------------------------------------------------------------- public
extern "C" {

cail_dev_comm *cail_dev_comm_get(MPI_Comm comm) {
    if (g_keyval == MPI_KEYVAL_INVALID &&
        PMPI_Comm_create_keyval(MPI_COMM_NULL_COPY_FN, delete_cb, &g_keyval, nullptr) != MPI_SUCCESS)
        return nullptr;
    void *val = nullptr;
    int flag = 0;
    PMPI_Comm_get_attr(comm, g_keyval, &val, &flag);
    cail_dev_comm *dc = flag ? static_cast<cail_dev_comm *>(val) : nullptr;
    if (!dc) {
        dc = create_context(comm);
        g_contexts.push_back(dc);
        PMPI_Comm_set_attr(comm, g_keyval, dc);
    }
    return dc->ok ? dc : nullptr;
}

int cail_dev_nvls_ok(cail_dev_comm *dc, cail_datatype_t dt, cail_op_t op) {
    if (!dc || !dc->nvls) return 0;
    return cail::nvls_supported((int)op, (int)cail_elem_class(dt));
}

int cail_dev_pick_algo(cail_dev_comm *dc, size_t bytes, int count, cail_datatype_t dt, cail_op_t op) {
    (void)count;
    if (dc->shared_gpu) return CAIL_ALGO_TWO_SHOT;  // test mode: the only kernel that may share a GPU
    return pick_nvlink(dc->P, bytes, cail_dev_nvls_ok(dc, dt, op) != 0);
}

const char *cail_nvlink_auto_algorithm(int nranks, size_t bytes, MPI_Datatype datatype, MPI_Op op) {
    if (nranks < 1 || !cail_type_supported(datatype) || !cail_op_supported(op)) return nullptr;
    cail_load_config();
    const cail_datatype_t dt = cail_mpi_type_to_dtype(datatype);
    const cail_op_t o = cail_mpi_op_to_optype(op);
    const bool pair = cail_global_state.nvls && cail::nvls_supported((int)o, (int)cail_elem_class(dt));
    return cail_algo_name(pick_nvlink(nranks, bytes, pair));
}

int cail_dev_allreduce(cail_dev_comm *dc, int algo, const void *sendbuf, void *recvbuf, int count,
                       cail_datatype_t dt, cail_op_t op) {
    if (dc->broken) {
        CAIL_ERR("nvlink context of this communicator failed earlier; refusing further calls");
        return MPI_ERR_OTHER;
    }
    if (poll_pending(dc) != MPI_SUCCESS) return MPI_ERR_OTHER;
    // A rank that left the job is noticed on the host before the next launch
    // (checked at most every 10 ms, so back-to-back calls pay nothing).
    double now = cail_now_us();
    if (now - dc->last_live_check > 10000.0) {
        dc->last_live_check = now;
        for (int q = 0; q < dc->P; ++q) {
            if (q != dc->rank && process_gone(dc->peer_pid[q])) {
                CAIL_ERR("rank %d: peer rank %d (pid %d) has exited; not launching", dc->rank, q,
                         dc->peer_pid[q]);
                dc->broken = true;
                return MPI_ERR_OTHER;
            }
        }
    }
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != dc->dev) cudaSetDevice(dc->dev);
    const size_t esz = (size_t)cail_type_size(dt);
    const char *src = (const char *)(sendbuf == MPI_IN_PLACE ? recvbuf : sendbuf);
    char *dst = (char *)recvbuf;
    const int ec = (int)cail_elem_class(dt);
    int rc = MPI_SUCCESS;
    const double ts = cail_global_state.profile ? cail_now_us() : 0.0;
    if (cail_global_state.stream_sync) {
        cudaEventRecord(dc->legacy_ev, cudaStreamLegacy);
        cudaStreamWaitEvent(dc->stream, dc->legacy_ev, 0);
    }
    cail_prof_mark(CAIL_PH_SETUP, ts);
    if (dc->shared_gpu && algo != CAIL_ALGO_CE_TWO_SHOT) {
        rc = run_twoshot(dc, src, dst, (size_t)count, esz, (int)op, ec);  // ranks share a GPU (test mode)
    } else if (algo == CAIL_ALGO_ONE_SHOT) {
        rc = run_oneshot(dc, src, dst, (size_t)count, esz, (int)op, ec, true);
    } else if (algo == CAIL_ALGO_NVLS && cail_dev_nvls_ok(dc, dt, op)) {
        rc = run_nvls(dc, src, dst, (size_t)count, esz, (int)op, ec, true);
    } else if (algo == CAIL_ALGO_CE_TWO_SHOT) {
        rc = run_twoshot(dc, src, dst, (size_t)count, esz, (int)op, ec, true);
    } else if (twoshot_zero_copy(dc)) {
        rc = run_twoshot(dc, src, dst, (size_t)count, esz, (int)op, ec);
    } else {
        rc = run_push(dc, src, dst, (size_t)count, esz, (int)op, ec, true);
    }
    if (prev >= 0 && prev != dc->dev) cudaSetDevice(prev);
    return rc;
}

void cail_dev_finalize_all(void) {
    // Deleting the attribute runs delete_cb, which destroys the context.
    std::vector<cail_dev_comm *> all = g_contexts;
    for (cail_dev_comm *dc : all) {
        if (dc->ok) PMPI_Barrier(dc->comm);
        PMPI_Comm_delete_attr(dc->comm, g_keyval);
    }
    g_contexts.clear();
    if (g_keyval != MPI_KEYVAL_INVALID) PMPI_Comm_free_keyval(&g_keyval);
}

// Test hook: the launch shape an NVLink path computes for a call, without a
// GPU (the tests check its invariants over many sizes).  kind 0: one-shot,
// out = {G, piece, area}; kind 1: push two-shot, out = {G, piece, rounds,
// max_slice, area, slice_off[0..P]}; kind 2: NVLS, out = {blocks, unit,
// staging bytes}.  gmax: CTAs per rank (two per SM on B200: 296); vec: the
// buffers are 16-byte aligned.  Returns the number of values written, or -1.
int cail_dev_plan(int kind, int P, size_t count, size_t esz, int vec, int gmax, unsigned long long *out, int nout) {
    if (P < 2 || P > kMaxRanks || gmax < 1 || gmax > cail::kMaxBlocks || !out) return -1;
    const size_t bytes = count * esz;
    if (kind == 0) {
        if (nout < 5) return -1;
        size_t piece = 0;
        int G = 0;
        oneshot_shape(bytes, gmax, os_piece_max_for(P, gmax), &piece, &G);
        out[0] = (unsigned long long)G;
        out[1] = piece;
        out[2] = os_area_for(P, gmax, os_piece_max_for(P, gmax));
        out[3] = (unsigned long long)gmax;  // slot stride in CTAs (run_oneshot: a.sg)
        out[4] = os_piece_max_for(P, gmax);  // the largest piece the area holds
        return 5;
    }
    if (kind == 1) {
        if (nout < 5 + P + 1) return -1;
        cail::PushArgs a;
        memset(&a, 0, sizeof(a));
        const size_t pm = push_piece_max_for(P, gmax);
        push_shape(a, P, count, esz, vec != 0, gmax, pm, push_piece_min_env());
        out[0] = (unsigned long long)a.G;
        out[1] = a.piece;
        out[2] = (unsigned long long)a.rounds;
        out[3] = a.max_slice;
        out[4] = push_area_for(P, gmax, pm);
        for (int q = 0; q <= P; ++q) out[5 + q] = a.slice_off[q];
        return 5 + P + 1;
    }
    if (kind == 2) {
        if (nout < 3) return -1;
        size_t unit = 0;
        int blocks = 0;
        nvls_shape(bytes, gmax, kDefaultNvlsUnit, &unit, &blocks);
        out[0] = (unsigned long long)blocks;
        out[1] = unit;
        out[2] = (unsigned long long)gmax * 2 * kDefaultNvlsUnit;
        return 3;
    }
    return -1;
}

// Self-test of the bounded device wait, on one GPU: a one-shot kernel for
// two ranks whose peer never arrives (its flag is never written).  The
// kernel must give up after timeout_ms and report DevStatus code 1; the
// context stays usable.  Returns the status code, or -1 on a CUDA error.
int cail_test_device_timeout(int timeout_ms) {
    char *ws = nullptr;
    DevStatus *st_h = nullptr, *st_d = nullptr;
    cudaStream_t s = nullptr;
    int code = -1;
    // layout: [flags of rank 0][flags of rank 1][src 16 KiB][dst 16 KiB]
    // [one-shot area of rank 0][of rank 1]; only rank 0's CTA runs, so rank 1
    // never raises its flag
    const size_t part = 16 << 10, piece = 16 << 10;
    const size_t area = (size_t)cail::kOsSlots * 1 * 2 * piece;
    const size_t total = 2 * kFlagBytes + 2 * part + 2 * area;
    if (cudaMalloc(&ws, total) == cudaSuccess && cudaMemset(ws, 0, total) == cudaSuccess &&
        cudaHostAlloc((void **)&st_h, sizeof(DevStatus), cudaHostAllocMapped) == cudaSuccess &&
        cudaHostGetDevicePointer((void **)&st_d, st_h, 0) == cudaSuccess &&
        cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) == cudaSuccess) {
        memset(st_h, 0, sizeof(DevStatus));
        cail::OneShotArgs a;
        memset(&a, 0, sizeof(a));
        a.flags[0] = (uint32_t *)ws;
        a.flags[1] = (uint32_t *)(ws + kFlagBytes);
        a.src[0] = ws + 2 * kFlagBytes;
        a.dst[0] = ws + 2 * kFlagBytes + part;
        a.slots[0] = ws + 2 * kFlagBytes + 2 * part;
        a.slots[1] = ws + 2 * kFlagBytes + 2 * part + area;
        a.rounds_done[0] = (uint32_t *)ws + cail::kOsRoundsBase;
        a.bytes = part;
        a.piece = piece;
        a.sg = 1;
        a.area = area;
        a.P = 2;
        a.rank0 = 0;
        a.G = 1;
        a.vec = 1;
        a.timeout_ns = (unsigned long long)timeout_ms * 1000000ull;
        a.status = st_d;
        if (cail::launch_oneshot(CAIL_SUM, CAIL_EC_F32, a, 1, false, s) == cudaSuccess &&
            cudaStreamSynchronize(s) == cudaSuccess)
            code = st_h->code;
    }
    cudaGetLastError();
    if (s) cudaStreamDestroy(s);
    if (st_h) cudaFreeHost(st_h);
    if (ws) cudaFree(ws);
    return code;
}

int cail_comm_uses_nvlink(MPI_Comm comm) {
    if (g_keyval == MPI_KEYVAL_INVALID) return 0;
    void *val = nullptr;
    int flag = 0;
    PMPI_Comm_get_attr(comm, g_keyval, &val, &flag);
    return flag && val && static_cast<cail_dev_comm *>(val)->ok ? 1 : 0;
}

int cail_comm_uses_nvls(MPI_Comm comm) {
    if (g_keyval == MPI_KEYVAL_INVALID) return 0;
    void *val = nullptr;
    int flag = 0;
    PMPI_Comm_get_attr(comm, g_keyval, &val, &flag);
    return flag && val && static_cast<cail_dev_comm *>(val)->nvls ? 1 : 0;
}

}  // extern "C"
