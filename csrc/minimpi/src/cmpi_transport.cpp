// cmpi_transport.cpp — job bootstrap, shared-memory channels and the
// point-to-point progress engine of minimpi.
//
// Bootstrap modes (first match wins):
//   launcher : CMPI_SHM, CMPI_RANK, CMPI_SIZE set by cail-mpirun, which has
//              already created and initialised the segment;
//   torchrun : RANK / WORLD_SIZE (and MASTER_PORT) set by
//              torch.distributed.run; rank 0 creates the segment
//              "/cmpi_t<agent pid>_<port>_<restart>" and stamps it with the
//              agent's start time so stale segments are recognised;
//   singleton: neither; a one-rank world without shared memory.
// Rank 0 unlinks the segment name once every rank has joined, so a crashed
// job leaves nothing behind in /dev/shm.
#include "cmpi_internal.h"

#include <errno.h>
#include <fcntl.h>
#include <sched.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <time.h>
#include <unistd.h>

#include <algorithm>
#include <cstdlib>
#include <fstream>
#include <sstream>

namespace cmpi {

int g_world_rank = 0;

double now_s() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

uint64_t node_id() {
    char host[256] = {0};
    gethostname(host, sizeof(host) - 1);
    uint64_t h = 1469598103934665603ull;  // FNV-1a
    for (const char *p = host; *p; ++p) { h ^= (unsigned char)*p; h *= 1099511628211ull; }
    return h;
}

// ------------------------------------------------------------------ engine
struct PeerOut {
    std::deque<Request *> q;      // messages in posting order
    std::deque<PktHdr> ctrl;      // ACK packets, sent between messages
};

struct PeerIn {
    bool have_hdr = false;
    PktHdr h{};
    uint64_t got = 0;
    Request *tgt = nullptr;
    Unexpected *ux = nullptr;
    RndvDesc desc{};
};

struct Engine {
    bool up = false;
    int rank = 0, size = 1;
    char *base = nullptr;
    size_t map_bytes = 0;
    SegHeader *hdr = nullptr;
    RankSlot *slots = nullptr;
    ChanCtl *ctl = nullptr;
    char *data = nullptr;
    uint32_t ring = 0;
    std::string shm_name;
    std::vector<PeerOut> out;
    std::vector<PeerIn> in;
    std::vector<uint64_t> head_cache, tail_cache;  // my head per out-chan, my tail per in-chan
    std::list<Request *> posted;
    std::list<Unexpected *> unexpected;
    std::map<uint64_t, Request *> rndv_pending;
    uint64_t next_rid = 1;
    // health
    double last_health = 0.0;
    double timeout_s = 0.0;
    // fault injection
    int fi_rank = -1;
    long fi_at = 1;
    long calls = 0;
    std::string fi_action;
    int fi_code = 3;
    bool fi_drop_next = false;
};

static Engine g_engine;
Engine &engine() { return g_engine; }
bool transport_up() { return g_engine.up; }
int world_size() { return g_engine.size; }

static inline ChanCtl &chan(int s, int d) { return g_engine.ctl[(size_t)s * g_engine.size + d]; }
static inline char *ring_of(int s, int d) {
    return g_engine.data + ((size_t)s * g_engine.size + d) * g_engine.ring;
}

static uint64_t parent_start_time(pid_t ppid) {
    std::ifstream f("/proc/" + std::to_string(ppid) + "/stat");
    std::string s((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    size_t rp = s.rfind(')');
    if (rp == std::string::npos) return 0;
    std::istringstream is(s.substr(rp + 2));
    std::string tok;
    // fields after the command: state(3) ... starttime is field 22
    for (int field = 3; field <= 22 && (is >> tok); ++field)
        if (field == 22) return strtoull(tok.c_str(), nullptr, 10);
    return 0;
}

static int map_segment(int fd, size_t bytes) {
    void *p = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    if (p == MAP_FAILED) return -1;
    Engine &e = g_engine;
    e.base = (char *)p;
    e.map_bytes = bytes;
    e.hdr = (SegHeader *)e.base;
    e.slots = (RankSlot *)(e.base + sizeof(SegHeader));
    e.ctl = (ChanCtl *)(e.base + sizeof(SegHeader) + sizeof(RankSlot) * e.size);
    e.data = e.base + sizeof(SegHeader) + sizeof(RankSlot) * e.size +
             sizeof(ChanCtl) * (size_t)e.size * e.size;
    return 0;
}

static int env_int(const char *name, int dflt) {
    const char *v = getenv(name);
    return (v && *v) ? atoi(v) : dflt;
}

static void setup_fault_injection() {
    Engine &e = g_engine;
    e.fi_rank = env_int("CMPI_FI_RANK", -1);
    e.fi_at = env_int("CMPI_FI_AT_CALL", 1);
    const char *a = getenv("CMPI_FI_ACTION");
    e.fi_action = a ? a : "";
    e.fi_code = env_int("CMPI_FI_EXIT_CODE", 3);
    const char *t = getenv("CMPI_TIMEOUT_S");
    e.timeout_s = t ? atof(t) : 0.0;
}

int init_transport(int *wr, int *ws) {
    Engine &e = g_engine;
    setup_fault_injection();
    const char *shm = getenv("CMPI_SHM");
    const char *trank = getenv("RANK");
    const char *tsize = getenv("WORLD_SIZE");
    bool launcher = shm && getenv("CMPI_RANK") && getenv("CMPI_SIZE");
    bool torchrun = !launcher && trank && tsize && atoi(tsize) > 1;
    if (!launcher && !torchrun) {
        e.rank = 0;
        e.size = 1;
        e.up = true;
        *wr = 0;
        *ws = 1;
        g_world_rank = 0;
        return MPI_SUCCESS;
    }
    int fd = -1;
    double deadline = now_s() + env_int("CMPI_JOIN_TIMEOUT_S", 120);
    if (launcher) {
        e.rank = atoi(getenv("CMPI_RANK"));
        e.size = atoi(getenv("CMPI_SIZE"));
        e.shm_name = shm;
        fd = shm_open(shm, O_RDWR, 0600);
        if (fd < 0) {
            std::fprintf(stderr, "[minimpi] cannot open job segment %s: %s\n", shm, strerror(errno));
            return MPI_ERR_INTERN;
        }
        struct stat st;
        fstat(fd, &st);
        e.size = atoi(getenv("CMPI_SIZE"));
        if (map_segment(fd, (size_t)st.st_size) != 0) { close(fd); return MPI_ERR_INTERN; }
        close(fd);
        while (e.hdr->magic.load(std::memory_order_acquire) != kMagic) {
            if (now_s() > deadline) return MPI_ERR_INTERN;
            usleep(100);
        }
    } else {
        e.rank = atoi(trank);
        e.size = atoi(tsize);
        pid_t pp = getppid();
        uint64_t nonce = parent_start_time(pp) ^ ((uint64_t)pp << 32);
        const char *port = getenv("MASTER_PORT");
        const char *restart = getenv("TORCHELASTIC_RESTART_COUNT");
        e.shm_name = "/cmpi_t" + std::to_string((long)pp) + "_" + (port ? port : "0") + "_" +
                     (restart ? restart : "0");
        uint32_t ring = default_ring_bytes((uint32_t)e.size);
        size_t bytes = segment_bytes((uint32_t)e.size, ring);
        if (e.rank == 0) {
            shm_unlink(e.shm_name.c_str());
            fd = shm_open(e.shm_name.c_str(), O_CREAT | O_EXCL | O_RDWR, 0600);
            if (fd < 0 || ftruncate(fd, (off_t)bytes) != 0) {
                std::fprintf(stderr, "[minimpi] cannot create %s: %s\n", e.shm_name.c_str(),
                             strerror(errno));
                return MPI_ERR_INTERN;
            }
            if (map_segment(fd, bytes) != 0) { close(fd); return MPI_ERR_INTERN; }
            close(fd);
            e.hdr->nranks = (uint32_t)e.size;
            e.hdr->ring_bytes = ring;
            e.hdr->nonce = nonce;
            e.hdr->magic.store(kMagic, std::memory_order_release);
        } else {
            for (;;) {
                if (now_s() > deadline) {
                    std::fprintf(stderr, "[minimpi] rank %d: timed out joining %s\n", e.rank,
                                 e.shm_name.c_str());
                    return MPI_ERR_INTERN;
                }
                fd = shm_open(e.shm_name.c_str(), O_RDWR, 0600);
                if (fd < 0) { usleep(500); continue; }
                struct stat st;
                if (fstat(fd, &st) != 0 || (size_t)st.st_size < bytes) { close(fd); usleep(500); continue; }
                if (map_segment(fd, bytes) != 0) { close(fd); return MPI_ERR_INTERN; }
                close(fd);
                bool ok = false;
                for (int i = 0; i < 2000; ++i) {
                    if (e.hdr->magic.load(std::memory_order_acquire) == kMagic) {
                        ok = e.hdr->nonce == nonce;
                        break;
                    }
                    usleep(500);
                }
                if (ok) break;
                munmap(e.base, e.map_bytes);  // stale segment of an earlier job
                e.base = nullptr;
                usleep(1000);
            }
        }
    }
    e.ring = e.hdr->ring_bytes;
    if ((int)e.hdr->nranks != e.size) {
        std::fprintf(stderr, "[minimpi] segment is for %u ranks, job has %d\n", e.hdr->nranks, e.size);
        return MPI_ERR_INTERN;
    }
    g_world_rank = e.rank;
    e.slots[e.rank].node_id = node_id();
    e.slots[e.rank].pid.store((int32_t)getpid(), std::memory_order_relaxed);
    e.slots[e.rank].state.store(1, std::memory_order_release);
    e.hdr->joined.fetch_add(1, std::memory_order_acq_rel);
    while (e.hdr->joined.load(std::memory_order_acquire) < (uint32_t)e.size) {
        if (e.hdr->abort_flag.load()) _exit(e.hdr->abort_code.load());
        if (now_s() > deadline) {
            std::fprintf(stderr, "[minimpi] rank %d: timed out waiting for %d ranks to join\n",
                         e.rank, e.size);
            return MPI_ERR_INTERN;
        }
        usleep(50);
    }
    if (e.rank == 0) shm_unlink(e.shm_name.c_str());
    e.out.assign(e.size, PeerOut{});
    e.in.assign(e.size, PeerIn{});
    e.head_cache.assign(e.size, 0);
    e.tail_cache.assign(e.size, 0);
    e.up = true;
    e.last_health = now_s();
    *wr = e.rank;
    *ws = e.size;
    return MPI_SUCCESS;
}

void finalize_transport() {
    Engine &e = g_engine;
    if (!e.up) return;
    if (e.base) {
        e.slots[e.rank].state.store(2, std::memory_order_release);
        munmap(e.base, e.map_bytes);
        e.base = nullptr;
    }
    for (auto *u : e.unexpected) delete u;
    e.unexpected.clear();
    e.up = false;
}

void request_abort(int code) {
    Engine &e = g_engine;
    if (e.base) {
        e.hdr->abort_code.store(code);
        e.hdr->abort_rank.store(e.rank);
        e.hdr->abort_flag.store(1, std::memory_order_release);
    }
}

// ------------------------------------------------------------------ health
// Gone = no such process, or a zombie its parent has not reaped yet.
static bool process_gone(int pid) {
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

int check_health() {
    Engine &e = g_engine;
    if (!e.base) return MPI_SUCCESS;
    if (e.hdr->abort_flag.load(std::memory_order_acquire)) {
        int code = e.hdr->abort_code.load();
        std::fflush(stdout);
        _exit(code ? code : 1);
    }
    double t = now_s();
    if (t - e.last_health < 0.05) return MPI_SUCCESS;
    e.last_health = t;
    for (int r = 0; r < e.size; ++r) {
        if (r == e.rank) continue;
        int32_t pid = e.slots[r].pid.load(std::memory_order_relaxed);
        uint32_t st = e.slots[r].state.load(std::memory_order_acquire);
        if (pid > 0 && st == 1 && process_gone(pid)) {
            CMPI_ERR("peer rank %d (pid %d) exited without MPI_Finalize", r, pid);
            return MPI_ERR_PROC_FAILED;
        }
    }
    return MPI_SUCCESS;
}

void note_call() {
    Engine &e = g_engine;
    if (e.fi_rank != e.rank || e.fi_action.empty()) return;
    if (++e.calls != e.fi_at) return;
    if (e.fi_action == "exit") {
        std::fprintf(stderr, "[minimpi] rank %d: fault injection: exit(%d) at call %ld\n", e.rank,
                     e.fi_code, e.calls);
        std::fflush(stderr);
        _exit(e.fi_code);
    } else if (e.fi_action == "hang") {
        std::fprintf(stderr, "[minimpi] rank %d: fault injection: stalling at call %ld\n", e.rank,
                     e.calls);
        std::fflush(stderr);
        int secs = env_int("CMPI_FI_HANG_S", 30);
        for (int i = 0; i < secs * 10; ++i) usleep(100000);
        _exit(e.fi_code);
    } else if (e.fi_action == "drop") {
        std::fprintf(stderr, "[minimpi] rank %d: fault injection: dropping next send\n", e.rank);
        e.fi_drop_next = true;
    }
}

// ------------------------------------------------------------------ ring io
static inline uint64_t out_space(int d) {
    Engine &e = g_engine;
    uint64_t tail = chan(e.rank, d).tail.load(std::memory_order_acquire);
    return e.ring - (e.head_cache[d] - tail);
}

static void out_write(int d, const char *src, uint64_t n) {
    Engine &e = g_engine;
    char *rb = ring_of(e.rank, d);
    uint64_t pos = e.head_cache[d] % e.ring;
    uint64_t first = std::min<uint64_t>(n, e.ring - pos);
    memcpy(rb + pos, src, first);
    if (n > first) memcpy(rb, src + first, n - first);
    e.head_cache[d] += n;
    chan(e.rank, d).head.store(e.head_cache[d], std::memory_order_release);
}

static inline uint64_t in_avail(int s) {
    Engine &e = g_engine;
    uint64_t head = chan(s, e.rank).head.load(std::memory_order_acquire);
    return head - e.tail_cache[s];
}

// Copies n bytes out of the ring from source s into dst (host or device).
static void in_read(int s, char *dst, uint64_t n, bool dev, int ord) {
    Engine &e = g_engine;
    const char *rb = ring_of(s, e.rank);
    uint64_t pos = e.tail_cache[s] % e.ring;
    uint64_t first = std::min<uint64_t>(n, e.ring - pos);
    if (dev) {
        cuda_copy(dst, rb + pos, first, ord);
        if (n > first) cuda_copy(dst + first, rb, n - first, ord);
    } else {
        memcpy(dst, rb + pos, first);
        if (n > first) memcpy(dst + first, rb, n - first);
    }
}

static void in_consume(int s, uint64_t n) {
    Engine &e = g_engine;
    e.tail_cache[s] += n;
    chan(s, e.rank).tail.store(e.tail_cache[s], std::memory_order_release);
}

// ------------------------------------------------------------------ matching
static inline bool matches(const Request *r, int src, int ctx, int tag) {
    return r->ctx == ctx && (r->peer == MPI_ANY_SOURCE || r->peer == src) &&
           (r->tag == MPI_ANY_TAG || r->tag == tag);
}

static void set_status(Request *r, int src, int tag, uint64_t len) {
    r->status.MPI_SOURCE = src;
    r->status.MPI_TAG = tag;
    r->status.nbytes = (long long)std::min<uint64_t>(len, r->bytes);
    r->status.MPI_ERROR = len > r->bytes ? MPI_ERR_TRUNCATE : MPI_SUCCESS;
    if (len > r->bytes) r->err = MPI_ERR_TRUNCATE;
}

static void queue_ack(int to, uint64_t rid) {
    PktHdr a{};
    a.type = PKT_ACK;
    a.src = g_engine.rank;
    a.rid = rid;
    g_engine.out[to].ctrl.push_back(a);
}

// Completes receive r from a fully arrived unexpected message u.
static void deliver_unexpected(Request *r, Unexpected *u) {
    if (u->type == PKT_EAGER) {
        set_status(r, u->src, u->tag, u->len);
        uint64_t n = std::min<uint64_t>(u->len, r->bytes);
        if (n) {
            if (r->dev) cuda_copy(r->buf, u->data.data(), n, r->dev_ordinal);
            else memcpy(r->buf, u->data.data(), n);
        }
    } else {
        RndvDesc d;
        memcpy(&d, u->data.data(), sizeof(d));
        set_status(r, u->src, u->tag, d.bytes);  // the message size, not the descriptor's
        d.bytes = std::min<uint64_t>(d.bytes, r->bytes);
        int rc = d.bytes ? ipc_pull(u->src, d, r->buf, r->dev, r->dev_ordinal) : MPI_SUCCESS;
        if (rc != MPI_SUCCESS) r->err = rc;
        queue_ack(u->src, u->rid);
    }
    r->done = true;
}

// ------------------------------------------------------------------ progress
static void progress_out(int d) {
    Engine &e = g_engine;
    PeerOut &po = e.out[d];
    for (;;) {
        bool mid = !po.q.empty() && po.q.front()->hdr_sent;
        if (!mid && !po.ctrl.empty()) {
            if (out_space(d) < kPktHdr) return;
            out_write(d, (const char *)&po.ctrl.front(), kPktHdr);
            po.ctrl.pop_front();
            continue;
        }
        if (po.q.empty()) return;
        Request *r = po.q.front();
        if (!r->hdr_sent) {
            if (out_space(d) < kPktHdr) return;
            PktHdr h{};
            h.type = r->proto;
            h.ctx = r->ctx;
            h.tag = r->tag;
            h.src = e.rank;
            h.len = r->proto == PKT_EAGER ? r->bytes : sizeof(RndvDesc);
            h.rid = r->rid;
            out_write(d, (const char *)&h, kPktHdr);
            r->hdr_sent = true;
            r->sent = 0;
        }
        const char *payload = r->proto == PKT_EAGER ? r->src_ptr : (const char *)&r->desc;
        uint64_t plen = r->proto == PKT_EAGER ? r->bytes : sizeof(RndvDesc);
        while (r->sent < plen) {
            uint64_t n = std::min<uint64_t>(out_space(d), plen - r->sent);
            if (n == 0) return;
            out_write(d, payload + r->sent, n);
            r->sent += n;
        }
        po.q.pop_front();
        if (r->proto == PKT_EAGER) r->done = true;
        else e.rndv_pending[r->rid] = r;
    }
}

static void progress_in(int s) {
    Engine &e = g_engine;
    PeerIn &pi = e.in[s];
    for (;;) {
        uint64_t avail = in_avail(s);
        if (!pi.have_hdr) {
            if (avail < kPktHdr) return;
            in_read(s, (char *)&pi.h, kPktHdr, false, -1);
            in_consume(s, kPktHdr);
            avail -= kPktHdr;
            if (pi.h.type == PKT_ACK) {
                auto it = e.rndv_pending.find(pi.h.rid);
                if (it != e.rndv_pending.end()) {
                    it->second->done = true;
                    e.rndv_pending.erase(it);
                }
                continue;
            }
            pi.have_hdr = true;
            pi.got = 0;
            pi.tgt = nullptr;
            pi.ux = nullptr;
            for (auto it = e.posted.begin(); it != e.posted.end(); ++it) {
                if (matches(*it, pi.h.src, pi.h.ctx, pi.h.tag)) {
                    pi.tgt = *it;
                    e.posted.erase(it);
                    break;
                }
            }
            if (!pi.tgt) {
                auto *u = new Unexpected();
                u->src = pi.h.src;
                u->ctx = pi.h.ctx;
                u->tag = pi.h.tag;
                u->type = pi.h.type;
                u->len = pi.h.len;
                u->rid = pi.h.rid;
                u->data.resize(pi.h.len);
                e.unexpected.push_back(u);
                pi.ux = u;
            } else if (pi.h.type == PKT_EAGER) {
                set_status(pi.tgt, pi.h.src, pi.h.tag, pi.h.len);
            }
        }
        uint64_t remain = pi.h.len - pi.got;
        uint64_t n = std::min<uint64_t>(avail, remain);
        if (n) {
            if (pi.ux) {
                in_read(s, pi.ux->data.data() + pi.got, n, false, -1);
            } else if (pi.h.type == PKT_RNDV) {
                in_read(s, (char *)&pi.desc + pi.got, n, false, -1);
            } else {
                Request *r = pi.tgt;
                uint64_t lo = pi.got, hi = pi.got + n;
                uint64_t cap = r->bytes;
                if (lo < cap) {
                    uint64_t m = std::min<uint64_t>(hi, cap) - lo;
                    in_read(s, r->buf + lo, m, r->dev, r->dev_ordinal);
                }
            }
            in_consume(s, n);
            pi.got += n;
        }
        if (pi.got < pi.h.len) return;
        // message complete
        if (pi.ux) {
            Unexpected *u = pi.ux;
            u->got = u->len;
            u->complete = true;
            if (u->bound) {
                deliver_unexpected(u->bound, u);
                e.unexpected.remove(u);
                delete u;
            }
        } else if (pi.h.type == PKT_RNDV) {
            Request *r = pi.tgt;
            set_status(r, pi.h.src, pi.h.tag, pi.desc.bytes);
            RndvDesc d = pi.desc;
            d.bytes = std::min<uint64_t>(d.bytes, r->bytes);
            int rc = d.bytes ? ipc_pull(pi.h.src, d, r->buf, r->dev, r->dev_ordinal) : MPI_SUCCESS;
            if (rc != MPI_SUCCESS) r->err = rc;
            queue_ack(pi.h.src, pi.h.rid);
            r->done = true;
        } else {
            pi.tgt->done = true;
        }
        pi.have_hdr = false;
        pi.tgt = nullptr;
        pi.ux = nullptr;
    }
}

void progress() {
    Engine &e = g_engine;
    if (!e.base) return;
    for (int p = 0; p < e.size; ++p) {
        if (p == e.rank) continue;
        progress_in(p);
        progress_out(p);
    }
}

// ------------------------------------------------------------------ requests
static void self_send(Request *s) {
    Engine &e = g_engine;
    for (auto it = e.posted.begin(); it != e.posted.end(); ++it) {
        Request *r = *it;
        if (!matches(r, e.rank, s->ctx, s->tag)) continue;
        e.posted.erase(it);
        set_status(r, e.rank, s->tag, s->bytes);
        uint64_t n = std::min<uint64_t>(s->bytes, r->bytes);
        if (n) {
            if (r->dev || s->dev) cuda_copy(r->buf, s->src_ptr, n, r->dev ? r->dev_ordinal : s->dev_ordinal);
            else memcpy(r->buf, s->src_ptr, n);
        }
        r->done = true;
        s->done = true;
        return;
    }
    auto *u = new Unexpected();
    u->src = e.rank;
    u->ctx = s->ctx;
    u->tag = s->tag;
    u->type = PKT_EAGER;
    u->len = s->bytes;
    u->data.resize(s->bytes);
    if (s->bytes) {
        if (s->dev) cuda_copy(u->data.data(), s->src_ptr, s->bytes, s->dev_ordinal);
        else memcpy(u->data.data(), s->src_ptr, s->bytes);
    }
    u->got = u->len;
    u->complete = true;
    e.unexpected.push_back(u);
    s->done = true;
}

int isend(const void *buf, uint64_t bytes, int dest, int tag, int ctx, Request **out) {
    Engine &e = g_engine;
    auto *r = new Request();
    r->kind = REQ_SEND;
    r->ctx = ctx;
    r->tag = tag;
    r->peer = dest;
    r->bytes = bytes;
    r->src_ptr = (const char *)buf;
    *out = r;
    if (dest == MPI_PROC_NULL) { r->done = true; return MPI_SUCCESS; }
    if (e.fi_drop_next && dest != e.rank) {
        e.fi_drop_next = false;
        r->done = true;
        return MPI_SUCCESS;
    }
    int ord = -1;
    r->dev = bytes > 0 && is_device_ptr(buf, &ord);
    r->dev_ordinal = ord;
    if (dest == e.rank) { self_send(r); return MPI_SUCCESS; }
    if (r->dev) {
        if (ipc_describe(buf, bytes, ord, &r->desc)) {
            r->proto = PKT_RNDV;
            r->rid = e.next_rid++;
        } else {
            r->stage.resize(bytes);
            int rc = cuda_copy(r->stage.data(), buf, bytes, ord);
            if (rc != MPI_SUCCESS) { r->err = rc; r->done = true; return rc; }
            r->src_ptr = r->stage.data();
            r->proto = PKT_EAGER;
        }
    }
    e.out[dest].q.push_back(r);
    progress_out(dest);
    return MPI_SUCCESS;
}

int irecv(void *buf, uint64_t bytes, int src, int tag, int ctx, Request **out) {
    Engine &e = g_engine;
    auto *r = new Request();
    r->kind = REQ_RECV;
    r->ctx = ctx;
    r->tag = tag;
    r->peer = src;
    r->buf = (char *)buf;
    r->bytes = bytes;
    *out = r;
    if (src == MPI_PROC_NULL) {
        r->status.MPI_SOURCE = MPI_PROC_NULL;
        r->status.MPI_TAG = MPI_ANY_TAG;
        r->done = true;
        return MPI_SUCCESS;
    }
    int ord = -1;
    r->dev = bytes > 0 && is_device_ptr(buf, &ord);
    r->dev_ordinal = ord;
    for (auto it = e.unexpected.begin(); it != e.unexpected.end(); ++it) {
        Unexpected *u = *it;
        if (u->bound || !matches(r, u->src, u->ctx, u->tag)) continue;
        if (u->complete) {
            deliver_unexpected(r, u);
            e.unexpected.erase(it);
            delete u;
        } else {
            u->bound = r;
        }
        return MPI_SUCCESS;
    }
    e.posted.push_back(r);
    return MPI_SUCCESS;
}

bool test(Request *r) {
    if (!r->done) progress();
    return r->done;
}

static int wait_one(Request *r) {
    Engine &e = g_engine;
    unsigned spins = 0;
    double t0 = e.timeout_s > 0 ? now_s() : 0.0;
    while (!r->done) {
        progress();
        if (r->done) break;
        if (++spins % 256 == 0) {
            int rc = check_health();
            if (rc != MPI_SUCCESS) return rc;
            if (e.timeout_s > 0 && now_s() - t0 > e.timeout_s) {
                CMPI_ERR("wait timed out after %.1f s (peer %d, tag %d)", e.timeout_s, r->peer, r->tag);
                return MPI_ERR_PROC_FAILED;
            }
            if (spins > 1u << 14) sched_yield();
        }
    }
    return r->err;
}

int wait(Request *r, MPI_Status *st) {
    int rc = wait_one(r);
    if (rc == MPI_ERR_PROC_FAILED && !r->done) return rc;  // request stays owned by the engine
    if (st && r->kind == REQ_RECV) *st = r->status;
    delete r;
    return rc;
}

int waitall(int n, Request **rs, MPI_Status *st) {
    int first_err = MPI_SUCCESS;
    for (int i = 0; i < n; ++i) {
        if (!rs[i]) continue;
        int rc = wait_one(rs[i]);
        if (rc == MPI_ERR_PROC_FAILED && !rs[i]->done) return rc;
        if (rc != MPI_SUCCESS && first_err == MPI_SUCCESS) first_err = rc;
    }
    for (int i = 0; i < n; ++i) {
        if (!rs[i]) continue;
        if (st && rs[i]->kind == REQ_RECV) st[i] = rs[i]->status;
        delete rs[i];
        rs[i] = nullptr;
    }
    return first_err;
}

// ------------------------------------------------------------------ request handles
static std::vector<Request *> g_handles(1, nullptr);
static std::vector<int> g_free_handles;

MPI_Request req_to_handle(Request *r) {
    if (!g_free_handles.empty()) {
        int h = g_free_handles.back();
        g_free_handles.pop_back();
        g_handles[h] = r;
        return h;
    }
    g_handles.push_back(r);
    return (MPI_Request)(g_handles.size() - 1);
}

Request *handle_to_req(MPI_Request h) {
    if (h <= 0 || (size_t)h >= g_handles.size()) return nullptr;
    return g_handles[h];
}

void handle_release(MPI_Request h) {
    if (h <= 0 || (size_t)h >= g_handles.size()) return;
    g_handles[h] = nullptr;
    g_free_handles.push_back(h);
}

}  // namespace cmpi
