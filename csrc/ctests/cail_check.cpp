// cail_check — MPI test program for the cail interposer.
//
// Covers the reference's test programs (tests/test_allreduce_basic.c,
// test_allreduce_correctness.c, test_allreduce_edge.c and
// test_allreduce_correctness_gpu.cu there) with a stronger oracle: inputs
// are seeded and position-dependent, and every MPI_Allreduce result is
// compared with PMPI_Allreduce of the same inputs (integers bit-exact,
// floats bit-exact or within a reassociation tolerance, see --tol).
//
//   cail_check -m basic|matrix|edge|slots|config1|config3|stress|leave|canary_selftest|expect_error|stall|
//                 memkinds|nan
//              [-c count] [-d] [-a algo]
//              [-p] [-r reps] [--bits]
//     -d      device buffers (cudaMalloc) instead of malloc
//     -a      sets CAIL_ALGO before the first MPI_Allreduce
//     -p      also run MPI_PROD (the reference skips PROD for P > 4; here
//             PROD inputs are +-1 so it never overflows)
//     --bits  require floats to be bit-identical to PMPI_Allreduce
//
// Exit status 0 when every check passed.  Each failure prints one line.
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <math.h>
#include <mpi.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <unistd.h>

#include <cmath>
#include <limits>
#include <random>
#include <string>
#include <vector>

namespace {

int g_rank = 0, g_size = 1, g_fail = 0, g_pass = 0;
bool g_dev = false, g_prod = false, g_bits = false, g_verbose = false;

struct TypeCase {
    const char *name;
    MPI_Datatype dt;
    int size;
    int kind;  // 0 signed int, 1 unsigned int, 2 float, 3 double
};

const TypeCase kTypes[] = {
    {"MPI_CHAR", MPI_CHAR, 1, 0},
    {"MPI_SHORT", MPI_SHORT, 2, 0},
    {"MPI_INT", MPI_INT, 4, 0},
    {"MPI_LONG", MPI_LONG, (int)sizeof(long), 0},
    {"MPI_LONG_LONG", MPI_LONG_LONG, 8, 0},
    {"MPI_FLOAT", MPI_FLOAT, 4, 2},
    {"MPI_DOUBLE", MPI_DOUBLE, 8, 3},
    {"MPI_UNSIGNED_CHAR", MPI_UNSIGNED_CHAR, 1, 1},
    {"MPI_UNSIGNED_SHORT", MPI_UNSIGNED_SHORT, 2, 1},
    {"MPI_UNSIGNED", MPI_UNSIGNED, 4, 1},
    {"MPI_UNSIGNED_LONG", MPI_UNSIGNED_LONG, (int)sizeof(unsigned long), 1},
    {"MPI_UNSIGNED_LONG_LONG", MPI_UNSIGNED_LONG_LONG, 8, 1},
    {"MPI_INT8_T", MPI_INT8_T, 1, 0},
    {"MPI_UINT8_T", MPI_UINT8_T, 1, 1},
    {"MPI_INT16_T", MPI_INT16_T, 2, 0},
    {"MPI_UINT16_T", MPI_UINT16_T, 2, 1},
    {"MPI_INT32_T", MPI_INT32_T, 4, 0},
    {"MPI_UINT32_T", MPI_UINT32_T, 4, 1},
    {"MPI_INT64_T", MPI_INT64_T, 8, 0},
    {"MPI_UINT64_T", MPI_UINT64_T, 8, 1},
};

struct OpCase {
    const char *name;
    MPI_Op op;
};
const OpCase kOps[] = {{"MPI_SUM", MPI_SUM}, {"MPI_PROD", MPI_PROD}, {"MPI_MAX", MPI_MAX}, {"MPI_MIN", MPI_MIN}};

const char *last_algo() {
    typedef const char *(*fn_t)(void);
    static fn_t fn = (fn_t)dlsym(RTLD_DEFAULT, "cail_last_algorithm");
    return fn ? fn() : "n/a";
}

// ---- buffers that may live on the device
// Every buffer sits between two 256-byte canary zones (the user region stays
// 256-byte aligned, as cudaMalloc's would be).  Reading a result back and
// releasing a buffer check that no call wrote outside [p, p + bytes);
// a damaged zone counts as a failure in the next report and in the summary.
constexpr size_t kGuard = 256;
constexpr unsigned char kCanary = 0xA5;
int g_canary_bad = 0;

struct Buf {
    size_t bytes = 0;
    char *base = nullptr;
    void *p = nullptr;
    explicit Buf(size_t b) : bytes(b) {
        const size_t total = b + 2 * kGuard;
        std::vector<unsigned char> fillv(total, kCanary);
        if (g_dev) {
            if (cudaMalloc((void **)&base, total) != cudaSuccess) { fprintf(stderr, "cudaMalloc failed\n"); MPI_Abort(MPI_COMM_WORLD, 2); }
            cudaMemcpy(base, fillv.data(), total, cudaMemcpyHostToDevice);
        } else {
            base = (char *)malloc(total);
            memcpy(base, fillv.data(), total);
        }
        p = base + kGuard;
    }
    ~Buf() {
        check_guards();
        if (g_dev) cudaFree(base); else free(base);
    }
    void put(const void *h) { if (g_dev) cudaMemcpy(p, h, bytes, cudaMemcpyHostToDevice); else memcpy(p, h, bytes); }
    void get(void *h) const {
        if (g_dev) cudaMemcpy(h, p, bytes, cudaMemcpyDeviceToHost); else memcpy(h, p, bytes);
        check_guards();
    }
    void check_guards() const {
        unsigned char z[2 * kGuard];
        if (g_dev) {
            cudaMemcpy(z, base, kGuard, cudaMemcpyDeviceToHost);
            cudaMemcpy(z + kGuard, base + kGuard + bytes, kGuard, cudaMemcpyDeviceToHost);
        } else {
            memcpy(z, base, kGuard);
            memcpy(z + kGuard, base + kGuard + bytes, kGuard);
        }
        for (size_t i = 0; i < 2 * kGuard; ++i)
            if (z[i] != kCanary) {
                if (g_canary_bad++ == 0)
                    fprintf(stderr, "rank %d: canary byte %s the buffer overwritten (%zu bytes buffer)\n", g_rank,
                            i < kGuard ? "before" : "after", bytes);
                break;
            }
    }
};

// Seeded, position-dependent inputs.  Integers in [-8, 8] (SUM/MAX/MIN) or
// {1, -1} (PROD); floats normal(0,1) or uniform [0.999, 1.001] for PROD.
void fill(std::vector<char> &h, const TypeCase &t, MPI_Op op, size_t count, int rank, uint64_t seed) {
    std::mt19937_64 rng(seed * 1000003ull + (uint64_t)rank * 7919ull + 17);
    h.resize(count * t.size);
    for (size_t i = 0; i < count; ++i) {
        char *e = h.data() + i * t.size;
        if (t.kind == 2 || t.kind == 3) {
            double v = op == MPI_PROD ? 0.999 + 0.002 * std::uniform_real_distribution<double>(0, 1)(rng)
                                      : std::normal_distribution<double>(0, 1)(rng);
            if (t.kind == 2) { float f = (float)v; memcpy(e, &f, 4); } else memcpy(e, &v, 8);
        } else {
            long long v = op == MPI_PROD ? ((rng() & 1) ? 1 : -1)
                                         : (long long)(rng() % 17) - 8;
            if (t.kind == 1 && op != MPI_PROD && v < 0) v = -v;  // unsigned: [0, 8]
            memcpy(e, &v, t.size);  // little-endian truncation
        }
    }
}

bool compare(const std::vector<char> &got, const std::vector<char> &want, const TypeCase &t, size_t count,
             double tol, size_t *bad_index) {
    for (size_t i = 0; i < count; ++i) {
        const char *g = got.data() + i * t.size, *w = want.data() + i * t.size;
        if (memcmp(g, w, t.size) == 0) continue;
        if (!g_bits && (t.kind == 2 || t.kind == 3)) {
            double a, b;
            if (t.kind == 2) { float x, y; memcpy(&x, g, 4); memcpy(&y, w, 4); a = x; b = y; }
            else { memcpy(&a, g, 8); memcpy(&b, w, 8); }
            if (fabs(a - b) <= tol * (1.0 + fabs(b))) continue;
        }
        *bad_index = i;
        return false;
    }
    return true;
}

void report(bool ok, const std::string &what) {
    static int canary_seen = 0;
    if (g_canary_bad != canary_seen) {  // a zone was damaged since the last report
        canary_seen = g_canary_bad;
        ok = false;
    }
    int mine = ok ? 1 : 0, all = 0;
    PMPI_Allreduce(&mine, &all, 1, MPI_INT, MPI_MIN, MPI_COMM_WORLD);
    if (all) g_pass++; else g_fail++;
    if (g_rank == 0 && (!all || g_verbose))
        printf("%s: %s np=%d algo=%s\n", all ? "PASS" : "FAIL", what.c_str(), g_size, last_algo());
}

// One checked MPI_Allreduce: inputs by seed, oracle = PMPI_Allreduce.
bool check_one(const TypeCase &t, const OpCase &o, size_t count, bool inplace, uint64_t seed, double tol,
               size_t offset_elems = 0) {
    std::vector<char> in, want(count * t.size), got(count * t.size);
    fill(in, t, o.op, count, g_rank, seed);
    PMPI_Allreduce(in.data(), want.data(), (int)count, t.dt, o.op, MPI_COMM_WORLD);
    size_t off = offset_elems * t.size;
    Buf s(count * t.size + off), r(count * t.size + off);
    std::vector<char> tmp(count * t.size + off, 0);
    memcpy(tmp.data() + off, in.data(), in.size());
    int rc;
    if (inplace) {
        r.put(tmp.data());
        rc = MPI_Allreduce(MPI_IN_PLACE, (char *)r.p + off, (int)count, t.dt, o.op, MPI_COMM_WORLD);
    } else {
        s.put(tmp.data());
        std::fill(tmp.begin(), tmp.end(), (char)0x5a);
        r.put(tmp.data());
        rc = MPI_Allreduce((char *)s.p + off, (char *)r.p + off, (int)count, t.dt, o.op, MPI_COMM_WORLD);
    }
    std::vector<char> all(count * t.size + off);
    r.get(all.data());
    memcpy(got.data(), all.data() + off, count * t.size);
    size_t bad = 0;
    bool ok = rc == MPI_SUCCESS && compare(got, want, t, count, tol, &bad);
    if (!ok && g_verbose)
        fprintf(stderr, "rank %d: %s %s count=%zu mismatch at %zu (rc=%d)\n", g_rank, t.name, o.name, count, bad, rc);
    return ok;
}

// ---------------------------------------------------------------- modes
void mode_basic(int opt_count) {
    std::vector<int> counts = {1, 10, 100, 1000, 4096, 100000, 200000};
    if (opt_count > 0) counts = {opt_count};
    for (int c : counts) {
        std::vector<float> h(c, (float)(g_rank + 1)), o(c, 0.f);
        Buf s(c * 4), r(c * 4);
        s.put(h.data());
        r.put(o.data());
        MPI_Allreduce(s.p, r.p, c, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
        r.get(o.data());
        float expect = 0;
        for (int q = 0; q < g_size; ++q) expect += (float)(q + 1);
        bool ok = true;
        for (int i = 0; i < c; ++i) ok = ok && fabsf(o[i] - expect) <= 1e-3f;
        report(ok, "basic float SUM count=" + std::to_string(c));
    }
}

void mode_matrix(int base, double tol) {
    std::vector<size_t> counts = {1, 2, 3};
    if (base > 3) { counts.push_back(base); counts.push_back(base + 1); counts.push_back(base + 3); }
    uint64_t seed = 1;
    for (size_t c : counts)
        for (const TypeCase &t : kTypes)
            for (const OpCase &o : kOps) {
                if (o.op == MPI_PROD && !g_prod && g_size > 4) continue;
                for (int ip = 0; ip < 2; ++ip) {
                    bool ok = check_one(t, o, c, ip == 1, seed++, tol);
                    report(ok, std::string(ip ? "MPI_IN_PLACE " : "") + t.name + " x " + o.name +
                                   " count=" + std::to_string(c));
                }
            }
}

// Dtype/op coverage at the two acceptance counts: 1,000,003 (not divisible
// by the world size) and 4,194,304; all 20 datatypes x SUM/PROD/MAX/MIN.
void mode_config3(double tol) {
    uint64_t seed = 77;
    for (size_t c : {(size_t)1000003, (size_t)4194304})
        for (const TypeCase &t : kTypes)
            for (const OpCase &o : kOps) {
                bool ok = check_one(t, o, c, false, seed++, tol);
                report(ok, std::string(t.name) + " x " + o.name + " count=" + std::to_string(c));
            }
}

// MAX / MIN on floats holding NaN and infinities.  The NVLink kernels fold in
// rank order with acc = (acc > x) ? acc : x (MIN with <), like the PMPI
// oracle, so the results must be bit-identical to PMPI's (NaN payloads
// included).  Device buffers only: the host algorithms (recursive doubling,
// ring, Rabenseifner) combine pairs in orders that differ between ranks, and
// with a NaN, max(NaN, 1) != max(1, NaN), so there the ranks may disagree
// (as with the reference's host algorithms).
void mode_nan() {
    if (!g_dev) {
        report(true, "NaN/Inf MAX/MIN (device buffers only; nothing to check)");
        return;
    }
    const float qnan = std::numeric_limits<float>::quiet_NaN(), inf = std::numeric_limits<float>::infinity();
    const double dnan = std::numeric_limits<double>::quiet_NaN(), dinf = std::numeric_limits<double>::infinity();
    for (size_t count : {(size_t)100003, (size_t)1000003}) {  // one-shot and two-shot sizes
        for (int dbl = 0; dbl < 2; ++dbl) {
            for (MPI_Op op : {MPI_MAX, MPI_MIN}) {
                const size_t esz = dbl ? 8 : 4;
                std::vector<char> h(count * esz), want(count * esz), got(count * esz);
                std::mt19937_64 rng(77 + (uint64_t)g_rank);
                for (size_t i = 0; i < count; ++i) {
                    double v = std::normal_distribution<double>(0, 1)(rng);
                    if (i % 7 == (size_t)(g_rank % 7)) v = dbl ? dnan : (double)qnan;
                    if (g_rank == 0 && i % 11 == 0) v = dinf;
                    if (g_rank == g_size - 1 && i % 13 == 0) v = -dinf;
                    if (dbl) memcpy(h.data() + i * 8, &v, 8);
                    else { float f = std::isnan(v) ? qnan : (std::isinf(v) ? (v > 0 ? inf : -inf) : (float)v); memcpy(h.data() + i * 4, &f, 4); }
                }
                MPI_Datatype dt = dbl ? MPI_DOUBLE : MPI_FLOAT;
                PMPI_Allreduce(h.data(), want.data(), (int)count, dt, op, MPI_COMM_WORLD);
                for (int ip = 0; ip < 2; ++ip) {
                    Buf s(count * esz), r(count * esz);
                    s.put(h.data());
                    r.put(h.data());
                    int rc = MPI_Allreduce(ip ? MPI_IN_PLACE : s.p, r.p, (int)count, dt, op, MPI_COMM_WORLD);
                    r.get(got.data());
                    report(rc == MPI_SUCCESS && memcmp(got.data(), want.data(), count * esz) == 0,
                           std::string(ip ? "MPI_IN_PLACE " : "") + (dbl ? "DOUBLE " : "FLOAT ") +
                               (op == MPI_MAX ? "MAX" : "MIN") + " with NaN/Inf count=" + std::to_string(count) +
                               " bit-identical to PMPI");
                }
            }
        }
    }
}

// Device-pointer detection over the four kinds of memory an application may
// hand in: cudaMalloc and managed memory run on cail's device path, pinned
// (cudaMallocHost) and malloc'd memory pass through to PMPI_Allreduce.
// Every call must produce the PMPI result.
void mode_memkinds() {
    const char *names[4] = {"cudaMalloc", "cudaMallocManaged", "cudaMallocHost", "malloc"};
    for (int kind = 0; kind < 4; ++kind) {
        for (size_t count : {(size_t)16384, (size_t)262144}) {  // 64 KiB and 1 MiB of floats
            const size_t bytes = count * sizeof(float);
            float *s = nullptr, *r = nullptr;
            bool alloc_ok = true;
            if (kind == 0) alloc_ok = cudaMalloc(&s, bytes) == cudaSuccess && cudaMalloc(&r, bytes) == cudaSuccess;
            if (kind == 1) alloc_ok = cudaMallocManaged(&s, bytes) == cudaSuccess && cudaMallocManaged(&r, bytes) == cudaSuccess;
            if (kind == 2) alloc_ok = cudaMallocHost(&s, bytes) == cudaSuccess && cudaMallocHost(&r, bytes) == cudaSuccess;
            if (kind == 3) { s = (float *)malloc(bytes); r = (float *)malloc(bytes); alloc_ok = s && r; }
            std::vector<float> h(count), want(count), got(count);
            for (size_t i = 0; i < count; ++i) h[i] = (float)((i * 7 + (size_t)g_rank * 13) % 101) - 50.0f;
            bool ok = alloc_ok;
            if (ok) {
                if (kind < 2) cudaMemcpy(s, h.data(), bytes, cudaMemcpyDefault);
                else memcpy(s, h.data(), bytes);
                PMPI_Allreduce(h.data(), want.data(), (int)count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
                ok = MPI_Allreduce(s, r, (int)count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD) == MPI_SUCCESS;
                if (kind < 2) cudaMemcpy(got.data(), r, bytes, cudaMemcpyDefault);
                else memcpy(got.data(), r, bytes);
                ok = ok && memcmp(got.data(), want.data(), bytes) == 0;
                const std::string algo = last_algo();
                const bool device_kind = kind < 2;
                // an interposer without cail_last_algorithm reports "n/a"
                if (algo != "n/a") ok = ok && ((algo == "pmpi") != device_kind);
            }
            report(ok, std::string(names[kind]) + " buffers, " + std::to_string(bytes) + " bytes, " +
                           (kind < 2 ? "device path" : "PMPI passthrough"));
            if (kind == 0 || kind == 1) { cudaFree(s); cudaFree(r); }
            if (kind == 2) { cudaFreeHost(s); cudaFreeHost(r); }
            if (kind == 3) { free(s); free(r); }
        }
    }
}

// With a failure injected on one rank (CAIL_FI_TWOSHOT_FAIL), a large call
// must return an error on every rank (none may hang or report success), and
// so must the next call on the same communicator.
// Rank 1 stalls on the host (3 s) before its call; the zero-copy two-shot
// path must not wait for it forever: with CAIL_HOST_TIMEOUT_MS=1000 rank 0
// gives up at its arrive barrier and returns an error, and rank 1, arriving
// late, sees rank 0's error bit and returns an error without launching.
void mode_stall(int count) {
    Buf s(count * sizeof(float)), r(count * sizeof(float));
    std::vector<float> h(count, 1.0f);
    s.put(h.data());
    // one call first: the communicator's device setup is collective and would
    // absorb the stall
    report(MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD) == MPI_SUCCESS, "warm-up call");
    if (g_rank == 1) sleep(3);
    const double t0 = MPI_Wtime();
    const int rc = MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
    const double dt = MPI_Wtime() - t0;
    report(rc != MPI_SUCCESS, "a call whose peer stalls on the host returns an error");
    if (g_rank == 0) {
        report(dt > 0.5 && dt < 2.5, "the waiting rank gives up at the host timeout");
        printf("STALL DETECTED after %.2f s\n", dt);
    } else {
        report(dt < 2.0, "the late rank returns at once");
    }
    const int rc2 = MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
    report(rc2 != MPI_SUCCESS, "the broken communicator refuses the next call");
}

void mode_expect_error(int count) {
    Buf s(count * sizeof(float)), r(count * sizeof(float));
    std::vector<float> h(count, 1.0f);
    s.put(h.data());
    double t0 = MPI_Wtime();
    int rc1 = MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
    int rc2 = MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
    double dt = MPI_Wtime() - t0;
    report(rc1 != MPI_SUCCESS, "failed call returns an error on every rank");
    report(rc2 != MPI_SUCCESS, "the next call on the broken communicator returns an error too");
    report(dt < 30.0, "both calls return within 30 s");
}

// Positive control of the canary zones: writes one byte just past a buffer
// (inside its own guard zone, so nothing outside the allocation is touched)
// and expects the check to notice.
void mode_canary_selftest() {
    Buf b(1024);
    const unsigned char x = 0;
    if (g_dev) cudaMemcpy((char *)b.p + 1024, &x, 1, cudaMemcpyHostToDevice);
    else memcpy((char *)b.p + 1024, &x, 1);
    std::vector<char> h(1024);
    b.get(h.data());
    report(g_canary_bad == 0, "canary zones intact after a deliberate one-byte overrun");
}

void mode_edge() {
    // count = 0
    {
        Buf a(16), b(16);
        int rc = MPI_Allreduce(a.p, b.p, 0, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
        report(rc == MPI_SUCCESS, "count=0");
        rc = MPI_Allreduce(MPI_IN_PLACE, b.p, 0, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
        report(rc == MPI_SUCCESS, "MPI_IN_PLACE count=0");
    }
    const TypeCase tf = kTypes[5], ti = kTypes[2], td = kTypes[6];
    report(check_one(tf, kOps[0], 1, false, 11, 1e-5), "count=1");
    report(check_one(tf, kOps[0], 1, true, 12, 1e-5), "MPI_IN_PLACE count=1");
    report(check_one(tf, kOps[0], 200000, false, 13, 1e-5), "count=200000 (large)");
    report(check_one(tf, kOps[0], 200000, true, 14, 1e-5), "MPI_IN_PLACE count=200000 (large)");
    report(check_one(ti, kOps[2], 4096, true, 15, 0), "MPI_IN_PLACE int MAX count=4096");
    report(check_one(td, kOps[3], 4096, true, 16, 0), "MPI_IN_PLACE double MIN count=4096");
    // unaligned buffers (odd element offsets) on every path
    report(check_one(tf, kOps[0], 100003, false, 17, 1e-5, 1), "unaligned float SUM count=100003");
    report(check_one(kTypes[0], kOps[0], 70001, true, 18, 0, 3), "unaligned char SUM in place");
    // host-side fallbacks: long double SUM, unsigned BAND, contiguous derived type
    {
        std::vector<long double> s(10, (long double)(g_rank + 1)), r(10, 0);
        MPI_Allreduce(s.data(), r.data(), 10, MPI_LONG_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        long double e = 0;
        for (int q = 0; q < g_size; ++q) e += q + 1;
        bool ok = true;
        for (auto v : r) ok = ok && fabsl(v - e) < 1e-6L;
        report(ok && std::string(last_algo()) != "one_shot", "MPI_LONG_DOUBLE fallback");
        std::vector<long double> ip(10, (long double)(g_rank + 1));
        MPI_Allreduce(MPI_IN_PLACE, ip.data(), 10, MPI_LONG_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        ok = true;
        for (auto v : ip) ok = ok && fabsl(v - e) < 1e-6L;
        report(ok, "MPI_IN_PLACE MPI_LONG_DOUBLE fallback");
    }
    {
        std::vector<unsigned> s(10, 0xFFFFFFFFu), r(10, 0);
        MPI_Allreduce(s.data(), r.data(), 10, MPI_UNSIGNED, MPI_BAND, MPI_COMM_WORLD);
        bool ok = true;
        for (auto v : r) ok = ok && v == 0xFFFFFFFFu;
        report(ok, "MPI_BAND fallback");
        MPI_Allreduce(MPI_IN_PLACE, s.data(), 10, MPI_UNSIGNED, MPI_BAND, MPI_COMM_WORLD);
        ok = true;
        for (auto v : s) ok = ok && v == 0xFFFFFFFFu;
        report(ok, "MPI_IN_PLACE MPI_BAND fallback");
    }
    {
        MPI_Datatype pair;
        MPI_Type_contiguous(2, MPI_INT, &pair);
        MPI_Type_commit(&pair);
        std::vector<int> s(2 * 20000), r(2 * 20000, 0);
        for (size_t i = 0; i < s.size(); ++i) s[i] = (int)(i % 7) + g_rank;
        MPI_Allreduce(s.data(), r.data(), 20000, pair, MPI_SUM, MPI_COMM_WORLD);
        bool ok = std::string(last_algo()) == "pmpi";
        for (size_t i = 0; i < s.size(); ++i) {
            long long e = 0;
            for (int q = 0; q < g_size; ++q) e += (long long)(i % 7) + q;
            ok = ok && r[i] == e;
        }
        report(ok, "derived datatype fallback");
        MPI_Type_free(&pair);
    }
    // intercommunicator branch (minimpi marks the communicator for the test)
    {
        MPI_Comm dup;
        MPI_Comm_dup(MPI_COMM_WORLD, &dup);
#ifdef MINIMPI
        MPIX_Comm_set_test_inter(dup, 1);
#endif
        std::vector<int> s(20000, 1), r(20000, 0);
        Buf sb(s.size() * 4), rb(r.size() * 4);
        sb.put(s.data());
        MPI_Allreduce(sb.p, rb.p, (int)s.size(), MPI_INT, MPI_SUM, dup);
        rb.get(r.data());
        bool ok = r[0] == g_size && r.back() == g_size;
#ifdef MINIMPI
        ok = ok && std::string(last_algo()) == "pmpi";
#endif
        report(ok, "intercommunicator fallback");
        MPI_Comm_free(&dup);
    }
}

// The host-only acceptance configuration: FLOAT SUM 262144 uniform[-1,1)
// seeded seed+rank and INT MAX 65536 uniform [-1000,1000], each algorithm x
// {separate, in place}, compared with PMPI_Allreduce; min-msg-size fallback
// at count 1024.
// Large messages with a ragged end (a length that is not a multiple of 16
// bytes) and with buffers one or three elements off a 16-byte boundary,
// separate and in place.  Run with CAIL_ALGO=nvls and a small CAIL_NVLS_UNIT
// they give each CTA several units, so its two staging slots are refilled
// while earlier units are copied out.  count (default 10,485,763 floats,
// 40 MiB + 12 bytes) sets the float and int cases; the 8-byte cases take
// half of it, rounded to an odd count.
void mode_slots(int count, double tol) {
    const TypeCase &tf = kTypes[5], &td = kTypes[6], &ti = kTypes[2], &tu = kTypes[11];
    const size_t n = count > 0 ? (size_t)count : 10485763;
    const size_t h = (n / 2) | 1;
    report(check_one(tf, kOps[0], n, false, 31, tol), "ragged float SUM count=" + std::to_string(n));
    report(check_one(tf, kOps[0], n, false, 32, tol, 1), "unaligned float SUM count=" + std::to_string(n));
    report(check_one(tf, kOps[0], n, true, 33, tol, 3), "unaligned float SUM in place count=" + std::to_string(n));
    report(check_one(td, kOps[0], h, true, 34, tol, 1), "unaligned double SUM in place count=" + std::to_string(h));
    report(check_one(ti, kOps[2], n, false, 35, 0, 1), "unaligned int MAX count=" + std::to_string(n));
    report(check_one(tu, kOps[0], h, false, 36, 0), "ragged unsigned long long SUM count=" + std::to_string(h));
}

void mode_config1(double tol) {
    const char *algo = getenv("CAIL_ALGO");
    std::string a = algo ? algo : "auto";
    for (int ip = 0; ip < 2; ++ip) {
        {
            const int n = 262144;
            std::mt19937 rng(1234 + g_rank);
            std::uniform_real_distribution<float> u(-1.f, 1.f);
            std::vector<float> in(n), want(n), got(n);
            for (auto &v : in) v = u(rng);
            PMPI_Allreduce(in.data(), want.data(), n, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
            Buf s(n * 4), r(n * 4);
            if (ip) { r.put(in.data()); MPI_Allreduce(MPI_IN_PLACE, r.p, n, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD); }
            else { s.put(in.data()); MPI_Allreduce(s.p, r.p, n, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD); }
            r.get(got.data());
            bool ok = true;
            for (int i = 0; i < n; ++i) ok = ok && fabs((double)got[i] - want[i]) <= tol * (1 + fabs(want[i]));
            std::string used = last_algo();
            // (an interposer without cail_last_algorithm reports "n/a")
            if (a != "auto" && used != "n/a") ok = ok && (used == a || g_size == 1);
            report(ok, std::string(ip ? "MPI_IN_PLACE " : "") + "config1 FLOAT SUM 262144 algo=" + a);
        }
        {
            const int n = 65536;
            std::mt19937 rng(4321 + g_rank);
            std::uniform_int_distribution<int> u(-1000, 1000);
            std::vector<int> in(n), want(n), got(n);
            for (auto &v : in) v = u(rng);
            PMPI_Allreduce(in.data(), want.data(), n, MPI_INT, MPI_MAX, MPI_COMM_WORLD);
            Buf s(n * 4), r(n * 4);
            if (ip) { r.put(in.data()); MPI_Allreduce(MPI_IN_PLACE, r.p, n, MPI_INT, MPI_MAX, MPI_COMM_WORLD); }
            else { s.put(in.data()); MPI_Allreduce(s.p, r.p, n, MPI_INT, MPI_MAX, MPI_COMM_WORLD); }
            r.get(got.data());
            report(got == want, std::string(ip ? "MPI_IN_PLACE " : "") + "config1 INT MAX 65536 algo=" + a);
        }
    }
    // below CAIL_MIN_MSG_SIZE (default 32 KiB): 1024 floats pass through
    {
        std::vector<float> in(1024, (float)g_rank), got(1024);
        Buf s(4096), r(4096);
        s.put(in.data());
        MPI_Allreduce(s.p, r.p, 1024, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
        r.get(got.data());
        float e = (float)(g_size * (g_size - 1) / 2);
        bool ok = got[0] == e && got[1023] == e;
        const char *mm = getenv("CAIL_MIN_MSG_SIZE");
        bool expect_pmpi = !mm || atol(mm) > 4096;
        if (std::string(last_algo()) != "n/a") ok = ok && ((std::string(last_algo()) == "pmpi") == expect_pmpi);
        report(ok, "config1 min_msg_size fallback at count 1024");
    }
}

// Alternates buffers among `nbuf` allocations and interleaves MPI_IN_PLACE
// (registration cache exercise).
void mode_stress(int count, int reps, int nbuf, double tol) {
    const TypeCase &t = kTypes[6];  // double
    std::vector<Buf *> bufs;
    for (int i = 0; i < nbuf; ++i) bufs.push_back(new Buf((size_t)count * 8));
    std::vector<char> in, want(count * 8), got(count * 8);
    bool ok = true;
    for (int it = 0; it < reps; ++it) {
        fill(in, t, MPI_SUM, count, g_rank, 1000 + it % 7);
        if (it < 7) {}
        PMPI_Allreduce(in.data(), want.data(), count, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        Buf *a = bufs[it % nbuf], *b = bufs[(it * 7 + 3) % nbuf];
        a->put(in.data());
        if (it % 2 || a == b) MPI_Allreduce(MPI_IN_PLACE, a->p, count, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        else MPI_Allreduce(a->p, b->p, count, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        ((it % 2 || a == b) ? a : b)->get(got.data());
        size_t bad;
        if (!compare(got, want, t, count, tol, &bad)) ok = false;
    }
    report(ok, "stress " + std::to_string(reps) + " calls over " + std::to_string(nbuf) + " buffers count=" +
                   std::to_string(count));
    for (auto *b : bufs) delete b;
}

// Rank 1 leaves the job between two allreduce steps (no collective in
// flight); rank 0 must get an error from its next MPI_Allreduce instead of
// waiting for it.  Exit 0 on rank 0 means the departure was detected.
void mode_leave(int count) {
    MPI_Comm_set_errhandler(MPI_COMM_WORLD, MPI_ERRORS_RETURN);
    Buf s((size_t)count * 4), r((size_t)count * 4);
    std::vector<float> h(count, 1.f);
    s.put(h.data());
    for (int it = 0; it < 6; ++it) {
        if (g_rank == 1 && it == 2) {
            fflush(stdout);
            _exit(0);
        }
        if (g_rank == 0) usleep(100000);
        int rc = MPI_Allreduce(s.p, r.p, count, MPI_FLOAT, MPI_SUM, MPI_COMM_WORLD);
        if (rc != MPI_SUCCESS) {
            if (g_rank == 0) printf("LEAVE DETECTED at step %d (rc=%d)\n", it, rc);
            fflush(stdout);
            _exit(it == 2 ? 0 : 4);
        }
    }
    if (g_rank == 0) printf("LEAVE NOT DETECTED\n");
    fflush(stdout);
    _exit(5);
}

}  // namespace

int main(int argc, char **argv) {
    std::string mode = "matrix";
    int count = 0, reps = 200, nbuf = 8;
    double tol = 1e-5;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "-m" && i + 1 < argc) mode = argv[++i];
        else if (a == "-c" && i + 1 < argc) count = atoi(argv[++i]);
        else if (a == "-r" && i + 1 < argc) reps = atoi(argv[++i]);
        else if (a == "-b" && i + 1 < argc) nbuf = atoi(argv[++i]);
        else if (a == "-a" && i + 1 < argc) setenv("CAIL_ALGO", argv[++i], 1);
        else if (a == "-d") g_dev = true;
        else if (a == "-p") g_prod = true;
        else if (a == "-v") g_verbose = true;
        else if (a == "--bits") g_bits = true;
        else if (a == "--tol" && i + 1 < argc) tol = atof(argv[++i]);
        else { fprintf(stderr, "unknown argument %s\n", argv[i]); return 2; }
    }
    MPI_Init(&argc, &argv);
    MPI_Comm_rank(MPI_COMM_WORLD, &g_rank);
    MPI_Comm_size(MPI_COMM_WORLD, &g_size);
    if (g_dev) {
        int n = 0;
        if (cudaGetDeviceCount(&n) != cudaSuccess || n == 0) {
            if (g_rank == 0) fprintf(stderr, "no CUDA device\n");
            MPI_Finalize();
            return 3;
        }
        const char *lr = getenv("CMPI_LOCAL_RANK");
        if (!lr) lr = getenv("LOCAL_RANK");
        cudaSetDevice((lr ? atoi(lr) : g_rank) % n);
    }
    if (mode == "basic") mode_basic(count);
    else if (mode == "matrix") mode_matrix(count ? count : 1000, tol);
    else if (mode == "edge") mode_edge();
    else if (mode == "slots") mode_slots(count, tol);
    else if (mode == "config3") mode_config3(tol);
    else if (mode == "config1") mode_config1(tol);
    else if (mode == "stress") mode_stress(count ? count : 4096, reps, nbuf, tol);
    else if (mode == "leave") mode_leave(count ? count : 65536);
    else if (mode == "canary_selftest") mode_canary_selftest();
    else if (mode == "expect_error") mode_expect_error(count ? count : (1 << 20));
    else if (mode == "stall") mode_stall(count ? count : (1 << 20));
    else if (mode == "memkinds") mode_memkinds();
    else if (mode == "nan") mode_nan();
    else { fprintf(stderr, "unknown mode %s\n", mode.c_str()); MPI_Abort(MPI_COMM_WORLD, 2); }
    if (mode != "leave") report(g_canary_bad == 0, "canary zones around every buffer intact");
    if (g_rank == 0) printf("=== Results: %d passed, %d failed ===\n", g_pass, g_fail);
    MPI_Finalize();
    return g_fail ? 1 : 0;
}
