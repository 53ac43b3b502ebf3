// cail_init.cpp — configuration from the environment, init and teardown.
//
// The six variables of the reference contract are read once, at the first
// MPI_Allreduce, with the reference's rules and messages
// (src/core/cail_init.c:20-126 there):
//   CAIL_DEBUG                any non-empty value not starting with '0'
//   CAIL_WARN                 off only when the value starts with '0'
//   CAIL_MSG_SMALL_THRESHOLD  integer > 0
//   CAIL_NPROCS_THRESHOLD     integer in (0, INT_MAX]  (parsed, unused)
//   CAIL_MIN_MSG_SIZE         integer >= 0
//   CAIL_ALGO                 auto | recursive_doubling | ring | rabenseifner
//                             | one_shot | two_shot | nvls
// An invalid value prints "[cail ERROR] invalid X='v', using default".
#include <ctype.h>
#include <limits.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include "../gpu/cail_gpu.h"
#include "cail_internal.h"

extern "C" {

cail_state_t cail_global_state = {
    /*initialized*/ 0, /*debug*/ 0, /*warn*/ 1,
    /*msg_small_threshold*/ CAIL_DEFAULT_MSG_SMALL_THRESHOLD, /*set*/ 0,
    /*nprocs_threshold*/ CAIL_DEFAULT_NPROCS_THRESHOLD,
    /*min_msg_size*/ CAIL_DEFAULT_MIN_MSG_SIZE,
    /*force_algo*/ CAIL_ALGO_AUTO,
    /*device_timeout_ms*/ CAIL_DEFAULT_DEVICE_TIMEOUT_MS,
    /*nvls*/ 1, /*oneshot_max*/ 0, /*flush_recv*/ 1, /*stats*/ 0, /*trace*/ nullptr,
    /*stream_sync*/ 1, /*profile*/ 0, /*stream_ordered*/ 0, /*nvtx*/ 0, /*device_checks*/ 0};

cail_stats_t cail_counters;
int cail_last_algo = -2;  // -2: none yet, -3: passthrough
double cail_prof_us[CAIL_PH_N];
unsigned long long cail_prof_calls = 0;

}  // extern "C"

namespace {

// Strict decimal parse: the whole string must be a number within [lo, hi].
bool parse_long(const char *name, const char *val, long lo, long hi, long *out) {
    char *end = nullptr;
    long v = strtol(val, &end, 10);
    if (*end != '\0' || v < lo || v > hi) {
        CAIL_ERR("invalid %s='%s', using default", name, val);
        return false;
    }
    *out = v;
    return true;
}

const char *env_nonempty(const char *name) {
    const char *v = getenv(name);
    return (v && v[0] != '\0') ? v : nullptr;
}

// CAIL_TUNE_FILE: one line per rank count, "nranks=8 oneshot_max=262144
// nvls_min=64M ce_min=512M" (any subset of the size keys; integers with an
// optional K, M or G suffix; '#' starts a comment).  A bad line is reported
// and ignored; a later line for the same nranks replaces an earlier one.
constexpr int kMaxTune = 64;
cail_tune_t g_tune[kMaxTune];
int g_ntune = 0;

bool parse_size(const char *v, long long *out) {
    char *end = nullptr;
    if (!isdigit((unsigned char)v[0])) return false;
    long long x = strtoll(v, &end, 10);
    long long mul = 1;
    if (*end == 'K' || *end == 'k') mul = 1LL << 10, ++end;
    else if (*end == 'M' || *end == 'm') mul = 1LL << 20, ++end;
    else if (*end == 'G' || *end == 'g') mul = 1LL << 30, ++end;
    if (*end != '\0' || x < 0 || x > (LLONG_MAX >> 30)) return false;
    *out = x * mul;
    return true;
}

void load_tune(const char *path) {
    FILE *f = fopen(path, "r");
    if (!f) {
        CAIL_ERR("cannot open CAIL_TUNE_FILE '%s'", path);
        return;
    }
    char line[512];
    int lineno = 0;
    while (fgets(line, sizeof line, f)) {
        ++lineno;
        if (char *h = strchr(line, '#')) *h = '\0';
        cail_tune_t t = {0, -1, -1, -1};
        bool bad = false, any = false;
        char *save = nullptr;
        for (char *tok = strtok_r(line, " \t\r\n", &save); tok && !bad; tok = strtok_r(nullptr, " \t\r\n", &save)) {
            any = true;
            char *eq = strchr(tok, '=');
            if (!eq) { bad = true; break; }
            *eq = '\0';
            const char *key = tok, *val = eq + 1;
            long long x = 0;
            if (!parse_size(val, &x)) bad = true;
            else if (!strcmp(key, "nranks")) {
                if (x >= 1 && x <= INT_MAX) t.nranks = (int)x;
                else bad = true;
            }
            else if (!strcmp(key, "oneshot_max")) t.oneshot_max = x;
            else if (!strcmp(key, "nvls_min")) t.nvls_min = x;
            else if (!strcmp(key, "ce_min")) t.ce_min = x;
            else bad = true;
        }
        if (!any) continue;
        if (bad || t.nranks < 1) {
            CAIL_ERR("CAIL_TUNE_FILE '%s' line %d: expected nranks=<n> and oneshot_max=, nvls_min=, ce_min= "
                     "sizes; line ignored", path, lineno);
            continue;
        }
        int i = 0;
        while (i < g_ntune && g_tune[i].nranks != t.nranks) ++i;
        if (i == kMaxTune) {
            CAIL_ERR("CAIL_TUNE_FILE '%s' line %d: more than %d rank counts; line ignored", path, lineno, kMaxTune);
            continue;
        }
        g_tune[i] = t;
        if (i == g_ntune) ++g_ntune;
    }
    fclose(f);
    CAIL_DBG("CAIL_TUNE_FILE '%s': %d rank count(s)", path, g_ntune);
}

bool g_stream_sync_set = false;  // cail_set_stream_sync() overrides the environment
bool g_stream_ordered_set = false;  // likewise cail_set_stream_ordered()

}  // namespace

extern "C" {

double cail_now_us(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e6 + ts.tv_nsec * 1e-3;
}

// Phase times of the call in progress; folded into cail_prof_us by
// cail_prof_end_call() unless the call took longer than CAIL_PROFILE_MAX_US
// (default 500), which keeps one-time costs such as lazy kernel loading out
// of the small-message averages.
static double g_call_us[CAIL_PH_N];

double cail_prof_mark(int ph, double t0) {
    if (!cail_global_state.profile) return t0;
    double t = cail_now_us();
    g_call_us[ph] += t - t0;
    return t;
}

void cail_prof_end_call(double total_us) {
    static const double cutoff = [] {
        const char *e = getenv("CAIL_PROFILE_MAX_US");
        return e ? atof(e) : 500.0;
    }();
    if (total_us <= cutoff) {
        for (int i = 0; i < CAIL_PH_N; ++i) cail_prof_us[i] += g_call_us[i];
        cail_prof_us[CAIL_PH_TOTAL] += total_us;
        cail_prof_calls++;
    }
    for (int i = 0; i < CAIL_PH_N; ++i) g_call_us[i] = 0.0;
}

// Reads the environment into cail_global_state, once per process (the first
// MPI_Allreduce, or a configuration query before it).
void cail_load_config(void) {
    static bool loaded = false;
    if (loaded) return;
    loaded = true;
    cail_state_t &s = cail_global_state;
    const char *e = getenv(CAIL_ENV_DEBUG);
    if (e && e[0] != '\0' && e[0] != '0') s.debug = 1;
    e = getenv(CAIL_ENV_WARN);
    if (e && e[0] == '0') s.warn = 0;

    long v;
    if ((e = env_nonempty(CAIL_ENV_MSG_SMALL_THRESHOLD))) {
        if (parse_long(CAIL_ENV_MSG_SMALL_THRESHOLD, e, 1, LONG_MAX, &v)) {
            s.msg_small_threshold = (size_t)v;
            s.msg_small_threshold_set = 1;
        } else {
            s.msg_small_threshold = CAIL_DEFAULT_MSG_SMALL_THRESHOLD;
        }
    }
    if ((e = env_nonempty(CAIL_ENV_NPROCS_THRESHOLD))) {
        s.nprocs_threshold = parse_long(CAIL_ENV_NPROCS_THRESHOLD, e, 1, INT_MAX, &v)
                                 ? (int)v : (int)CAIL_DEFAULT_NPROCS_THRESHOLD;
    }
    if ((e = env_nonempty(CAIL_ENV_MIN_MSG_SIZE))) {
        s.min_msg_size = parse_long(CAIL_ENV_MIN_MSG_SIZE, e, 0, LONG_MAX, &v)
                             ? (size_t)v : (size_t)CAIL_DEFAULT_MIN_MSG_SIZE;
    }
    if ((e = env_nonempty(CAIL_ENV_ALGO))) {
        static const struct { const char *n; int a; } names[] = {
            {"auto", CAIL_ALGO_AUTO},
            {"recursive_doubling", CAIL_ALGO_RECURSIVE_DOUBLING},
            {"ring", CAIL_ALGO_RING},
            {"rabenseifner", CAIL_ALGO_RABENSEIFNER},
            {"one_shot", CAIL_ALGO_ONE_SHOT},
            {"two_shot", CAIL_ALGO_TWO_SHOT},
            {"nvls", CAIL_ALGO_NVLS},
            {"ce_two_shot", CAIL_ALGO_CE_TWO_SHOT},
        };
        bool found = false;
        for (auto &n : names)
            if (strcmp(e, n.n) == 0) { s.force_algo = n.a; found = true; }
        if (!found) {
            CAIL_ERR("unknown CAIL_ALGO='%s', using auto", e);
            s.force_algo = CAIL_ALGO_AUTO;
        }
    }
    if ((e = env_nonempty(CAIL_ENV_DEVICE_TIMEOUT_MS)))
        s.device_timeout_ms = parse_long(CAIL_ENV_DEVICE_TIMEOUT_MS, e, 1, 3600000L, &v)
                                  ? v : CAIL_DEFAULT_DEVICE_TIMEOUT_MS;
    if ((e = env_nonempty(CAIL_ENV_NVLS))) s.nvls = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_ONESHOT_MAX)))
        s.oneshot_max = parse_long(CAIL_ENV_ONESHOT_MAX, e, 0, LONG_MAX, &v) ? (size_t)v : 0;
    if ((e = env_nonempty(CAIL_ENV_FLUSH_RECV))) s.flush_recv = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_STATS))) s.stats = e[0] != '0';
    if ((e = env_nonempty("CAIL_PROFILE"))) s.profile = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_STREAM_SYNC)) && !g_stream_sync_set) s.stream_sync = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_STREAM_ORDERED)) && !g_stream_ordered_set) s.stream_ordered = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_TRACE))) {
        s.trace = fopen(e, "a");
        if (!s.trace) CAIL_ERR("cannot open CAIL_TRACE file '%s'", e);
    }
    if ((e = env_nonempty(CAIL_ENV_TUNE_FILE))) load_tune(e);
    if ((e = env_nonempty("CAIL_NVTX"))) s.nvtx = e[0] != '0';
    if ((e = env_nonempty(CAIL_ENV_DEVICE_CHECKS))) s.device_checks = e[0] != '0';
}

const cail_tune_t *cail_tune_for(int nranks) {
    for (int i = 0; i < g_ntune; ++i)
        if (g_tune[i].nranks == nranks) return &g_tune[i];
    return nullptr;
}

int cail_init(MPI_Comm comm) {
    (void)comm;
    cail_state_t &s = cail_global_state;
    if (s.initialized) return MPI_SUCCESS;
    cail_load_config();

    int rc = cail_gpu_init();
    if (rc != 0) {
        CAIL_ERR("cail_gpu_init failed (rc=%d)", rc);
        return MPI_ERR_INTERN;
    }
    s.initialized = 1;
    CAIL_DBG("initialized: min_msg_size=%zu msg_small_threshold=%zu nprocs_threshold=%d "
             "force_algo=%d debug=%d warn=%d",
             s.min_msg_size, s.msg_small_threshold, s.nprocs_threshold, s.force_algo, s.debug,
             s.warn);
    return MPI_SUCCESS;
}

void cail_finalize(void) {
    cail_state_t &s = cail_global_state;
    if (!s.initialized) return;
    if (s.stats) {
        const cail_stats_t &c = cail_counters;
        fprintf(stderr,
                "[cail] stats: calls=%llu passthrough=%llu rd=%llu ring=%llu rab=%llu "
                "one_shot=%llu two_shot=%llu nvls=%llu ce_two_shot=%llu copy=%llu bytes=%llu reg_hits=%llu "
                "reg_misses=%llu device_errors=%llu\n",
                c.calls, c.passthrough, c.by_algo[1], c.by_algo[2], c.by_algo[3], c.by_algo[4],
                c.by_algo[5], c.by_algo[6], c.by_algo[7], c.by_algo[8], c.bytes, c.reg_hits, c.reg_misses,
                c.device_errors);
    }
    if (s.profile && cail_prof_calls) {
        const double n = (double)cail_prof_calls;
        fprintf(stderr,
                "[cail] profile: %llu calls, mean us: filter=%.2f order=%.2f launch=%.2f wait=%.2f "
                "hostsync=%.2f total=%.2f\n",
                cail_prof_calls, cail_prof_us[CAIL_PH_FILTER] / n, cail_prof_us[CAIL_PH_SETUP] / n,
                cail_prof_us[CAIL_PH_LAUNCH] / n, cail_prof_us[CAIL_PH_WAIT] / n,
                cail_prof_us[CAIL_PH_HOSTSYNC] / n, cail_prof_us[CAIL_PH_TOTAL] / n);
    }
    cail_gpu_finalize();
    cail_buf_finalize();
    if (s.trace) { fclose(s.trace); s.trace = nullptr; }
    s.initialized = 0;
}

int cail_is_initialized(void) { return cail_global_state.initialized; }

void cail_trace_call(int algo, size_t bytes, int count, cail_datatype_t dt, cail_op_t op,
                     int nprocs, double usec) {
    FILE *f = cail_global_state.trace;
    if (!f) return;
    fprintf(f, "%s,%zu,%d,%s,%s,%d,%.3f\n", algo == -3 ? "pmpi" : cail_algo_name(algo), bytes,
            count, cail_dtype_name(dt), cail_op_name(op), nprocs, usec);
}

const char *cail_version(void) {
#ifdef CAIL_HOST_PATH
    return "0.1.0 (host)";
#else
    return "0.1.0 (cuda sm_100a)";
#endif
}

const char *cail_last_algorithm(void) {
    if (cail_last_algo == -2) return "none";
    if (cail_last_algo == -3) return "pmpi";
    return cail_algo_name(cail_last_algo);
}

int cail_set_stream_sync(int mode) {
    int prev = cail_global_state.stream_sync;
    cail_global_state.stream_sync = mode ? 1 : 0;
    g_stream_sync_set = true;
    return prev;
}

int cail_set_stream_ordered(int mode) {
    int prev = cail_global_state.stream_ordered;
    cail_global_state.stream_ordered = mode ? 1 : 0;
    g_stream_ordered_set = true;
    return prev;
}

int cail_get_stats(cail_stats_t *out) {
    if (!out) return MPI_ERR_ARG;
    *out = cail_counters;
    return MPI_SUCCESS;
}

#ifdef CAIL_HOST_PATH
int cail_comm_uses_nvlink(MPI_Comm comm) {
    (void)comm;
    return 0;
}
int cail_comm_uses_nvls(MPI_Comm comm) {
    (void)comm;
    return 0;
}
#endif

}  // extern "C"
