// cail-mpirun — process launcher for minimpi jobs on one node.
//
//   cail-mpirun -np N [-x VAR[=VALUE]]... [--timeout SECONDS] [--] program [args...]
//
// Creates the job's shared-memory segment, forks N ranks (environment:
// CMPI_SHM, CMPI_RANK, CMPI_SIZE, CMPI_LOCAL_RANK plus every -x VAR=VALUE),
// and waits.  If one rank fails (non-zero exit or a signal) the others are
// terminated and its exit status is returned; on --timeout every rank is
// killed and 124 is returned.  `-x VAR` without a value exports the
// launcher's own value, as other launchers do.
#include <errno.h>
#include <fcntl.h>
#include <signal.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <sys/wait.h>
#include <time.h>
#include <unistd.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "../src/cmpi_internal.h"

static std::vector<pid_t> g_children;
static volatile sig_atomic_t g_signalled = 0;

static void on_signal(int sig) { g_signalled = sig; }

static void kill_all(int sig) {
    for (pid_t p : g_children)
        if (p > 0) kill(p, sig);
}

static double mono() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec + 1e-9 * ts.tv_nsec;
}

static void usage() {
    std::fprintf(stderr,
                 "usage: cail-mpirun -np N [-x VAR[=VALUE]]... [--timeout SECONDS] [--] program "
                 "[args...]\n");
}

int main(int argc, char **argv) {
    int np = 1;
    double timeout = 0;
    std::vector<std::pair<std::string, std::string>> exports;
    int i = 1;
    for (; i < argc; ++i) {
        std::string a = argv[i];
        if ((a == "-np" || a == "-n") && i + 1 < argc) {
            np = atoi(argv[++i]);
        } else if (a == "-x" && i + 1 < argc) {
            std::string kv = argv[++i];
            size_t eq = kv.find('=');
            if (eq == std::string::npos) {
                const char *v = getenv(kv.c_str());
                if (v) exports.push_back({kv, v});
            } else {
                exports.push_back({kv.substr(0, eq), kv.substr(eq + 1)});
            }
        } else if (a == "--timeout" && i + 1 < argc) {
            timeout = atof(argv[++i]);
        } else if (a == "--") {
            ++i;
            break;
        } else if (a == "-h" || a == "--help") {
            usage();
            return 0;
        } else {
            break;
        }
    }
    if (i >= argc || np < 1) {
        usage();
        return 2;
    }

    uint32_t ring = cmpi::default_ring_bytes((uint32_t)np);
    size_t bytes = cmpi::segment_bytes((uint32_t)np, ring);
    char name[96];
    snprintf(name, sizeof(name), "/cmpi_l%d_%lx", (int)getpid(), (unsigned long)time(nullptr));
    shm_unlink(name);
    int fd = shm_open(name, O_CREAT | O_EXCL | O_RDWR, 0600);
    if (fd < 0 || ftruncate(fd, (off_t)bytes) != 0) {
        std::fprintf(stderr, "cail-mpirun: cannot create shared memory %s: %s\n", name, strerror(errno));
        return 1;
    }
    void *base = mmap(nullptr, bytes, PROT_READ | PROT_WRITE, MAP_SHARED, fd, 0);
    close(fd);
    if (base == MAP_FAILED) {
        std::fprintf(stderr, "cail-mpirun: mmap failed: %s\n", strerror(errno));
        shm_unlink(name);
        return 1;
    }
    auto *hdr = (cmpi::SegHeader *)base;
    hdr->nranks = (uint32_t)np;
    hdr->ring_bytes = ring;
    hdr->nonce = (uint64_t)getpid();
    hdr->magic.store(cmpi::kMagic, std::memory_order_release);

    struct sigaction sa;
    memset(&sa, 0, sizeof(sa));
    sa.sa_handler = on_signal;
    sigaction(SIGINT, &sa, nullptr);
    sigaction(SIGTERM, &sa, nullptr);

    g_children.assign(np, -1);
    for (int r = 0; r < np; ++r) {
        pid_t pid = fork();
        if (pid < 0) {
            std::fprintf(stderr, "cail-mpirun: fork failed: %s\n", strerror(errno));
            kill_all(SIGKILL);
            shm_unlink(name);
            return 1;
        }
        if (pid == 0) {
            signal(SIGINT, SIG_DFL);
            signal(SIGTERM, SIG_DFL);
            setenv("CMPI_SHM", name, 1);
            setenv("CMPI_RANK", std::to_string(r).c_str(), 1);
            setenv("CMPI_SIZE", std::to_string(np).c_str(), 1);
            setenv("CMPI_LOCAL_RANK", std::to_string(r).c_str(), 1);
            for (auto &kv : exports) setenv(kv.first.c_str(), kv.second.c_str(), 1);
            execvp(argv[i], argv + i);
            std::fprintf(stderr, "cail-mpirun: cannot execute %s: %s\n", argv[i], strerror(errno));
            _exit(127);
        }
        g_children[r] = pid;
    }

    int result = 0;
    int alive = np;
    bool failing = false;
    double t0 = mono(), kill_at = 0;
    while (alive > 0) {
        int status = 0;
        pid_t p = waitpid(-1, &status, WNOHANG);
        if (p > 0) {
            int rank = -1;
            for (int r = 0; r < np; ++r)
                if (g_children[r] == p) { rank = r; g_children[r] = -1; }
            --alive;
            int code = WIFEXITED(status) ? WEXITSTATUS(status) : 128 + WTERMSIG(status);
            if (code != 0 && !failing) {
                std::fprintf(stderr, "cail-mpirun: rank %d (pid %d) exited with status %d; "
                             "terminating the job\n", rank, (int)p, code);
                result = code;
                failing = true;
                kill_all(SIGTERM);
                kill_at = mono() + 3.0;
            }
            continue;
        }
        if (p < 0 && errno == ECHILD) break;
        if (g_signalled && !failing) {
            failing = true;
            result = 128 + g_signalled;
            kill_all(SIGTERM);
            kill_at = mono() + 3.0;
        }
        if (timeout > 0 && !failing && mono() - t0 > timeout) {
            std::fprintf(stderr, "cail-mpirun: timeout after %.0f s; killing the job\n", timeout);
            failing = true;
            result = 124;
            kill_all(SIGKILL);
        }
        if (failing && kill_at > 0 && mono() > kill_at) {
            kill_all(SIGKILL);
            kill_at = 0;
        }
        usleep(2000);
    }
    munmap(base, bytes);
    shm_unlink(name);
    return result;
}
