// cail_buf.cpp — grow-only scratch buffer for the point-to-point algorithms.
//
// Same contract as the reference (src/core/cail_buf.c:28-87 there): one
// process-wide buffer, reallocated only when a request exceeds its size,
// never shrunk, released at MPI_Finalize.  Device memory in the CUDA build,
// host memory in the host-only build (both through cail_gpu_malloc).  The
// NVLink kernels do not use it: their scratch lives in the per-communicator
// IPC workspace.
#include <stdlib.h>

#include "../gpu/cail_gpu.h"
#include "cail_internal.h"

namespace {
void *g_buf = nullptr;
size_t g_size = 0;

// Host-side fault injection (tests only): CAIL_FI_SCRATCH_FAIL=1 makes every
// scratch request fail as a failed allocation would, so that the shim's
// fallback to PMPI_Allreduce after a dispatch error can be tested.
bool fi_scratch_fail() {
    static const bool v = [] {
        const char *e = getenv("CAIL_FI_SCRATCH_FAIL");
        return e && e[0] == '1';
    }();
    return v;
}
}  // namespace

extern "C" {

int cail_buf_get_tmp(void **ptr, size_t size) {
    if (size == 0) {
        *ptr = nullptr;
        return MPI_SUCCESS;
    }
    if (fi_scratch_fail()) {
        CAIL_ERR("scratch request of %zu bytes failed (injected by CAIL_FI_SCRATCH_FAIL)", size);
        return MPI_ERR_NO_MEM;
    }
    if (size > g_size) {
        if (g_buf) cail_gpu_free(g_buf);
        g_buf = nullptr;
        g_size = 0;
        int rc = cail_gpu_malloc(&g_buf, size);
        if (rc != 0 || !g_buf) {
            CAIL_ERR("cail_gpu_malloc(%zu) failed (rc=%d)", size, rc);
            g_buf = nullptr;
            return MPI_ERR_NO_MEM;
        }
        g_size = size;
        CAIL_DBG("buf: allocated %zu bytes", size);
    } else {
        CAIL_DBG("buf: reusing cached %zu bytes (requested %zu)", g_size, size);
    }
    *ptr = g_buf;
    return MPI_SUCCESS;
}

void cail_buf_release_tmp(void *ptr) { (void)ptr; }

void cail_buf_finalize(void) {
    if (g_buf) cail_gpu_free(g_buf);
    g_buf = nullptr;
    g_size = 0;
}

}  // extern "C"
