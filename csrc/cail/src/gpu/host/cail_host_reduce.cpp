// cail_host_reduce.cpp — host-only backend (CAIL_HOST_PATH builds).
//
// Plays the role of the reference's host path (src/gpu/host/cail_host_reduce.c
// there), but reduces with cail's own templated loops instead of forwarding
// to MPI_Reduce_local, so the host build needs nothing from the MPI library
// beyond point-to-point and the semantics match the device kernels exactly
// (cail_ops.h).  The loops are written so the compiler vectorises them.
#include <stdlib.h>
#include <string.h>

#include "../../core/cail_internal.h"
#include "../cail_gpu.h"
#include "../cail_ops.h"

namespace {

template <int OP, int EC>
void reduce_loop(const void *in, void *inout, size_t n) {
    using T = typename cail::EcType<EC>::T;
    const T *__restrict a = (const T *)in;
    T *__restrict b = (T *)inout;
    for (size_t i = 0; i < n; ++i) b[i] = cail::apply<OP, T>(b[i], a[i]);
}

struct Run {
    const void *in;
    void *io;
    size_t n;
    template <int OP, int EC> void operator()() { reduce_loop<OP, EC>(in, io, n); }
};

}  // namespace

extern "C" {

int cail_gpu_is_device_pointer(const void *ptr) {
    (void)ptr;
    return 0;
}

void cail_gpu_restore_device(void) {}

int cail_gpu_reduce_local(const void *in, void *inout, size_t count, cail_datatype_t dtype,
                          cail_op_t op) {
    cail_elem_class_t ec = cail_elem_class(dtype);
    Run run{in, inout, count};
    if (!cail::dispatch_op_class((int)op, (int)ec, run)) {
        CAIL_WARN("gpu_reduce_local: no reduction for dtype=%s op=%s", cail_dtype_name(dtype),
                  cail_op_name(op));
        return -1;
    }
    return 0;
}

int cail_gpu_malloc(void **ptr, size_t size) {
    *ptr = malloc(size);
    return *ptr ? 0 : -1;
}

int cail_gpu_free(void *ptr) {
    free(ptr);
    return 0;
}

int cail_gpu_memcpy(void *dst, const void *src, size_t size) {
    memmove(dst, src, size);
    return 0;
}

int cail_gpu_synchronize(void) { return 0; }
int cail_gpu_flush_recv_buf(const void *recv_buf, size_t recv_bytes) {
    (void)recv_buf;
    (void)recv_bytes;
    return 0;
}
int cail_gpu_init(void) { return 0; }
void cail_gpu_finalize(void) {}

}  // extern "C"
