// cail_gpu.h — backend seam between the algorithms and the memory they run on.
//
// The same nine entry points as the reference's backend interface
// (src/gpu/cail_gpu.h:19-47 there), implemented by
//   gpu/cuda/  CUDA runtime + sm_100a kernels (default build)
//   gpu/host/  host memory and a templated host reduction (CAIL_HOST_PATH)
// A ROCm backend would plug in here; none is built for B200.
#pragma once

#include <stddef.h>

#include "../core/cail_types.h"

#ifdef __cplusplus
extern "C" {
#endif

/* 1 if ptr is device (or managed) memory.  Makes the buffer's device current
 * for the call, remembering the caller's; cail_gpu_restore_device() puts the
 * caller's back when the call returns. */
int cail_gpu_is_device_pointer(const void *ptr);
void cail_gpu_restore_device(void);

/* inout[i] = op(inout[i], in[i]) for i in [0, count) */
int cail_gpu_reduce_local(const void *in, void *inout, size_t count, cail_datatype_t dtype,
                          cail_op_t op);

int cail_gpu_malloc(void **ptr, size_t size);
int cail_gpu_free(void *ptr);

/* Copy between device buffers or device<->host; returns after completion. */
int cail_gpu_memcpy(void *dst, const void *src, size_t size);

int cail_gpu_synchronize(void);

/* The allreduce of a one-rank communicator: dst = src (nothing to do when they
 * are the same buffer).  Runs on the legacy stream (stream sync mode 1) with
 * cail's copy kernel, or cudaMemcpyAsync above CAIL_COPY_KERNEL_MAX bytes, and
 * returns after completion unless stream-ordered completion is on.  0 or -1. */
int cail_gpu_single_rank(const void *src, void *dst, size_t bytes);

/* Read fence after a network receive into device memory: a 1-byte
 * device->host read of the last byte drains earlier posted writes (NIC RDMA,
 * GDRCopy stores).  No-op when CAIL_FLUSH_RECV=0 or in the host build. */
int cail_gpu_flush_recv_buf(const void *recv_buf, size_t recv_bytes);

int cail_gpu_init(void);
void cail_gpu_finalize(void);

#ifdef __cplusplus
}
#endif
