// cail_dev_localbench.cu — single-GPU harness for the NVLink kernels.
//
// cail_bench_kernel_local() launches the one-shot or two-shot kernel of a
// P-rank communicator with every "peer" emulated by a separate buffer on
// the current GPU: the two-shot kernel reads P inputs and writes P outputs,
// the one-shot kernel pushes into P scratch areas and folds P slots, with
// its peers' arrival flags set in advance (so it never waits).  The fold
// kernel of the copy-engine two-shot runs on P local sources as it does in
// production (there it is local already).  Kernel 3 is the experimental
// TMA bulk-copy kernel (a one-rank allreduce is a copy), checked against its
// source after timing.  The
// instruction stream is the production one; only NVLink is replaced by
// local HBM.  This is the case a profiler can capture on one GPU.
#include <cuda_runtime.h>
#include <string.h>

#include <vector>

#include "../core/cail_internal.h"
#include "cail_dev_kernels.cuh"

namespace {

// Counts 16-byte words that differ between a and b (n16 words).
__global__ void count_diff(const uint4 *a, const uint4 *b, size_t n16, unsigned long long *bad) {
    unsigned long long mine = 0;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n16; i += (size_t)gridDim.x * blockDim.x) {
        const uint4 x = a[i], y = b[i];
        mine += (x.x != y.x) | (x.y != y.y) | (x.z != y.z) | (x.w != y.w);
    }
    if (mine) atomicAdd(bad, mine);
}

__global__ void fill_pattern(uint32_t *p, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = (uint32_t)(i * 2654435761u) ^ 0x5bd1e995u;
}

struct Bufs {
    std::vector<void *> ptrs;
    ~Bufs() {
        for (void *p : ptrs) cudaFree(p);
    }
    char *get(size_t n) {
        void *p = nullptr;
        if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
        cudaMemset(p, 0, n);
        ptrs.push_back(p);
        return (char *)p;
    }
};

}  // namespace

// kernel: 0 = one_shot, 1 = two_shot, 2 = fold (P sources of `bytes`),
// 3 = bulk copy of `bytes` (P ignored; returns -2 if the copy differs).  Runs `iters` launches of a float SUM
// over `bytes` bytes per rank with P emulated ranks (2..8) and writes the
// mean time per launch in milliseconds to *ms.  Returns 0 or -1.
extern "C" int cail_bench_kernel_local(int kernel, int P, size_t bytes, int iters, float *ms) {
    if (P < 1 || P > cail::kMaxRanks || iters < 1 || !ms) return -1;
    const size_t count = bytes / 4;
    const size_t esz = 4;
    Bufs b;
    cudaStream_t s = nullptr;
    cudaEvent_t e0 = nullptr, e1 = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return -1;
    cudaEventCreate(&e0);
    cudaEventCreate(&e1);
    int sms = 148, dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cail::DevStatus *st = (cail::DevStatus *)b.get(sizeof(cail::DevStatus));
    int rc = 0;
    if (kernel == 0) {
        const size_t slot = bytes;
        char *src = b.get(bytes), *dst = b.get(bytes);
        uint32_t *flags = (uint32_t *)b.get(cail::kFlagWords * 4);
        std::vector<char *> area(P);
        for (int q = 0; q < P; ++q) area[q] = b.get(slot * P);
        if (!src || !dst || !flags || !st) { rc = -1; goto out; }
        // every peer has already arrived for all epochs used below
        cudaMemset(flags, 0x7f, cail::kFlagWords * 4);
        cail::OneShotArgs a;
        memset(&a, 0, sizeof(a));
        a.src = src;
        a.dst = dst;
        a.count = count;
        for (int q = 0; q < P; ++q) {
            a.slot_out[q] = area[q];  // this rank is rank 0: slot 0 of each peer's area
            a.peer_flags[q] = flags;
        }
        a.slot_in = area[0];
        a.slot_bytes = slot;
        a.my_flags = flags;
        a.P = P;
        a.rank = 0;
        a.epoch = 1;
        a.timeout_ns = 1000000000ull;
        a.status = st;
        size_t vec = (bytes + 15) / 16;
        size_t want = (vec + 1023) / 1024;
        int blocks = (int)(want < 1 ? 1 : (want > (size_t)cail::kMaxBlocks ? cail::kMaxBlocks : want));
        cail::launch_oneshot(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);  // warm-up
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) cail::launch_oneshot(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);
        cudaEventRecord(e1, s);
    } else if (kernel == 3) {
        char *src = b.get(bytes + 16), *dst = b.get(bytes + 16);
        int *bst = (int *)b.get(sizeof(int));
        unsigned long long *bad = (unsigned long long *)b.get(sizeof(unsigned long long));
        if (!src || !dst || !bst || !bad || bytes % 16) { rc = -1; goto out; }
        fill_pattern<<<1024, 256, 0, s>>>((uint32_t *)src, bytes / 4);
        const unsigned long long limit = 1ull << 24;  // try_wait polls before giving up
        int blocks = sms;
        if (cail::launch_bulk_copy(dst, src, bytes, blocks, limit, bst, s) != cudaSuccess) { rc = -1; goto out; }
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) cail::launch_bulk_copy(dst, src, bytes, blocks, limit, bst, s);
        cudaEventRecord(e1, s);
        count_diff<<<1024, 256, 0, s>>>((const uint4 *)src, (const uint4 *)dst, bytes / 16, bad);
        unsigned long long h_bad = 0;
        int h_st = 0;
        if (cudaStreamSynchronize(s) != cudaSuccess ||
            cudaMemcpy(&h_bad, bad, sizeof(h_bad), cudaMemcpyDeviceToHost) != cudaSuccess ||
            cudaMemcpy(&h_st, bst, sizeof(h_st), cudaMemcpyDeviceToHost) != cudaSuccess) {
            rc = -1;
            goto out;
        }
        if (h_bad || h_st) rc = -2;
    } else if (kernel == 2) {
        cail::FoldArgs a;
        memset(&a, 0, sizeof(a));
        for (int q = 0; q < P; ++q) {
            a.src[q] = b.get(bytes);
            if (!a.src[q]) { rc = -1; goto out; }
        }
        a.dst = b.get(bytes);
        if (!a.dst) { rc = -1; goto out; }
        a.P = P;
        a.count = count;
        size_t want = (bytes / 16 + 1023) / 1024;
        int blocks = (int)(want > (size_t)(sms * 2) ? sms * 2 : (want < 1 ? 1 : want));
        cail::launch_fold(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) cail::launch_fold(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);
        cudaEventRecord(e1, s);
    } else {
        cail::TwoShotArgs a;
        memset(&a, 0, sizeof(a));
        for (int q = 0; q < P; ++q) {
            a.src[q] = b.get(bytes);
            a.dst[q] = b.get(bytes);
            if (!a.src[q] || !a.dst[q]) { rc = -1; goto out; }
        }
        a.P = P;
        a.rank = 0;
        a.count = count;
        a.vector_ok = 1;
        a.nvec = count * esz / 16;
        a.head = 0;
        size_t work = a.nvec / P + 1;
        size_t want = (work + 511) / 512;
        int blocks = (int)(want > (size_t)(sms * 2) ? sms * 2 : (want < 1 ? 1 : want));
        cail::launch_twoshot(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) cail::launch_twoshot(CAIL_SUM, CAIL_EC_F32, a, blocks, 512, s);
        cudaEventRecord(e1, s);
    }
    if (cudaStreamSynchronize(s) != cudaSuccess || cudaGetLastError() != cudaSuccess) {
        rc = -1;
    } else {
        float t = 0;
        cudaEventElapsedTime(&t, e0, e1);
        *ms = t / iters;
    }
out:
    cudaEventDestroy(e0);
    cudaEventDestroy(e1);
    cudaStreamDestroy(s);
    return rc;
}
