// cail_dev_bulkcopy.cu — device-to-device copy through TMA bulk copies.
//
// With one rank an allreduce is a plain copy.  This kernel moves the 16-byte
// aligned body of the buffer with the bulk-copy engine: per CTA one thread
// streams chunks global -> shared (cp.async.bulk with an mbarrier that counts
// the arriving bytes) and shared -> global (cp.async.bulk bulk_group) through
// a ring of kBulkStages shared-memory stages, so address generation and the
// data path stay off the SM's load/store pipes.  No multicast is used.  The
// unaligned head and the tail (< 16 bytes each) are copied with plain loads
// by the other threads.
//
// Every mbarrier wait is bounded (spin_limit polls of try_wait); on expiry the
// kernel records code 1 in *status, waits (bounded again) for its own loads
// in flight and for its stores, and returns.
//
// Experimental: reached only from the single-GPU harness
// (cail_bench_kernel_local, kernel 3); no allreduce path launches it.
#include <cuda_runtime.h>
#include <stdint.h>

namespace cail {

namespace {

constexpr int kBulkStages = 4;
constexpr uint32_t kBulkChunk = 32u << 10;  // bytes per stage, a multiple of 16

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, unsigned long long limit) {
    for (unsigned long long i = 0; i < limit; ++i) {
        uint32_t done;
        asm volatile(
            "{\n\t.reg .pred p;\n\t"
            "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
            "selp.u32 %0, 1, 0, p;\n\t}"
            : "=r"(done)
            : "r"(bar), "r"(parity)
            : "memory");
        if (done) return true;
    }
    return false;
}

__device__ __forceinline__ void bulk_load(uint32_t smem, const char *gsrc, uint32_t n, uint32_t bar) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(n) : "memory");
    asm volatile("cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem),
                 "l"(gsrc), "r"(n), "r"(bar)
                 : "memory");
}

__device__ __forceinline__ void bulk_store(char *gdst, uint32_t smem, uint32_t n) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(smem), "r"(n)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

// body: [src + head, src + head + body) -> same offsets of dst, body % 16 == 0,
// both addresses 16-byte aligned there.
__global__ void __launch_bounds__(128) bulk_copy_kernel(char *dst, const char *src, size_t head, size_t body,
                                                        size_t bytes, unsigned long long spin_limit, int *status) {
    extern __shared__ __align__(128) unsigned char stage[];
    __shared__ __align__(8) uint64_t bars[kBulkStages];

    // ragged head and tail: plain copies by block 0's other threads
    if (blockIdx.x == 0 && threadIdx.x > 0) {
        for (size_t i = threadIdx.x - 1; i < head; i += blockDim.x - 1) dst[i] = src[i];
        for (size_t i = head + body + threadIdx.x - 1; i < bytes; i += blockDim.x - 1) dst[i] = src[i];
    }
    if (threadIdx.x != 0) return;

    const size_t nchunks = (body + kBulkChunk - 1) / kBulkChunk;
    const size_t mine = nchunks > blockIdx.x ? (nchunks - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
    if (mine == 0) return;
    for (int s = 0; s < kBulkStages; ++s)
        asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(&bars[s])), "r"(1) : "memory");
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");

    auto chunk_off = [&](size_t k) { return head + (blockIdx.x + k * gridDim.x) * (size_t)kBulkChunk; };
    auto chunk_len = [&](size_t k) {
        const size_t off = chunk_off(k), end = head + body;
        return (uint32_t)(end - off < kBulkChunk ? end - off : kBulkChunk);
    };
    auto stage_at = [&](size_t k) { return smem_u32(stage + (k % kBulkStages) * kBulkChunk); };
    auto bar_at = [&](size_t k) { return smem_u32(&bars[k % kBulkStages]); };

    uint32_t parity_bits = 0;  // bit s: parity of the next completion of stage s
    size_t issued = 0;
    for (; issued < mine && issued < (size_t)kBulkStages; ++issued)
        bulk_load(stage_at(issued), src + chunk_off(issued), chunk_len(issued), bar_at(issued));

    size_t failed_at = mine;  // first chunk whose load never arrived
    for (size_t k = 0; k < mine; ++k) {
        const int s = (int)(k % kBulkStages);
        if (!bar_wait(bar_at(k), (parity_bits >> s) & 1u, spin_limit)) {
            failed_at = k;
            break;
        }
        parity_bits ^= 1u << s;
        bulk_store(dst + chunk_off(k), stage_at(k), chunk_len(k));
        // refill the stage of store k-1 once that store has read it (all
        // bulk groups but the newest, store k, are done reading)
        if (k >= 1 && issued < mine) {
            asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
            bulk_load(stage_at(issued), src + chunk_off(issued), chunk_len(issued), bar_at(issued));
            ++issued;
        }
    }
    if (failed_at < mine) {
        atomicExch(status, 1);
        // loads still in flight (chunks failed_at .. issued-1, at most one
        // per stage) land in shared memory: let them finish, bounded, before
        // the CTA's shared memory goes away
        for (size_t k = failed_at; k < issued; ++k) {
            const int s = (int)(k % kBulkStages);
            if (bar_wait(bar_at(k), (parity_bits >> s) & 1u, spin_limit)) parity_bits ^= 1u << s;
        }
    }
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}

}  // namespace

// Copies bytes from src to dst (device memory of the current GPU) with the
// bulk-copy kernel.  src and dst must share their alignment modulo 16.
cudaError_t launch_bulk_copy(char *dst, const char *src, size_t bytes, int blocks, unsigned long long spin_limit,
                             int *status, cudaStream_t s) {
    if ((((uintptr_t)src ^ (uintptr_t)dst) & 15) != 0) return cudaErrorInvalidValue;
    const size_t head = ((16 - ((uintptr_t)src & 15)) & 15) < bytes ? ((16 - ((uintptr_t)src & 15)) & 15) : bytes;
    const size_t body = (bytes - head) & ~(size_t)15;
    const int smem = kBulkStages * (int)kBulkChunk;
    // per device, so set on every launch (cheap)
    cudaError_t e = cudaFuncSetAttribute(bulk_copy_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
    if (e != cudaSuccess) return e;
    bulk_copy_kernel<<<blocks, 128, smem, s>>>(dst, src, head, body, bytes, spin_limit, status);
    return cudaGetLastError();
}

}  // namespace cail
