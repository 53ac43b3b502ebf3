// cail_kbench.cu — one-GPU harness for cail's kernels (test-only library,
// libcail_kbench.so; the interposer itself does not contain it).
//
// Two entry points:
//
// cail_bench_kernel_local() times one kernel of libcail on the current GPU,
// with every "peer" of a P-rank communicator emulated by a separate buffer
// on the same GPU.  The instruction stream is the production one; only
// NVLink is replaced by local HBM, which is the case a profiler can capture
// on one GPU.
//
// cail_emulate_push() runs the push two-shot allreduce of P ranks on the
// current GPU in one cooperative launch: CTAs [r * G, (r + 1) * G) play rank
// r, with rank r's workspace, flag array, input and output all being
// separate buffers of this GPU.  The CTAs of different ranks wait on one
// another through the flags exactly as across GPUs, and the cooperative
// launch guarantees that they are all resident.  The caller passes the P
// inputs and outputs (device pointers) and checks the outputs itself.
#include <cuda_runtime.h>
#include <string.h>

#include <vector>

#include "../cail/src/core/cail_types.h"
#include "../cail/src/dev/cail_dev_kernels.cuh"

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

// Emulated ranks' workspaces: rank q's is [flag area | one-shot area | RS area
// | AG area], all on this GPU.
struct Emu {
    Bufs b;
    char *ws[cail::kMaxRanks] = {};
    size_t os_area = 0, area = 0;
    int os_g = 0;
    uint32_t epoch = 0;
    cail::DevStatus *st = nullptr;
    static constexpr size_t kFlags = 64 << 10;
    bool init(int P, int G, size_t piece) {
        os_g = G;
        os_area = ((size_t)cail::kOsSlots * G * P * piece + 255) / 256 * 256;
        area = ((size_t)2 * G * P * piece + 255) / 256 * 256;
        for (int q = 0; q < P; ++q)
            if (!(ws[q] = b.get(kFlags + os_area + 2 * area))) return false;
        st = (cail::DevStatus *)b.get(sizeof(cail::DevStatus));
        return st != nullptr;
    }
    // fills the per-call part of a push (epochs advance by the rounds of the call)
    void args(cail::PushArgs &a, int P, unsigned long long timeout_ns) {
        for (int q = 0; q < P; ++q) {
            a.flags[q] = (uint32_t *)ws[q];
            a.rs[q] = ws[q] + kFlags + os_area;
            a.ag[q] = ws[q] + kFlags + os_area + area;
        }
        a.rank0 = 0;
        a.area = area;
        a.epoch0 = epoch + 1;
        epoch += (uint32_t)a.rounds;
        a.timeout_ns = timeout_ns;
        a.status = st;
    }
    void args(cail::OneShotArgs &a, int P, unsigned long long timeout_ns) {
        for (int q = 0; q < P; ++q) {
            a.flags[q] = (uint32_t *)ws[q];
            a.slots[q] = ws[q] + kFlags;
            a.rounds_done[q] = (uint32_t *)ws[q] + cail::kOsRoundsBase;
        }
        a.rank0 = 0;
        a.area = os_area;
        a.sg = os_g;  // slot stride: the largest CTA count the area was sized for
        a.timeout_ns = timeout_ns;
        a.status = st;
    }
};

// The slice table and launch shape, computed as the production path does.
void shape(cail::PushArgs &a, int P, size_t count, size_t esz, bool vec, int G, size_t piece) {
    const size_t bytes = count * esz, unit = vec ? 16 : esz, nunits = bytes / unit;
    size_t mx = 0;
    for (int q = 0; q < P; ++q) a.slice_off[q] = nunits * q / P * unit;
    a.slice_off[P] = bytes;
    for (int q = 0; q < P; ++q) mx = mx > a.slice_off[q + 1] - a.slice_off[q] ? mx : a.slice_off[q + 1] - a.slice_off[q];
    a.max_slice = mx;
    a.piece = piece;
    a.G = G;
    a.rounds = (int)((mx + (size_t)G * piece - 1) / ((size_t)G * piece));
    if (a.rounds < 1) a.rounds = 1;
    a.P = P;
    a.vec = vec ? 1 : 0;
}

}  // namespace

// Runs `calls` back-to-back push two-shot allreduces of P emulated ranks
// (2..8) over srcs[r] -> dsts[r] (device buffers of the current GPU, `count`
// elements of storage class ec, operator op: cail_elem_class_t and
// cail_op_t values).  G CTAs per rank (0: as many as can be co-resident) and
// `piece` bytes per CTA, round and slice (0: 32 KiB; a multiple of 16).
// options: bit 0 turns on the kernel's argument checks (CAIL_DEVICE_CHECKS);
// bit 1 passes one round too few, an inconsistent argument that the checks
// must catch (unchecked, the kernel would only leave the end of the longest
// slice unreduced: it never reaches beyond its buffers).
// Returns 0, the device status code (1: a wait timed out, 2: an argument
// check failed), or -1 on a CUDA or argument error.
extern "C" int cail_emulate_push(int P, const void *const *srcs, void *const *dsts, size_t count, int ec, int op,
                                 int G, size_t piece, int calls, int options) {
    if (P < 2 || P > cail::kMaxRanks || calls < 1 || !srcs || !dsts) return -1;
    static const int esz_of[CAIL_EC_NUM] = {1, 1, 2, 2, 4, 4, 8, 8, 4, 8};
    if (ec < 0 || ec >= CAIL_EC_NUM) return -1;
    const size_t esz = (size_t)esz_of[ec];
    if (piece == 0) piece = 32 << 10;
    if (piece % 16) return -1;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int gmax = cail::push_max_ctas(P, sms);
    if (G <= 0 || G > gmax) G = gmax;
    bool vec = true;
    for (int q = 0; q < P; ++q)
        if ((((uintptr_t)srcs[q]) | ((uintptr_t)dsts[q])) & 15) vec = false;
    Emu emu;
    if (!emu.init(P, G, piece)) return -1;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return -1;
    int rc = 0;
    for (int c = 0; c < calls && rc == 0; ++c) {
        cail::PushArgs a;
        memset(&a, 0, sizeof(a));
        shape(a, P, count, esz, vec, G, piece);
        for (int q = 0; q < P; ++q) {
            a.src[q] = (const char *)srcs[q];
            a.dst[q] = (char *)dsts[q];
        }
        emu.args(a, P, 2000000000ull);
        a.checks = options & 1;
        if ((options & 2) && a.rounds > 1) a.rounds -= 1;
        if (cail::launch_push(op, ec, a, P, true, s) != cudaSuccess) rc = -1;
    }
    cail::DevStatus h;
    memset(&h, 0, sizeof(h));
    if (cudaStreamSynchronize(s) != cudaSuccess ||
        cudaMemcpy(&h, emu.st, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = -1;
    else if (rc == 0 && h.code != 0)
        rc = h.code;
    cudaStreamDestroy(s);
    cudaGetLastError();
    return rc;
}

// The one-shot allreduce of P emulated ranks, as cail_emulate_push (same
// arguments; `piece` 0: 16 KiB; options bit 0: argument checks).
extern "C" int cail_emulate_oneshot(int P, const void *const *srcs, void *const *dsts, size_t count, int ec,
                                    int op, int G, size_t piece, int calls, int options) {
    if (P < 2 || P > cail::kMaxRanks || calls < 1 || !srcs || !dsts) return -1;
    static const int esz_of[CAIL_EC_NUM] = {1, 1, 2, 2, 4, 4, 8, 8, 4, 8};
    if (ec < 0 || ec >= CAIL_EC_NUM) return -1;
    const size_t esz = (size_t)esz_of[ec];
    if (piece == 0) piece = 16 << 10;
    if (piece % 16) return -1;
    int dev = 0, sms = 148;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    const int gmax = cail::push_max_ctas(P, sms);
    if (G <= 0 || G > gmax) G = gmax;
    bool vec = true;
    for (int q = 0; q < P; ++q)
        if ((((uintptr_t)srcs[q]) | ((uintptr_t)dsts[q])) & 15) vec = false;
    Emu emu;
    if (!emu.init(P, G, piece)) return -1;
    cudaStream_t s = nullptr;
    if (cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking) != cudaSuccess) return -1;
    int rc = 0;
    for (int c = 0; c < calls && rc == 0; ++c) {
        cail::OneShotArgs a;
        memset(&a, 0, sizeof(a));
        a.bytes = count * esz;
        a.piece = piece;
        a.P = P;
        a.G = G;
        a.vec = vec ? 1 : 0;
        for (int q = 0; q < P; ++q) {
            a.src[q] = (const char *)srcs[q];
            a.dst[q] = (char *)dsts[q];
        }
        emu.args(a, P, 2000000000ull);
        a.checks = options & 1;
        if (cail::launch_oneshot(op, ec, a, P, true, s) != cudaSuccess) rc = -1;
    }
    cail::DevStatus h;
    memset(&h, 0, sizeof(h));
    if (cudaStreamSynchronize(s) != cudaSuccess ||
        cudaMemcpy(&h, emu.st, sizeof(h), cudaMemcpyDeviceToHost) != cudaSuccess)
        rc = -1;
    else if (rc == 0 && h.code != 0)
        rc = h.code;
    cudaStreamDestroy(s);
    cudaGetLastError();
    return rc;
}

// kernel: 0 = one_shot of P emulated ranks (one cooperative launch; the time
// is per call of all P ranks),
// 1 = zero-copy two_shot (reads P inputs, writes P outputs), 2 = fold (P
// sources), 3 = bulk (TMA) copy, 4 = push two_shot of P emulated ranks (one
// cooperative launch; the time is per call of all P ranks), 5 = copy kernel,
// 6 = local reduction io = io + in.  Runs `iters` launches of a float SUM
// over `bytes` bytes per rank (2..8 ranks where it applies) and writes the
// mean time per launch in milliseconds to *ms.  Kernels 3 and 5 check the
// copy afterwards.  Returns 0, -1 on an error, -2 when a copy differs.
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
        if (P < 2) { rc = -1; goto out; }
        std::vector<char *> src(P), dst(P);
        for (int q = 0; q < P; ++q) {
            src[q] = b.get(bytes);
            dst[q] = b.get(bytes);
            if (!src[q] || !dst[q]) { rc = -1; goto out; }
        }
        const int G = cail::push_max_ctas(P, sms);
        size_t piece = (bytes + G - 1) / G;
        piece = (piece + 8191) / 8192 * 8192;
        if (piece > (16 << 10)) piece = 16 << 10;
        const int g = (int)((bytes + piece - 1) / piece < (size_t)G ? (bytes + piece - 1) / piece : (size_t)G);
        Emu emu;
        if (!emu.init(P, G, piece)) { rc = -1; goto out; }
        auto launch = [&]() {
            cail::OneShotArgs a;
            memset(&a, 0, sizeof(a));
            a.bytes = bytes;
            a.piece = piece;
            a.P = P;
            a.G = g;
            a.vec = 1;
            for (int q = 0; q < P; ++q) {
                a.src[q] = src[q];
                a.dst[q] = dst[q];
            }
            emu.args(a, P, 2000000000ull);
            return cail::launch_oneshot(CAIL_SUM, CAIL_EC_F32, a, P, true, s);
        };
        if (launch() != cudaSuccess) { rc = -1; goto out; }
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) launch();
        cudaEventRecord(e1, s);
    } else if (kernel == 3 || kernel == 5) {
        char *src = b.get(bytes + 16), *dst = b.get(bytes + 16);
        int *bst = (int *)b.get(sizeof(int));
        unsigned long long *bad = (unsigned long long *)b.get(sizeof(unsigned long long));
        if (!src || !dst || !bst || !bad || bytes % 16) { rc = -1; goto out; }
        fill_pattern<<<1024, 256, 0, s>>>((uint32_t *)src, bytes / 4);
        auto launch = [&]() {
            return kernel == 3 ? cail::launch_bulk_copy(dst, src, bytes, sms, 2000000000ull, bst, s)
                               : cail::launch_copy(dst, src, bytes, sms, s, bytes > ((size_t)48 << 20));
        };
        if (launch() != cudaSuccess) { rc = -1; goto out; }
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) launch();
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
    } else if (kernel == 4) {
        if (P < 2) { rc = -1; goto out; }
        std::vector<char *> src(P), dst(P);
        for (int q = 0; q < P; ++q) {
            src[q] = b.get(bytes);
            dst[q] = b.get(bytes);
            if (!src[q] || !dst[q]) { rc = -1; goto out; }
        }
        const int G = cail::push_max_ctas(P, sms);
        const size_t piece = 32 << 10;
        Emu emu;
        if (!emu.init(P, G, piece)) { rc = -1; goto out; }
        auto launch = [&]() {
            cail::PushArgs a;
            memset(&a, 0, sizeof(a));
            shape(a, P, count, esz, true, G, piece);
            for (int q = 0; q < P; ++q) {
                a.src[q] = src[q];
                a.dst[q] = dst[q];
            }
            emu.args(a, P, 2000000000ull);
            return cail::launch_push(CAIL_SUM, CAIL_EC_F32, a, P, true, s);
        };
        if (launch() != cudaSuccess) { rc = -1; goto out; }
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) launch();
        cudaEventRecord(e1, s);
    } else if (kernel == 6) {
        char *in = b.get(bytes), *io = b.get(bytes);
        if (!in || !io) { rc = -1; goto out; }
        cail::launch_reduce_local(CAIL_SUM, CAIL_EC_F32, in, io, count, sms, s);
        cudaEventRecord(e0, s);
        for (int i = 0; i < iters; ++i) cail::launch_reduce_local(CAIL_SUM, CAIL_EC_F32, in, io, count, sms, s);
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
    } else if (rc == 0) {
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
