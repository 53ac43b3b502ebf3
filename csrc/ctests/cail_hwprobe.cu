// cail_hwprobe — NVLink / NVSwitch transfer rates of this box, measured from
// one process that drives every visible GPU (no MPI).
//
//   cail_hwprobe [ngpus] [p2p|nvls|all]
//
// p2p:  every GPU moves 1 GiB to (push: SM stores into peer memory) or from
//       (pull: SM loads of peer memory) its peers, all GPUs at once, so both
//       directions of every link are busy; then the same with the copy
//       engines (cudaMemcpyPeerAsync).  Prints GB/s per direction per GPU.
// nvls: binds one multicast object over all GPUs and times, with every GPU
//       working on its own 1/P slice: multimem.ld_reduce + multimem.st (the
//       NVLS allreduce core), each of them alone, a local copy, and the
//       copy + multimem mix in one kernel; then the latency of a two-level
//       cross-GPU barrier (local atomic, one multimem.red per GPU, poll).
//
// These are the measurements behind the algorithm choices of the library
// (two-shot's pull/push mix, NVLS kept opt-in, the copy-engine two-shot).
// Every device wait is bounded (2 s) and reported, never fatal.
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#include <algorithm>
#include <string>
#include <vector>

#define CR(x)                                                                                   \
    do {                                                                                        \
        cudaError_t r_ = (x);                                                                   \
        if (r_ != cudaSuccess) {                                                                \
            printf("cuda error %s at %s:%d: %s\n", cudaGetErrorString(r_), __FILE__, __LINE__, #x); \
            exit(1);                                                                            \
        }                                                                                       \
    } while (0)

// ---------------------------------------------------------------- driver API
// Resolved through the runtime so the probe needs no -lcuda.
struct Drv {
    CUresult (*mcGran)(size_t *, const CUmulticastObjectProp *, CUmulticastGranularity_flags);
    CUresult (*mcCreate)(CUmemGenericAllocationHandle *, const CUmulticastObjectProp *);
    CUresult (*mcAdd)(CUmemGenericAllocationHandle, CUdevice);
    CUresult (*mcBind)(CUmemGenericAllocationHandle, size_t, CUmemGenericAllocationHandle, size_t, size_t,
                       unsigned long long);
    CUresult (*memCreate)(CUmemGenericAllocationHandle *, size_t, const CUmemAllocationProp *, unsigned long long);
    CUresult (*reserve)(CUdeviceptr *, size_t, size_t, CUdeviceptr, unsigned long long);
    CUresult (*map)(CUdeviceptr, size_t, size_t, CUmemGenericAllocationHandle, unsigned long long);
    CUresult (*access)(CUdeviceptr, size_t, const CUmemAccessDesc *, size_t);
    CUresult (*devGet)(CUdevice *, int);
};

template <typename F> static bool sym(const char *name, F &f) {
    void *p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || !p) return false;
    f = reinterpret_cast<F>(p);
    return true;
}

static bool load(Drv &d) {
    return sym("cuMulticastGetGranularity", d.mcGran) && sym("cuMulticastCreate", d.mcCreate) &&
           sym("cuMulticastAddDevice", d.mcAdd) && sym("cuMulticastBindMem", d.mcBind) &&
           sym("cuMemCreate", d.memCreate) && sym("cuMemAddressReserve", d.reserve) && sym("cuMemMap", d.map) &&
           sym("cuMemSetAccess", d.access) && sym("cuDeviceGet", d.devGet);
}

__device__ __forceinline__ unsigned long long gtime() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// ---------------------------------------------------------------- kernels
// P2P: npeer chunks of n16 16-byte vectors each; push stores local data into
// the peers, pull loads the peers' data into local memory.  Consecutive
// vectors go to consecutive peers, so every link carries traffic at once.
template <bool PUSH>
__global__ void __launch_bounds__(512) p2p_kernel(const uint4 *const *peer_src, uint4 *const *peer_dst,
                                                  const uint4 *local_src, uint4 *local_dst, int npeer, size_t n16) {
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t nt = (size_t)gridDim.x * blockDim.x;
    const size_t total = n16 * npeer;
    constexpr int U = 4;
    for (size_t i = tid; i < total; i += U * nt) {
        uint4 v[U];
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const size_t w = i + q * nt;
            if (w < total) v[q] = PUSH ? local_src[w] : peer_src[w % npeer][w / npeer];
        }
#pragma unroll
        for (int q = 0; q < U; ++q) {
            const size_t w = i + q * nt;
            if (w < total) {
                if (PUSH) peer_dst[w % npeer][w / npeer] = v[q];
                else local_dst[w] = v[q];
            }
        }
    }
}

// NVLS: mode 0 ld_reduce + st, 1 ld_reduce only (result stored locally),
// 2 st only; units of 16 bytes [lo, hi) of the multicast view.
template <int MODE>
__global__ void __launch_bounds__(512) mm_kernel(char *mc, char *uc, size_t lo, size_t hi) {
    const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
    const size_t nt = (size_t)gridDim.x * blockDim.x;
    for (size_t u = lo + tid; u < hi; u += nt) {
        float4 v = make_float4(1.f, 2.f, 3.f, 4.f);
        if (MODE != 2)
            asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                         : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                         : "l"(mc + u * 16)
                         : "memory");
        if (MODE == 1)
            *reinterpret_cast<float4 *>(uc + u * 16) = v;
        else
            asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + u * 16), "f"(v.x),
                         "f"(v.y), "f"(v.z), "f"(v.w)
                         : "memory");
    }
}

// CTAs [0, C) copy n bytes locally, the others run ld_reduce + st on [lo, hi).
__global__ void __launch_bounds__(512) mixed_kernel(char *mc, const char *src, char *dst, size_t n, size_t lo,
                                                    size_t hi, int C) {
    if ((int)blockIdx.x < C) {
        const size_t tid = (size_t)blockIdx.x * blockDim.x + threadIdx.x;
        const size_t nt = (size_t)C * blockDim.x;
        for (size_t i = tid; i < n / 16; i += nt)
            reinterpret_cast<uint4 *>(dst)[i] = reinterpret_cast<const uint4 *>(src)[i];
        return;
    }
    const size_t tid = (size_t)(blockIdx.x - C) * blockDim.x + threadIdx.x;
    const size_t nt = (size_t)(gridDim.x - C) * blockDim.x;
    for (size_t u = lo + tid; u < hi; u += nt) {
        float4 v;
        asm volatile("multimem.ld_reduce.relaxed.sys.global.add.v4.f32 {%0,%1,%2,%3}, [%4];"
                     : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                     : "l"(mc + u * 16)
                     : "memory");
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(mc + u * 16), "f"(v.x),
                     "f"(v.y), "f"(v.z), "f"(v.w)
                     : "memory");
    }
}

// K rounds of the two-level barrier; out[0] = ns per round (block 0),
// out[1] = 1 if a wait ran out.
__global__ void barrier_kernel(uint32_t *mc_counter, const uint32_t *uc_counter, uint32_t *local, int P, int K,
                               unsigned long long *out) {
    const unsigned long long t0 = gtime();
    for (int k = 0; k < K; ++k) {
        __syncthreads();
        if (threadIdx.x == 0) {
            __threadfence();
            if (atomicAdd(local, 1u) + 1u == (uint32_t)(k + 1) * gridDim.x) {
                __threadfence();
                asm volatile("fence.proxy.alias;" ::: "memory");
                asm volatile("multimem.red.release.sys.global.add.u32 [%0], %1;" ::"l"(mc_counter), "r"(1u)
                             : "memory");
            }
            const uint32_t target = (uint32_t)(k + 1) * P;
            const unsigned long long deadline = gtime() + 2000000000ull;
            uint32_t v;
            do {
                asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(uc_counter) : "memory");
                if (gtime() > deadline) {
                    out[1] = 1;
                    break;
                }
            } while ((int32_t)(v - target) < 0);
        }
        __syncthreads();
    }
    if (blockIdx.x == 0 && threadIdx.x == 0) out[0] = (gtime() - t0) / (unsigned long long)K;
}

// ---------------------------------------------------------------- timing
// Runs launch(d, stream) on every GPU at once, `reps` times after 2 warm-up
// rounds; returns the mean over rounds of the slowest GPU's event time (s).
template <typename F>
static double time_all(int n, std::vector<cudaStream_t> &st, int reps, F launch) {
    std::vector<cudaEvent_t> e0(n), e1(n);
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        CR(cudaEventCreate(&e0[d]));
        CR(cudaEventCreate(&e1[d]));
    }
    double acc = 0;
    for (int rep = 0; rep < reps + 2; ++rep) {
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            CR(cudaDeviceSynchronize());
        }
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            CR(cudaEventRecord(e0[d], st[d]));
            launch(d, st[d]);
            CR(cudaGetLastError());
            CR(cudaEventRecord(e1[d], st[d]));
        }
        float worst = 0;
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            CR(cudaEventSynchronize(e1[d]));
            float ms;
            CR(cudaEventElapsedTime(&ms, e0[d], e1[d]));
            worst = std::max(worst, ms);
        }
        if (rep >= 2) acc += worst * 1e-3;
    }
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        CR(cudaEventDestroy(e0[d]));
        CR(cudaEventDestroy(e1[d]));
    }
    return acc / reps;
}

static void probe_p2p(int n, int sms) {
    const size_t B = (size_t)1 << 30;
    std::vector<char *> a(n), b(n);
    std::vector<cudaStream_t> st(n);
    std::vector<const uint4 **> ps(n);
    std::vector<uint4 **> pd(n);
    const size_t per = B / (n - 1) / 16 * 16;
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        for (int e = 0; e < n; ++e)
            if (e != d) {
                cudaError_t r = cudaDeviceEnablePeerAccess(e, 0);
                if (r != cudaSuccess && r != cudaErrorPeerAccessAlreadyEnabled) CR(r);
                cudaGetLastError();
            }
        CR(cudaMalloc(&a[d], B));
        CR(cudaMalloc(&b[d], B));
        CR(cudaMemset(a[d], 1, B));
        CR(cudaStreamCreateWithFlags(&st[d], cudaStreamNonBlocking));
    }
    for (int d = 0; d < n; ++d) {
        std::vector<const uint4 *> hs;
        std::vector<uint4 *> hd;
        for (int k = 1; k < n; ++k) {  // peers in the order d+1, d+2, ...: no common first target
            const int e = (d + k) % n;
            const int slot = d < e ? d : d - 1;  // d's chunk inside peer e's buffer
            hs.push_back((const uint4 *)(a[e] + (size_t)slot * per));
            hd.push_back((uint4 *)(b[e] + (size_t)slot * per));
        }
        CR(cudaSetDevice(d));
        CR(cudaMalloc(&ps[d], sizeof(void *) * hs.size()));
        CR(cudaMalloc(&pd[d], sizeof(void *) * hd.size()));
        CR(cudaMemcpy(ps[d], hs.data(), sizeof(void *) * hs.size(), cudaMemcpyHostToDevice));
        CR(cudaMemcpy(pd[d], hd.data(), sizeof(void *) * hd.size(), cudaMemcpyHostToDevice));
    }
    const double moved = (double)per * (n - 1);
    printf("# p2p: %d GPUs, %.0f MiB per GPU and direction, all GPUs at once\n", n, moved / (1 << 20));
    for (int grid : {sms, 2 * sms, 4 * sms}) {
        double tpull = time_all(n, st, 5, [&](int d, cudaStream_t s) {
            p2p_kernel<false><<<grid, 512, 0, s>>>(ps[d], pd[d], (const uint4 *)a[d], (uint4 *)b[d], n - 1, per / 16);
        });
        double tpush = time_all(n, st, 5, [&](int d, cudaStream_t s) {
            p2p_kernel<true><<<grid, 512, 0, s>>>(ps[d], pd[d], (const uint4 *)a[d], (uint4 *)b[d], n - 1, per / 16);
        });
        printf("p2p sm_pull grid=%d %.1f GB/s   sm_push grid=%d %.1f GB/s\n", grid, moved / tpull / 1e9, grid,
               moved / tpush / 1e9);
    }
    double tce = time_all(n, st, 5, [&](int d, cudaStream_t s) {
        for (int k = 1; k < n; ++k) {
            const int e = (d + k) % n;
            const int slot = d < e ? d : d - 1;
            CR(cudaMemcpyPeerAsync(b[e] + (size_t)slot * per, e, a[d] + (size_t)(k - 1) * per, d, per, s));
        }
    });
    printf("p2p copy_engine_push %.1f GB/s\n", moved / tce / 1e9);
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        CR(cudaFree(a[d]));
        CR(cudaFree(b[d]));
        CR(cudaFree(ps[d]));
        CR(cudaFree(pd[d]));
        CR(cudaStreamDestroy(st[d]));
    }
}

static void probe_nvls(int n, int sms) {
    Drv drv;
    if (!load(drv)) {
        printf("nvls: driver entry points unavailable\n");
        return;
    }
    CUmulticastObjectProp mp;
    memset(&mp, 0, sizeof(mp));
    mp.numDevices = (unsigned)n;
    mp.handleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
    size_t gran = 0;
    if (drv.mcGran(&gran, &mp, CU_MULTICAST_GRANULARITY_RECOMMENDED) != CUDA_SUCCESS) {
        printf("nvls: multicast unsupported\n");
        return;
    }
    const size_t region = ((size_t)1 << 30) + (2 << 20);
    const size_t size = (region + gran - 1) / gran * gran;
    mp.size = size;
    CUmemGenericAllocationHandle mch;
    if (drv.mcCreate(&mch, &mp) != CUDA_SUCCESS) {
        printf("nvls: cuMulticastCreate failed for %d GPUs\n", n);
        return;
    }
    std::vector<char *> uc(n), mc(n);
    std::vector<cudaStream_t> st(n);
    for (int d = 0; d < n; ++d) {
        CUdevice cd;
        CR(cudaSetDevice(d));
        CR(cudaFree(0));
        if (drv.devGet(&cd, d) != CUDA_SUCCESS || drv.mcAdd(mch, cd) != CUDA_SUCCESS) {
            printf("nvls: cuMulticastAddDevice failed\n");
            return;
        }
    }
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        CUmemAllocationProp ap;
        memset(&ap, 0, sizeof(ap));
        ap.type = CU_MEM_ALLOCATION_TYPE_PINNED;
        ap.location.type = CU_MEM_LOCATION_TYPE_DEVICE;
        ap.location.id = d;
        ap.requestedHandleTypes = CU_MEM_HANDLE_TYPE_POSIX_FILE_DESCRIPTOR;
        CUmemAccessDesc acc;
        memset(&acc, 0, sizeof(acc));
        acc.location = ap.location;
        acc.flags = CU_MEM_ACCESS_FLAGS_PROT_READWRITE;
        CUmemGenericAllocationHandle ph;
        CUdeviceptr u, m;
        if (drv.memCreate(&ph, size, &ap, 0) != CUDA_SUCCESS || drv.reserve(&u, size, gran, 0, 0) != CUDA_SUCCESS ||
            drv.map(u, size, 0, ph, 0) != CUDA_SUCCESS || drv.access(u, size, &acc, 1) != CUDA_SUCCESS ||
            drv.mcBind(mch, 0, ph, 0, size, 0) != CUDA_SUCCESS || drv.reserve(&m, size, gran, 0, 0) != CUDA_SUCCESS ||
            drv.map(m, size, 0, mch, 0) != CUDA_SUCCESS || drv.access(m, size, &acc, 1) != CUDA_SUCCESS) {
            printf("nvls: binding the multicast region failed on GPU %d\n", d);
            return;
        }
        uc[d] = (char *)u;
        mc[d] = (char *)m;
        CR(cudaMemset(uc[d], 0, size));
        CR(cudaStreamCreateWithFlags(&st[d], cudaStreamNonBlocking));
    }
    const size_t data0 = 2 << 20, M = (size_t)512 << 20, units = M / 16;
    printf("# nvls: %d GPUs, message %zu MiB, every GPU on its 1/%d slice\n", n, M >> 20, n);
    const char *names[3] = {"ld_reduce+st", "ld_reduce", "st"};
    for (int mode = 0; mode < 3; ++mode) {
        double t = time_all(n, st, 5, [&](int d, cudaStream_t s) {
            const size_t lo = units * d / n, hi = units * (d + 1) / n;
            if (mode == 0) mm_kernel<0><<<2 * sms, 512, 0, s>>>(mc[d] + data0, uc[d] + data0, lo, hi);
            if (mode == 1) mm_kernel<1><<<2 * sms, 512, 0, s>>>(mc[d] + data0, uc[d] + data0, lo, hi);
            if (mode == 2) mm_kernel<2><<<2 * sms, 512, 0, s>>>(mc[d] + data0, uc[d] + data0, lo, hi);
        });
        // bytes per GPU and direction: ld_reduce sends the whole local copy
        // and receives 1/P, st sends 1/P and receives the whole message
        const double per_dir = mode == 0 ? M * (1.0 + 1.0 / n) : M;
        printf("nvls %-13s %8.1f us  %7.1f GB/s per direction  allreduce-equivalent busbw %7.1f GB/s\n", names[mode],
               t * 1e6, per_dir / t / 1e9, mode == 0 ? 2.0 * (n - 1) / n * M / t / 1e9 : 0.0);
    }
    // copy + multimem interference: message M/2 of ld_reduce + st and M of local copy
    std::vector<char *> ca(n), cb(n);
    for (int d = 0; d < n; ++d) {
        CR(cudaSetDevice(d));
        CR(cudaMalloc(&ca[d], M));
        CR(cudaMalloc(&cb[d], M));
        CR(cudaMemset(ca[d], 0, M));
    }
    const size_t hu = units / 2;
    double t_mm = time_all(n, st, 5, [&](int d, cudaStream_t s) {
        mixed_kernel<<<2 * sms, 512, 0, s>>>(mc[d] + data0, ca[d], cb[d], 0, hu * d / n, hu * (d + 1) / n, sms);
    });
    double t_cp = time_all(n, st, 5, [&](int d, cudaStream_t s) {
        mixed_kernel<<<2 * sms, 512, 0, s>>>(mc[d] + data0, ca[d], cb[d], M, 0, 0, sms);
    });
    double t_mix = time_all(n, st, 5, [&](int d, cudaStream_t s) {
        mixed_kernel<<<2 * sms, 512, 0, s>>>(mc[d] + data0, ca[d], cb[d], M, hu * d / n, hu * (d + 1) / n, sms);
    });
    printf("nvls overlap: ld_reduce+st alone %.1f us, copy alone %.1f us, both in one kernel %.1f us\n", t_mm * 1e6,
           t_cp * 1e6, t_mix * 1e6);
    for (int grid : {1, sms, 2 * sms}) {
        std::vector<unsigned long long *> out(n);
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            CR(cudaMemset(uc[d], 0, 4096));
            CR(cudaDeviceSynchronize());
            CR(cudaMallocHost(&out[d], 16));
            out[d][0] = out[d][1] = 0;
        }
        const int K = 200;
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            barrier_kernel<<<grid, 512, 0, st[d]>>>((uint32_t *)mc[d], (const uint32_t *)uc[d],
                                                    (uint32_t *)(uc[d] + 256), n, K, out[d]);
        }
        unsigned long long worst = 0;
        int fail = 0;
        for (int d = 0; d < n; ++d) {
            CR(cudaSetDevice(d));
            CR(cudaStreamSynchronize(st[d]));
            worst = std::max(worst, out[d][0]);
            fail |= (int)out[d][1];
            CR(cudaFreeHost(out[d]));
        }
        printf("nvls barrier grid=%d %.2f us per round%s\n", grid, worst / 1e3, fail ? " (a wait ran out)" : "");
    }
}

int main(int argc, char **argv) {
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) n = 0;
    if (argc > 1) n = std::min(n, atoi(argv[1]));
    const std::string what = argc > 2 ? argv[2] : "all";
    if (n < 2) {
        printf("cail_hwprobe needs at least 2 GPUs (found %d)\n", n);
        return 0;
    }
    cudaDeviceProp prop;
    CR(cudaGetDeviceProperties(&prop, 0));
    printf("# cail_hwprobe: %d x %s, %d SMs\n", n, prop.name, prop.multiProcessorCount);
    if (what == "p2p" || what == "all") probe_p2p(n, prop.multiProcessorCount);
    if (what == "nvls" || what == "all") probe_nvls(n, prop.multiProcessorCount);
    return 0;
}
