// cail_bench — MPI_Allreduce latency / bus-bandwidth sweep on device buffers.
//
// Counterpart of the reference's tests/bench_allreduce_gpu.cu, with the
// statistics this repository reports: every call is timed on the host
// (MPI_Allreduce is blocking), p50 / p99 / mean per size, each the max over
// ranks; busbw = 2 (P-1)/P * bytes / mean.
//
//   cail-mpirun -np N -x LD_PRELOAD=build/lib/libcail.so cail_bench \
//       [-b min_bytes] [-e max_bytes] [-i iters] [-w warmup] [-d double] [--inplace]
//   cail_bench --host [-b] [-e] [-i] [-w]   the same sweep on malloc'd host
//       buffers (host-only build, CPU ranks; also runs without a GPU)
//   cail_bench --stress [-i calls]    latency / stress workload: MPI_DOUBLE SUM,
//       `calls` (default 10000) back-to-back calls at 32, 64, 128 and 256 KiB
//       rotating over 64 distinct allocations with MPI_IN_PLACE on every other
//       call, then a 1 GiB call; p50 / p99 per size and the 1 GiB bus bandwidth
//       as a fraction of the NVLink bound (2(P-1)/P * N bytes per GPU and
//       direction at 900 GB/s nominal, 770 GB/s measured peer copy).
#include <cuda_runtime.h>
#include <dlfcn.h>
#include <mpi.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>

#include <algorithm>
#include <string>
#include <vector>

static double now_us() {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return ts.tv_sec * 1e6 + ts.tv_nsec * 1e-3;
}

__global__ void fill(float *p, size_t n, float v) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        p[i] = v + (float)(i % 1024) * 1e-3f;
}

__global__ void fill_uniform(double *p, size_t n, unsigned seed) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        unsigned long long x = (i + 1) * 0x9E3779B97F4A7C15ull ^ ((unsigned long long)seed << 32);
        x ^= x >> 31; x *= 0xBF58476D1CE4E5B9ull; x ^= x >> 29;
        p[i] = (double)(x >> 11) * (1.0 / 9007199254740992.0) * 2.0 - 1.0;  // uniform [-1, 1)
    }
}

typedef const char *(*algo_fn)(void);

static void max_over_ranks(double *loc, int n, double *mx) { PMPI_Allreduce(loc, mx, n, MPI_DOUBLE, MPI_MAX, MPI_COMM_WORLD); }

static int run_stress(int rank, int P, int calls, algo_fn last) {
    const int nbuf = 64;
    const size_t maxsmall = 256 << 10;
    std::vector<double *> sb(nbuf), rb(nbuf);
    for (int i = 0; i < nbuf; ++i) {
        if (cudaMalloc(&sb[i], maxsmall) != cudaSuccess || cudaMalloc(&rb[i], maxsmall) != cudaSuccess) return 1;
        fill_uniform<<<64, 256>>>(sb[i], maxsmall / 8, 1000u * rank + i);
        fill_uniform<<<64, 256>>>(rb[i], maxsmall / 8, 7000u * rank + i);
    }
    cudaDeviceSynchronize();
    if (rank == 0) printf("# cail_bench --stress np=%d calls=%d MPI_DOUBLE SUM, %d buffers, MPI_IN_PLACE on odd calls\n"
                          "kind,bytes,algo,p50_us,p99_us,mean_us\n", P, calls, nbuf);
    std::vector<double> t(calls);
    for (size_t b = 32 << 10; b <= maxsmall; b *= 2) {
        const int n = (int)(b / 8);
        for (int k = 0; k < 100; ++k) MPI_Allreduce(sb[k % nbuf], rb[k % nbuf], n, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        MPI_Barrier(MPI_COMM_WORLD);
        for (int k = 0; k < calls; ++k) {
            const int i = k % nbuf;
            const double t0 = now_us();
            if (k & 1) MPI_Allreduce(MPI_IN_PLACE, rb[i], n, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
            else MPI_Allreduce(sb[i], rb[i], n, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
            t[k] = now_us() - t0;
        }
        std::vector<double> v(t);
        std::sort(v.begin(), v.end());
        double loc[3] = {v[calls / 2], v[std::min(calls - 1, (int)(0.99 * calls))], 0}, mx[3];
        for (double x : v) loc[2] += x / calls;
        max_over_ranks(loc, 3, mx);
        if (rank == 0) printf("small,%zu,%s,%.2f,%.2f,%.2f\n", b, last ? last() : "n/a", mx[0], mx[1], mx[2]);
        fflush(stdout);
    }
    for (int i = 0; i < nbuf; ++i) { cudaFree(sb[i]); cudaFree(rb[i]); }
    const size_t big = (size_t)1 << 30;
    double *s = nullptr, *r = nullptr;
    if (cudaMalloc(&s, big) != cudaSuccess || cudaMalloc(&r, big) != cudaSuccess) return 1;
    fill_uniform<<<1024, 256>>>(s, big / 8, 5000u + rank);
    cudaDeviceSynchronize();
    const int n = (int)(big / 8), reps = 10;
    for (int k = 0; k < 3; ++k) MPI_Allreduce(s, r, n, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
    MPI_Barrier(MPI_COMM_WORLD);
    std::vector<double> tb(reps);
    for (int k = 0; k < reps; ++k) {
        const double t0 = now_us();
        MPI_Allreduce(s, r, n, MPI_DOUBLE, MPI_SUM, MPI_COMM_WORLD);
        tb[k] = now_us() - t0;
    }
    std::sort(tb.begin(), tb.end());
    double loc[2] = {tb[reps / 2], 0}, mx[2];
    for (double x : tb) loc[1] += x / reps;
    max_over_ranks(loc, 2, mx);
    const double bus = (double)big / (mx[1] * 1e-6) / 1e9 * (P > 1 ? 2.0 * (P - 1) / P : 1.0);
    if (rank == 0) {
        printf("kind,bytes,algo,p50_us,mean_us,busbw_gbps,frac_of_900,frac_of_770\n");
        printf("big,%zu,%s,%.2f,%.2f,%.2f,%.3f,%.3f\n", big, last ? last() : "n/a", mx[0], mx[1], bus, bus / 900.0,
               bus / 770.0);
    }
    cudaFree(s);
    cudaFree(r);
    return 0;
}

int main(int argc, char **argv) {
    size_t minb = 32 << 10, maxb = 1 << 30;
    int iters = 100, warm = 20;
    bool dbl = false, inplace = false, stress = false, host = false;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "-b" && i + 1 < argc) minb = strtoull(argv[++i], nullptr, 10);
        else if (a == "-e" && i + 1 < argc) maxb = strtoull(argv[++i], nullptr, 10);
        else if (a == "-i" && i + 1 < argc) iters = atoi(argv[++i]);
        else if (a == "-w" && i + 1 < argc) warm = atoi(argv[++i]);
        else if (a == "-d") dbl = true;
        else if (a == "--inplace") inplace = true;
        else if (a == "--stress") stress = true;
        else if (a == "--host") host = true;
    }
    MPI_Init(&argc, &argv);
    int rank, P;
    MPI_Comm_rank(MPI_COMM_WORLD, &rank);
    MPI_Comm_size(MPI_COMM_WORLD, &P);
    int ndev = 0;
    if (!host) {
        cudaGetDeviceCount(&ndev);
        const char *lr = getenv("CMPI_LOCAL_RANK");
        cudaSetDevice((lr ? atoi(lr) : rank) % (ndev ? ndev : 1));
    }
    algo_fn last = (algo_fn)dlsym(RTLD_DEFAULT, "cail_last_algorithm");
    if (stress) {
        int rc = run_stress(rank, P, iters == 100 ? 10000 : iters, last);
        MPI_Finalize();
        return rc;
    }
    float *s = nullptr, *r = nullptr;
    if (host) {
        s = (float *)malloc(maxb);
        r = (float *)malloc(maxb);
        if (!s || !r) { MPI_Abort(MPI_COMM_WORLD, 1); }
        for (size_t i = 0; i < maxb / 4; ++i) s[i] = r[i] = (float)rank + (float)(i % 1024) * 1e-3f;
    } else {
        cudaMalloc(&s, maxb);
        cudaMalloc(&r, maxb);
        fill<<<1024, 256>>>(s, maxb / 4, (float)rank);
        fill<<<1024, 256>>>(r, maxb / 4, (float)rank);
        cudaDeviceSynchronize();
    }
    MPI_Datatype dt = dbl ? MPI_DOUBLE : MPI_FLOAT;
    int esz = dbl ? 8 : 4;
    if (rank == 0) printf("# cail_bench np=%d iters=%d warmup=%d %s %s %s\nbytes,algo,p50_us,p99_us,mean_us,busbw_gbps\n",
                          P, iters, warm, dbl ? "MPI_DOUBLE" : "MPI_FLOAT", inplace ? "in_place" : "separate",
                          host ? "host" : "device");
    std::vector<double> t(iters);
    for (size_t b = minb; b <= maxb; b *= 2) {
        int n = (int)(b / esz);
        int it = b > (128u << 20) ? std::max(10, iters / 5) : iters;
        for (int w = 0; w < warm; ++w)
            MPI_Allreduce(inplace ? MPI_IN_PLACE : s, r, n, dt, MPI_SUM, MPI_COMM_WORLD);
        MPI_Barrier(MPI_COMM_WORLD);
        for (int k = 0; k < it; ++k) {
            double t0 = now_us();
            MPI_Allreduce(inplace ? MPI_IN_PLACE : s, r, n, dt, MPI_SUM, MPI_COMM_WORLD);
            t[k] = now_us() - t0;
        }
        std::vector<double> v(t.begin(), t.begin() + it);
        std::sort(v.begin(), v.end());
        double loc[3] = {v[it / 2], v[std::min(it - 1, (int)(0.99 * it))], 0};
        for (double x : v) loc[2] += x / it;
        double mx[3];
        PMPI_Allreduce(loc, mx, 3, MPI_DOUBLE, MPI_MAX, MPI_COMM_WORLD);
        double bus = (double)b / (mx[2] * 1e-6) / 1e9 * (P > 1 ? 2.0 * (P - 1) / P : 1.0);
        if (rank == 0)
            printf("%zu,%s,%.2f,%.2f,%.2f,%.2f\n", b, last ? last() : "n/a", mx[0], mx[1], mx[2], bus);
        fflush(stdout);
    }
    if (host) {
        free(s);
        free(r);
    } else {
        cudaFree(s);
        cudaFree(r);
    }
    MPI_Finalize();
    return 0;
}
