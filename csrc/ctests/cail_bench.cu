// cail_bench — MPI_Allreduce latency / bus-bandwidth sweep on device buffers.
//
// Counterpart of the reference's tests/bench_allreduce_gpu.cu, with the
// statistics this repository reports: every call is timed on the host
// (MPI_Allreduce is blocking), p50 / p99 / mean per size, each the max over
// ranks; busbw = 2 (P-1)/P * bytes / mean.
//
//   cail-mpirun -np N -x LD_PRELOAD=build/lib/libcail.so cail_bench \
//       [-b min_bytes] [-e max_bytes] [-i iters] [-w warmup] [-d double] [--inplace]
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

int main(int argc, char **argv) {
    size_t minb = 32 << 10, maxb = 1 << 30;
    int iters = 100, warm = 20;
    bool dbl = false, inplace = false;
    for (int i = 1; i < argc; ++i) {
        std::string a = argv[i];
        if (a == "-b" && i + 1 < argc) minb = strtoull(argv[++i], nullptr, 10);
        else if (a == "-e" && i + 1 < argc) maxb = strtoull(argv[++i], nullptr, 10);
        else if (a == "-i" && i + 1 < argc) iters = atoi(argv[++i]);
        else if (a == "-w" && i + 1 < argc) warm = atoi(argv[++i]);
        else if (a == "-d") dbl = true;
        else if (a == "--inplace") inplace = true;
    }
    MPI_Init(&argc, &argv);
    int rank, P;
    MPI_Comm_rank(MPI_COMM_WORLD, &rank);
    MPI_Comm_size(MPI_COMM_WORLD, &P);
    int ndev = 0;
    cudaGetDeviceCount(&ndev);
    const char *lr = getenv("CMPI_LOCAL_RANK");
    cudaSetDevice((lr ? atoi(lr) : rank) % (ndev ? ndev : 1));
    typedef const char *(*algo_fn)(void);
    algo_fn last = (algo_fn)dlsym(RTLD_DEFAULT, "cail_last_algorithm");
    float *s = nullptr, *r = nullptr;
    cudaMalloc(&s, maxb);
    cudaMalloc(&r, maxb);
    fill<<<1024, 256>>>(s, maxb / 4, (float)rank);
    fill<<<1024, 256>>>(r, maxb / 4, (float)rank);
    cudaDeviceSynchronize();
    MPI_Datatype dt = dbl ? MPI_DOUBLE : MPI_FLOAT;
    int esz = dbl ? 8 : 4;
    if (rank == 0) printf("# cail_bench np=%d iters=%d warmup=%d %s %s\nbytes,algo,p50_us,p99_us,mean_us,busbw_gbps\n",
                          P, iters, warm, dbl ? "MPI_DOUBLE" : "MPI_FLOAT", inplace ? "in_place" : "separate");
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
    cudaFree(s);
    cudaFree(r);
    MPI_Finalize();
    return 0;
}
