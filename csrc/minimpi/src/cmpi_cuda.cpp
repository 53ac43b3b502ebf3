// cmpi_cuda.cpp — the CUDA-aware part of minimpi.
//
// Point-to-point messages whose send buffer is device memory use a CUDA-IPC
// rendezvous: the sender exports its allocation (cached per allocation,
// keyed by CU_POINTER_ATTRIBUTE_BUFFER_ID, which the driver never reuses
// within a process), the receiver opens it once (cached per sender and
// allocation) and copies straight out of it with a copy-engine memcpy on a
// private stream.  This is the intra-node path of production CUDA-aware MPIs
// (UCX cuda_ipc and similar).
//
// Everything degrades to "host memory only" when no CUDA driver or device is
// present (the CPU development machine), or when CMPI_NO_CUDA=1.
#include "cmpi_internal.h"

#include <cuda.h>
#include <cuda_runtime.h>

#include <cstdlib>
#include <list>
#include <unordered_map>

namespace cmpi {

namespace {

int g_state = -1;  // -1 unknown, 0 unavailable, 1 available

typedef CUresult (*PFN_getattr)(void *, CUpointer_attribute, CUdeviceptr);
typedef CUresult (*PFN_range)(CUdeviceptr *, size_t *, CUdeviceptr);
PFN_getattr p_getattr = nullptr;
PFN_range p_range = nullptr;

struct Export {
    cudaIpcMemHandle_t handle;
    uintptr_t base;
    bool ok;
};
std::unordered_map<uint64_t, Export> g_exports;  // buffer_id -> handle

struct ImportKey {
    int src;
    uint64_t id;
    int dev;
    bool operator==(const ImportKey &o) const { return src == o.src && id == o.id && dev == o.dev; }
};
struct ImportKeyHash {
    size_t operator()(const ImportKey &k) const {
        return std::hash<uint64_t>()(k.id * 1315423911u + (uint64_t)k.src * 64 + (uint64_t)k.dev);
    }
};
struct Import {
    void *base;
    std::list<ImportKey>::iterator lru;
};
std::unordered_map<ImportKey, Import, ImportKeyHash> g_imports;
std::list<ImportKey> g_lru;
constexpr size_t kMaxImports = 512;

void load_driver_entry_points() {
    cudaDriverEntryPointQueryResult q;
    void *fn = nullptr;
    if (cudaGetDriverEntryPoint("cuPointerGetAttribute", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        p_getattr = (PFN_getattr)fn;
    fn = nullptr;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
        p_range = (PFN_range)fn;
}

// Copies run on the legacy default stream: they are then ordered after all
// earlier legacy-stream work of the process, including the DMA of a
// cudaMemcpy from pageable memory, which may still be in flight when that
// call returns.  A private non-blocking stream could read stale data.
cudaStream_t stream_for(int dev) {
    (void)dev;
    return cudaStreamLegacy;
}

// Runs f with device `dev` current and restores the caller's device.
template <typename F>
int with_device(int dev, F f) {
    int prev = -1;
    cudaGetDevice(&prev);
    if (dev >= 0 && dev != prev) cudaSetDevice(dev);
    int rc = f(dev >= 0 ? dev : prev);
    if (dev >= 0 && prev >= 0 && dev != prev) cudaSetDevice(prev);
    return rc;
}

}  // namespace

bool cuda_available() {
    if (g_state >= 0) return g_state == 1;
    const char *off = getenv("CMPI_NO_CUDA");
    if (off && *off && *off != '0') { g_state = 0; return false; }
    int n = 0;
    if (cudaGetDeviceCount(&n) == cudaSuccess && n > 0) {
        g_state = 1;
        load_driver_entry_points();
    } else {
        cudaGetLastError();
        g_state = 0;
    }
    return g_state == 1;
}

bool is_device_ptr(const void *p, int *ordinal) {
    if (!p || p == MPI_IN_PLACE || !cuda_available()) return false;
    cudaPointerAttributes a;
    if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
        cudaGetLastError();
        return false;
    }
    if (a.type == cudaMemoryTypeDevice || a.type == cudaMemoryTypeManaged) {
        if (ordinal) *ordinal = a.device;
        return true;
    }
    return false;
}

int cuda_copy(void *dst, const void *src, uint64_t bytes, int ordinal_hint) {
    if (bytes == 0) return MPI_SUCCESS;
    return with_device(ordinal_hint, [&](int dev) {
        cudaStream_t s = stream_for(dev);
        cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDefault, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            CMPI_ERR("cudaMemcpy of %llu bytes failed: %s", (unsigned long long)bytes,
                     cudaGetErrorString(e));
            return MPI_ERR_OTHER;
        }
        return MPI_SUCCESS;
    });
}

bool ipc_describe(const void *p, uint64_t bytes, int ordinal, RndvDesc *d) {
    if (!p_getattr || !p_range) return false;
    if (const char *e = getenv("CMPI_NO_IPC"); e && *e && *e != '0') return false;
    // The receiver copies out of this buffer from its own process, outside
    // this process' stream order: let queued legacy-stream work that may
    // still write the buffer (e.g. the DMA of a pageable cudaMemcpy) finish.
    with_device(ordinal, [](int) { return cudaStreamSynchronize(cudaStreamLegacy) == cudaSuccess ? 0 : 1; });
    unsigned long long id = 0;
    if (p_getattr(&id, CU_POINTER_ATTRIBUTE_BUFFER_ID, (CUdeviceptr)p) != CUDA_SUCCESS) return false;
    auto it = g_exports.find(id);
    if (it == g_exports.end()) {
        Export ex{};
        CUdeviceptr base = 0;
        size_t size = 0;
        ex.ok = p_range(&base, &size, (CUdeviceptr)p) == CUDA_SUCCESS;
        if (ex.ok) {
            ex.base = (uintptr_t)base;
            int rc = with_device(ordinal, [&](int) {
                return cudaIpcGetMemHandle(&ex.handle, (void *)base) == cudaSuccess ? 0 : 1;
            });
            if (rc != 0) { cudaGetLastError(); ex.ok = false; }
        }
        it = g_exports.emplace(id, ex).first;
    }
    if (!it->second.ok) return false;
    memcpy(d->handle, &it->second.handle, sizeof(d->handle));
    d->buffer_id = id;
    d->offset = (uint64_t)((uintptr_t)p - it->second.base);
    d->bytes = bytes;
    d->device = ordinal;
    return true;
}

int ipc_pull(int src, const RndvDesc &d, void *dst, bool dst_dev, int dst_ordinal) {
    return with_device(dst_dev ? dst_ordinal : -1, [&](int dev) {
        ImportKey key{src, d.buffer_id, dev};
        auto it = g_imports.find(key);
        void *base = nullptr;
        if (it != g_imports.end()) {
            base = it->second.base;
            g_lru.splice(g_lru.begin(), g_lru, it->second.lru);
        } else {
            cudaIpcMemHandle_t h;
            memcpy(&h, d.handle, sizeof(h));
            cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
            if (e == cudaErrorAlreadyMapped) {
                // The sender freed an allocation we still map and reused its
                // memory; drop our mappings of that sender and retry.
                cudaGetLastError();
                for (auto it = g_imports.begin(); it != g_imports.end();) {
                    if (it->first.src == src) {
                        cudaIpcCloseMemHandle(it->second.base);
                        g_lru.erase(it->second.lru);
                        it = g_imports.erase(it);
                    } else {
                        ++it;
                    }
                }
                e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
            }
            if (e != cudaSuccess) {
                CMPI_ERR("cudaIpcOpenMemHandle from rank %d failed: %s", src, cudaGetErrorString(e));
                return MPI_ERR_OTHER;
            }
            if (g_imports.size() >= kMaxImports) {
                ImportKey old = g_lru.back();
                g_lru.pop_back();
                auto o = g_imports.find(old);
                if (o != g_imports.end()) {
                    cudaIpcCloseMemHandle(o->second.base);
                    g_imports.erase(o);
                }
            }
            g_lru.push_front(key);
            g_imports[key] = Import{base, g_lru.begin()};
        }
        cudaStream_t s = stream_for(dev);
        cudaError_t e = cudaMemcpyAsync(dst, (const char *)base + d.offset, d.bytes,
                                        cudaMemcpyDefault, s);
        if (e == cudaSuccess) e = cudaStreamSynchronize(s);
        if (e != cudaSuccess) {
            CMPI_ERR("IPC copy of %llu bytes from rank %d failed: %s", (unsigned long long)d.bytes,
                     src, cudaGetErrorString(e));
            return MPI_ERR_OTHER;
        }
        return MPI_SUCCESS;
    });
}

void cuda_finalize() {
    if (g_state != 1) return;
    for (auto &kv : g_imports) cudaIpcCloseMemHandle(kv.second.base);
    g_imports.clear();
    g_lru.clear();
    g_exports.clear();
}

}  // namespace cmpi
