// cail_torch — thin PyTorch extension over the interposed MPI_Allreduce.
//
// Python hands over the address of MPI_Allreduce of the loaded interposer
// (cail-b200's, or the reference's for comparison runs), so the extension
// never resolves MPI symbols itself and cannot bind to the wrong library.
// The call releases the GIL: the data-parallel harness issues it from a
// communication thread while the main thread keeps launching backward.  The
// tensor's device is made current for the call (a CUDA-aware MPI allocates
// and launches on the caller's current device).
#include <c10/core/DeviceGuard.h>
#include <torch/extension.h>

#include <cstdint>

namespace {

typedef int (*allreduce_fn)(const void *, void *, int, int, int, int);
allreduce_fn g_allreduce = nullptr;
intptr_t g_in_place = -1;

void set_allreduce(int64_t fn_addr, int64_t in_place) {
    g_allreduce = reinterpret_cast<allreduce_fn>(static_cast<intptr_t>(fn_addr));
    g_in_place = static_cast<intptr_t>(in_place);
}

int64_t allreduce_inplace(const at::Tensor &t, int64_t datatype, int64_t op, int64_t comm) {
    TORCH_CHECK(g_allreduce != nullptr, "cail_torch: set_allreduce() was not called");
    TORCH_CHECK(t.is_contiguous(), "cail_torch: tensor must be contiguous");
    TORCH_CHECK(t.numel() < (int64_t(1) << 31), "cail_torch: MPI counts are int");
    void *p = t.data_ptr();
    int n = static_cast<int>(t.numel());
    c10::DeviceGuard guard(t.device());
    int rc;
    {
        pybind11::gil_scoped_release nogil;
        rc = g_allreduce(reinterpret_cast<const void *>(g_in_place), p, n, static_cast<int>(datatype),
                         static_cast<int>(op), static_cast<int>(comm));
    }
    return rc;
}

int64_t allreduce(const at::Tensor &src, const at::Tensor &dst, int64_t datatype, int64_t op,
                  int64_t comm) {
    TORCH_CHECK(g_allreduce != nullptr, "cail_torch: set_allreduce() was not called");
    TORCH_CHECK(src.is_contiguous() && dst.is_contiguous() && src.numel() == dst.numel(),
                "cail_torch: contiguous tensors of equal size required");
    const void *s = src.data_ptr();
    void *d = dst.data_ptr();
    int n = static_cast<int>(src.numel());
    c10::DeviceGuard guard(dst.device());
    int rc;
    {
        pybind11::gil_scoped_release nogil;
        rc = g_allreduce(s, d, n, static_cast<int>(datatype), static_cast<int>(op), static_cast<int>(comm));
    }
    return rc;
}

}  // namespace

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
    m.doc() = "GIL-free MPI_Allreduce on tensors through the loaded interposer";
    m.def("set_allreduce", &set_allreduce, "set the MPI_Allreduce entry point and MPI_IN_PLACE");
    m.def("allreduce_inplace", &allreduce_inplace, "MPI_Allreduce(MPI_IN_PLACE, t, ...)");
    m.def("allreduce", &allreduce, "MPI_Allreduce(src, dst, ...)");
}
