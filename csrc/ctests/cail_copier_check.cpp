// cail_copier_check — CPU check of the NVLS kernel's copier loop.
//
// The copier warps of the NVLS kernel copy unit j out of a staging slot and
// then, with no barrier in between, copy unit j + 2 into the same slot.  That
// is correct only if each slot byte is read by the copy-out and written by
// the copy-in from the same thread.  This program compiles the loop
// (cail_dev_copier.cuh) as host code and runs its kNvlsCopiers threads one
// after another, each doing its copy-out and then its copy-in, in several
// orders (ascending, descending, shuffled).  A thread that overwrote a byte
// another thread had not yet copied out shows up as a wrong copy-out.
//
// Cases: float and double elements; full, ragged (not a multiple of 16
// bytes) and short units on either side; the user buffer on either side
// aligned or one or more elements off a 16-byte boundary.
//
// Prints "COPIER OK <cases>" and exits 0 when every case passed.
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <numeric>
#include <random>
#include <vector>

#define CAIL_COPIER_FN inline
#include "../cail/src/dev/cail_dev_copier.cuh"

namespace {

struct HostV4 {
    static uint4 ld(const void *p) {
        uint4 v;
        memcpy(&v, p, 16);
        return v;
    }
    static void st(void *p, uint4 v) { memcpy(p, &v, 16); }
};

constexpr size_t kUnit = 65536;  // the smallest NVLS unit

// 0 on success; 1: the copy-out returned refilled bytes; 2: the copy-in is
// incomplete; 3: a byte outside [0, n) of the user buffer was written.
template <typename T>
int run_case(size_t n_out, size_t n_in, size_t off_out, size_t off_in, const std::vector<int> &order) {
    std::vector<uint4> slot_mem(kUnit / 16), out_mem(kUnit / 16 + 2), in_mem(kUnit / 16 + 2);
    char *slot = reinterpret_cast<char *>(slot_mem.data());
    char *out0 = reinterpret_cast<char *>(out_mem.data());
    char *dst = out0 + off_out;
    const char *src = reinterpret_cast<const char *>(in_mem.data()) + off_in;
    for (size_t i = 0; i < kUnit; ++i) slot[i] = (char)(i * 7 + 1);
    for (size_t i = 0; i < n_in; ++i) const_cast<char *>(src)[i] = (char)(i * 13 + 5);
    memset(out0, 0x5a, out_mem.size() * 16);
    const std::vector<char> want(slot, slot + n_out);
    for (int tid : order) {
        cail::copier_copy<T, HostV4>(dst, slot, n_out, tid);  // unit j out
        cail::copier_copy<T, HostV4>(slot, src, n_in, tid);   // unit j + 2 in
    }
    if (memcmp(dst, want.data(), n_out) != 0) return 1;
    if (memcmp(slot, src, n_in) != 0) return 2;
    for (size_t i = 0; i < out_mem.size() * 16; ++i)
        if ((out0 + i < dst || out0 + i >= dst + n_out) && out0[i] != 0x5a) return 3;
    return 0;
}

template <typename T>
void run_all(const char *name, int *cases, int *fails) {
    std::vector<std::vector<int>> orders;
    std::vector<int> up(cail::kNvlsCopiers);
    std::iota(up.begin(), up.end(), 0);
    orders.push_back(up);
    orders.emplace_back(up.rbegin(), up.rend());
    std::mt19937 rng(7);
    for (int s = 0; s < 3; ++s) {
        std::vector<int> o = up;
        std::shuffle(o.begin(), o.end(), rng);
        orders.push_back(o);
    }
    const size_t e = sizeof(T);
    // lengths: whole units, ragged ends, one partial chunk, a handful of
    // chunks with a tail, four vectors per thread plus a tail
    const size_t lens[] = {kUnit, kUnit - e, kUnit - 16 + e, e, 16 + e, 2064 + e, 16 * 128 * 4 * 3 + e, 16 * 129};
    for (size_t n_out : lens)
        for (size_t n_in : lens)
            for (size_t off_out = 0; off_out < 16; off_out += e)
                for (size_t off_in = 0; off_in < 16; off_in += e) {
                    if ((off_out && off_out != e && off_out != 16 - e) || (off_in && off_in != e && off_in != 16 - e))
                        continue;  // aligned, one element off, one element short of the next boundary
                    for (const auto &o : orders) {
                        ++*cases;
                        const int r = run_case<T>(n_out, n_in, off_out, off_in, o);
                        if (r) {
                            if (++*fails <= 20)
                                printf("FAIL %s n_out=%zu n_in=%zu off_out=%zu off_in=%zu order[0]=%d: %s\n", name,
                                       n_out, n_in, off_out, off_in, o[0],
                                       r == 1 ? "copy-out read a refilled byte"
                                              : r == 2 ? "copy-in incomplete" : "wrote outside the buffer");
                        }
                    }
                }
}

}  // namespace

int main() {
    int cases = 0, fails = 0;
    run_all<float>("float", &cases, &fails);
    run_all<double>("double", &cases, &fails);
    if (fails) {
        printf("COPIER FAILED %d of %d\n", fails, cases);
        return 1;
    }
    printf("COPIER OK %d\n", cases);
    return 0;
}
