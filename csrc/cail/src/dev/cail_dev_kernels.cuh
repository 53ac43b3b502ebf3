// cail_dev_kernels.cuh — argument blocks and launchers of the NVLink kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cail {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 512;           // flag slots per (source rank) and barrier kind
constexpr int kFlagWords = kMaxRanks * kMaxBlocks;

// Device-side error report (host-mapped).  code: 0 ok, 1 barrier timeout.
struct DevStatus {
    int code;
    int rank;       // rank whose kernel gave up
    int waited_on;  // peer it was waiting for
    int block;
    unsigned int epoch;
    unsigned int seen;
};

// One-shot (push): every rank writes its input into slot `rank` of every
// rank's scratch (posted NVLink stores), signals each peer with a release
// flag per CTA, waits for the P-1 flags addressed to it, then folds its P
// local slots in rank order into its output.  Scratch is double-buffered
// by epoch parity, so no trailing barrier is needed.
struct OneShotArgs {
    const char *src;                 // this rank's input (user buffer)
    char *dst;                       // this rank's output (user buffer)
    size_t count;                    // elements (count * size <= slot bytes)
    char *slot_out[kMaxRanks];       // slot `rank` of each rank's scratch, this parity (peer mappings)
    const char *slot_in;             // slot 0 of this rank's scratch, this parity
    size_t slot_bytes;               // distance between slots
    uint32_t *peer_flags[kMaxRanks]; // each rank's arrival flag array (peer mappings)
    uint32_t *my_flags;              // this rank's arrival flag array
    int P, rank;
    uint32_t epoch;
    unsigned long long timeout_ns;
    DevStatus *status;
};

// Two-shot over registered user buffers: rank r reduces slice r of the
// vectorised range from all P inputs and stores it into all P outputs;
// rank 0 also handles the unaligned head and the tail elements.
struct TwoShotArgs {
    const char *src[kMaxRanks];      // every rank's input (peer mappings)
    char *dst[kMaxRanks];            // every rank's output (peer mappings)
    size_t count;                    // elements
    size_t head;                     // leading elements before the first 16-byte boundary
    size_t nvec;                     // 16-byte vectors after the head
    int P, rank;
    int vector_ok;                   // all buffers share the same alignment mod 16
    int unroll2;                     // process two vectors per loop iteration
};

// NVLS two-shot of one chunk: every rank copies its chunk into its unicast
// view of a multicast-bound staging buffer; after a barrier rank r reduces
// its slice with multimem.ld_reduce through the multicast view and
// broadcasts it with multimem.st; after a second barrier every rank copies
// the chunk out.  The barrier is a counter in the multicast region that each
// CTA of each rank increments once (multimem.red); a barrier is passed when
// the local copy of the counter reaches its target.
struct NvlsArgs {
    const char *src;                 // this rank's input chunk (user buffer)
    char *dst;                       // this rank's output chunk (user buffer)
    char *uc;                        // unicast view of this chunk's staging half
    char *mc;                        // multicast view of the same staging half
    uint32_t *mc_counter;            // multicast view of the barrier counter
    const uint32_t *uc_counter;      // this rank's unicast view of the counter
    size_t count;                    // elements in this chunk
    int P, rank;
    uint32_t target_a, target_b;     // counter values that complete barrier A / B
    unsigned long long timeout_ns;
    DevStatus *status;
};

// Launchers: return cudaSuccess or the launch error.  ec is a
// cail_elem_class_t, op a cail_op_t.
cudaError_t launch_oneshot(int op, int ec, const OneShotArgs &a, int blocks, int threads,
                           cudaStream_t s);
cudaError_t launch_twoshot(int op, int ec, const TwoShotArgs &a, int blocks, int threads,
                           cudaStream_t s);
cudaError_t launch_nvls(int op, int ec, const NvlsArgs &a, int blocks, int threads, cudaStream_t s);
// 1 if the NVLS kernel exists for (op, ec).
int nvls_supported(int op, int ec);
// Element-wise local reduction io = op(io, in) (PMPI algorithm path).
cudaError_t launch_reduce_local(int op, int ec, const void *in, void *io, size_t n, int sm_count,
                                cudaStream_t s);

}  // namespace cail
