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

// Pipelined NVLS allreduce of a whole message.  The message is cut into
// sub-chunks that flow through a ring of 3 staging slots in a
// multicast-bound region.  Iteration k (k = 0 .. K+1) copies sub-chunk k into
// this rank's slot k%3, reduces this rank's slice of sub-chunk k-1 with
// multimem.ld_reduce through the multicast view and broadcasts it with
// multimem.st, and copies sub-chunk k-2 out of its slot; then all CTAs of
// all ranks meet at a barrier.  With 3 slots, every slot's previous readers
// and writers are done before the barrier that precedes its reuse.  The
// barrier has two levels: CTAs arrive on a counter local to their GPU
// (complete at local0 + (k + 1) * gridDim.x); the last arrival adds 1 to a
// counter in the multicast region on every GPU (multimem.red); iteration k
// is complete when the local copy of that counter reaches
// target0 + (k + 1) * P.  Copy work and multimem work run on disjoint CTAs.
constexpr int kNvlsSlots = 3;
struct NvlsArgs {
    const char *src;                 // this rank's input (user buffer)
    char *dst;                       // this rank's output (user buffer)
    char *uc;                        // unicast view of slot 0 (slots are slot_bytes apart)
    char *mc;                        // multicast view of slot 0
    uint32_t *mc_counter;            // multicast view of the cross-rank counter
    const uint32_t *uc_counter;      // this rank's unicast view of that counter
    uint32_t *local_counter;         // this GPU's arrival counter (unicast only)
    size_t count;                    // elements in the message
    size_t sub;                      // elements per sub-chunk (sub * size is a multiple of 16)
    size_t slot_bytes;
    int P, rank;
    int copy_blocks;                 // CTAs [0, copy_blocks) copy, the rest reduce
    uint32_t target0, local0;
    unsigned long long timeout_ns;
    DevStatus *status;
};

// Rank-order fold of P local sources into dst: dst = src[0] op src[1] op ...
// (the copy-engine two-shot reduces its slice of each chunk with it, after
// the copy engines have pulled the peers' parts into local scratch).
struct FoldArgs {
    const char *src[kMaxRanks];
    char *dst;
    size_t count;                    // elements
    int P;
};

// Launchers: return cudaSuccess or the launch error.  ec is a
// cail_elem_class_t, op a cail_op_t.
cudaError_t launch_oneshot(int op, int ec, const OneShotArgs &a, int blocks, int threads,
                           cudaStream_t s);
cudaError_t launch_twoshot(int op, int ec, const TwoShotArgs &a, int blocks, int threads,
                           cudaStream_t s);
cudaError_t launch_nvls(int op, int ec, const NvlsArgs &a, int blocks, int threads, cudaStream_t s);
cudaError_t launch_fold(int op, int ec, const FoldArgs &a, int blocks, int threads, cudaStream_t s);
// Device copy through TMA bulk copies (experimental, single-GPU harness only);
// src and dst must share their alignment modulo 16.  *status gets 1 when a
// wait ran out after spin_limit polls.
cudaError_t launch_bulk_copy(char *dst, const char *src, size_t bytes, int blocks, unsigned long long spin_limit,
                             int *status, cudaStream_t s);
// 1 if the NVLS kernel exists for (op, ec).
int nvls_supported(int op, int ec);
// Element-wise local reduction io = op(io, in) (PMPI algorithm path).
cudaError_t launch_reduce_local(int op, int ec, const void *in, void *io, size_t n, int sm_count,
                                cudaStream_t s);

}  // namespace cail
