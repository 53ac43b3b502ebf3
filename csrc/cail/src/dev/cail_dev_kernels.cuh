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

// Push two-shot over the communicator's IPC workspace (no host exchange).
// The message is cut into P slices (16-byte units; slice P-1 also holds the
// ragged tail); slice q is reduced by rank q.  CTA b of every rank handles,
// in round k, the piece of every slice at slice-relative byte offset
// (k * G + b) * piece:
//   1. it pushes its piece of slice q into RS slot (parity, b, rank) of rank
//      q's workspace, for every q != rank (NVLink stores), and raises
//      flag RS[rank][b] = epoch on each peer with st.release.sys;
//   2. it waits for RS[q][b] >= epoch from every peer (ld.acquire.sys), folds
//      the P pieces of its own slice in rank order (its own piece straight
//      from the input), stores the result into its output and into AG slot
//      (parity, b, rank) of every peer, and raises AG[rank][b];
//   3. it waits for every peer's AG[q][b] and copies the gathered pieces of
//      the other slices from its AG slots into its output.
// Epochs grow by one per round, so flags never need resetting, and slots
// alternate between two parities: round k + 2 of a CTA starts only after it
// has received the peers' AG pieces of round k + 1, which each peer sends
// after it finished reading its slots of round k.  No rank reads or writes
// another rank's user buffers, so the call needs no host barrier and the
// buffers are free for reuse as soon as the kernel has finished.
// A launch may run several ranks' CTAs (the one-GPU emulation used by the
// tests): CTA i belongs to rank rank0 + i / G and is CTA i % G of that rank.
constexpr int kRsFlagBase = kFlagWords;      // word offsets in the flag array
constexpr int kAgFlagBase = 2 * kFlagWords;
struct PushArgs {
    const char *src[kMaxRanks];      // input of each rank this launch runs (production: [rank])
    char *dst[kMaxRanks];            // output of each rank this launch runs
    char *rs[kMaxRanks];             // RS area of every rank's workspace (peer mappings)
    char *ag[kMaxRanks];             // AG area of every rank's workspace (peer mappings)
    uint32_t *flags[kMaxRanks];      // flag array of every rank (peer mappings)
    size_t slice_off[kMaxRanks + 1]; // byte offset of slice q; slice_off[P] = message bytes
    size_t max_slice;                // bytes of the longest slice
    size_t piece;                    // bytes per CTA, round and slice (a multiple of 16)
    int P, rank0, G, rounds;
    uint32_t epoch0;                 // epoch of round 0
    int vec;                         // every user buffer is 16-byte aligned
    unsigned long long timeout_ns;
    DevStatus *status;
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
// Push two-shot: a.G * ranks CTAs of 512 threads, where ranks = 1 in
// production; cooperative = true launches it as a cooperative kernel (the
// emulation of several ranks on one GPU, whose CTAs wait on one another).
cudaError_t launch_push(int op, int ec, const PushArgs &a, int ranks, bool cooperative, cudaStream_t s);
// Largest G for which `ranks` x G CTAs of the push kernel are co-resident.
int push_max_ctas(int ranks, int sm_count);
// Device copy through TMA bulk copies, one CTA per SM (large one-rank
// copies); src and dst must share their alignment modulo 16.  *status gets 1
// when a wait ran out after timeout_ns, 2 when the drain after it also did.
cudaError_t launch_bulk_copy(char *dst, const char *src, size_t bytes, int sm_count, unsigned long long timeout_ns,
                             int *status, cudaStream_t s);
// 1 if the NVLS kernel exists for (op, ec).
int nvls_supported(int op, int ec);
// Device-to-device copy of `bytes` bytes (the one-rank allreduce); src and dst
// must share their alignment modulo 16.  16-byte vectors, eight loads in
// flight per thread, at most two 512-thread CTAs per SM.
cudaError_t launch_copy(char *dst, const char *src, size_t bytes, int sm_count, cudaStream_t s);
// Element-wise local reduction io = op(io, in) (PMPI algorithm path).
cudaError_t launch_reduce_local(int op, int ec, const void *in, void *io, size_t n, int sm_count,
                                cudaStream_t s);

}  // namespace cail
