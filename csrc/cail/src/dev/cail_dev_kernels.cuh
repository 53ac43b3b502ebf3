// cail_dev_kernels.cuh — argument blocks and launchers of the NVLink kernels.
#pragma once

#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

namespace cail {

constexpr int kMaxRanks = 8;
constexpr int kMaxBlocks = 512;           // flag slots per (source rank) and barrier kind
constexpr int kFlagWords = kMaxRanks * kMaxBlocks;

// Device-side error report (host-mapped).  code: 0 ok, 1 barrier timeout,
// 2 argument check failed (CAIL_DEVICE_CHECKS; waited_on holds the check).
struct DevStatus {
    int code;
    int rank;       // rank whose kernel gave up
    int waited_on;  // peer it was waiting for (code 2: the failed check)
    int block;
    unsigned int epoch;
    unsigned int seen;
};

// One-shot (push): every rank pushes its whole input, piece by piece, into
// its slot of every other rank's one-shot area (NVLink stores), and every
// rank folds the P copies of each piece in rank order (its own piece straight
// from its input) into its output.  CTA b of every rank handles, in round k,
// the piece at byte offset (k * G + b) * piece:
//   wait until every peer raised OS[q][b] >= epoch (its piece of round k is
//   in this rank's area), push the piece of round k + 1 and raise
//   OS[rank][b] = epoch + 1 on every peer, then fold round k.
// Round k + 1 goes out before round k is folded, so slots rotate through
// three: the slot of round k + 1 was last used by round k - 2, which every
// peer folded before it raised the flag of round k that this CTA has just
// received.  The rotation must advance by exactly one per round of a CTA,
// across calls too, so each CTA keeps its own completed-round count in
// `rounds_done` (this GPU's memory; the same on every rank because every rank
// runs the same rounds): round k of a call has epoch rounds_done[b] + k + 1.
// A single round per CTA (small messages) costs one flag exchange.
constexpr int kOsSlots = 3;
struct OneShotArgs {
    const char *src[kMaxRanks];      // input of each rank this launch runs (production: [rank])
    char *dst[kMaxRanks];            // output of each rank this launch runs
    char *slots[kMaxRanks];          // one-shot area of every rank (peer mappings)
    uint32_t *flags[kMaxRanks];      // flag array of every rank (peer mappings)
    uint32_t *rounds_done[kMaxRanks];// per-CTA completed rounds of each rank this launch runs
    size_t bytes;                    // message bytes
    size_t piece;                    // bytes per CTA and round (a multiple of 16)
    size_t area;                     // bytes of each one-shot area
    // Slot layout: slot s of CTA b for source q starts at
    // ((s * sg + b) * P + q) * piece, with sg >= G fixed for the
    // communicator (its largest CTA count).  A CTA's slots then sit at the
    // same place in every call with the same piece, whatever the call's G:
    // a rank may start pushing its next call while a peer still folds the
    // last rounds of the previous one, and the slot rotation protects only
    // the slots of the same CTA.  (The host separates calls whose pieces
    // differ; every message up to sg x 8 KiB has the 8 KiB piece.)
    int sg;
    int P, rank0, G;
    int vec;                         // every user buffer is 16-byte aligned
    unsigned long long timeout_ns;
    DevStatus *status;
    int checks;                      // validate the arguments first (CAIL_DEVICE_CHECKS)
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
// alternate between two parities.  A CTA pushes round k + 1's pieces (step 1)
// right after it raised AG for round k, before it waits for the peers' AG of
// round k: those RS slots (round k - 1's parity) are free because every peer
// raised AG for round k - 1 only after folding them.  Its AG pieces of round
// k go out after it received the peers' RS pieces of round k, which each
// peer sends after it finished copying out its AG slots of round k - 2.  No rank reads or writes
// another rank's user buffers, so the call needs no host barrier and the
// buffers are free for reuse as soon as the kernel has finished.
// A launch may run several ranks' CTAs (the one-GPU emulation used by the
// tests): CTA i belongs to rank rank0 + i / G and is CTA i % G of that rank.
// With checks set, every CTA first validates the arguments (rank and CTA
// counts against the grid, piece alignment, slot bounds against the area,
// the slice table, round coverage, pointer alignment) and, if one fails,
// reports DevStatus code 2 with the check's number and returns before it
// touches memory or waits on a flag; every CTA sees the same arguments, so
// all of them return.
constexpr int kOsFlagBase = 0;               // word offsets in the flag array
constexpr int kRsFlagBase = kFlagWords;
constexpr int kAgFlagBase = 2 * kFlagWords;
constexpr int kNvlsStepsBase = 3 * kFlagWords;      // NVLS per-CTA steps (kMaxBlocks words)
constexpr int kOsRoundsBase = 3 * kFlagWords + kMaxBlocks;  // one-shot per-CTA rounds (kMaxBlocks words)
constexpr int kFlagAreaWords = 3 * kFlagWords + 2 * kMaxBlocks;
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
    size_t area;                     // bytes of each RS / AG area (bounds of the slots)
    int checks;                      // validate the arguments first (CAIL_DEVICE_CHECKS)
};

// NVLS allreduce through NVSwitch multicast, one independent pipeline per
// CTA.  The message is cut into units of `unit` bytes; CTA b handles units
// b, b + G, b + 2G, ... through two staging slots of `unit` bytes in the
// multicast-bound region of every GPU.  For each of its units k:
//   1. copier warps copy the unit from the input into slot k % 2 (local HBM),
//   2. the leader meets CTA b of every other rank: fence, one
//      multimem.red.release that adds 1 to its counter A[b] on every GPU,
//      then a wait until this GPU's copy of A[b] shows all P arrivals,
//   3. reducer warps reduce this rank's 1/P of the unit with
//      multimem.ld_reduce through the multicast view and broadcast it with
//      multimem.st,
//   4. the leader meets the others again on counter B[b] (every rank's share
//      is now in every GPU's slot),
//   5. copier warps copy the reduced unit from the slot into the output.
// Copier warps run one unit ahead (copy-in of k + 1, copy-out of k - 1)
// while the reducers work on unit k, and different CTA indices never wait on
// one another, so local copies overlap the NVLink traffic without a
// grid-wide barrier.  Counters only grow: steps[b] (this GPU's unicast
// memory, the same on every GPU) holds the units CTA b completed in earlier
// calls, so unit k of this call is complete at (steps[b] + k + 1) * P
// arrivals.  Counters are kNvlsCtrStride bytes apart.
constexpr int kNvlsCtrStride = 128;
constexpr size_t kNvlsCtrBytes = 2 * (size_t)kMaxBlocks * kNvlsCtrStride;  // A and B counters
struct NvlsArgs {
    const char *src;                 // this rank's input (user buffer)
    char *dst;                       // this rank's output (user buffer)
    char *uc;                        // unicast view of slot 0 (CTA b's slots at uc + (2b + s) * unit)
    char *mc;                        // multicast view of slot 0
    char *mc_ctr;                    // multicast view of the counters (A[b], then B[b])
    const char *uc_ctr;              // this GPU's unicast view of the counters
    uint32_t *steps;                 // per-CTA completed steps (unicast, kMaxBlocks words)
    size_t bytes;                    // message bytes
    size_t unit;                     // bytes per CTA and step (a multiple of 16)
    size_t area;                     // bytes of the staging region (bounds of the slots)
    int P, rank;
    unsigned long long timeout_ns;
    DevStatus *status;
    int checks;                      // validate the arguments first (CAIL_DEVICE_CHECKS)
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
// One-shot: a.G * ranks CTAs of 512 threads (ranks = 1 in production;
// cooperative for the one-GPU emulation of several ranks).
cudaError_t launch_oneshot(int op, int ec, const OneShotArgs &a, int ranks, bool cooperative, cudaStream_t s);
cudaError_t launch_twoshot(int op, int ec, const TwoShotArgs &a, int blocks, int threads,
                           cudaStream_t s);
cudaError_t launch_nvls(int op, int ec, const NvlsArgs &a, int blocks, cudaStream_t s);
// CTAs of the NVLS kernel that are co-resident on one GPU (512 threads each).
int nvls_max_ctas(int sm_count);
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
// stream: streaming cache hints (messages whose buffers overflow L2).
cudaError_t launch_copy(char *dst, const char *src, size_t bytes, int sm_count, cudaStream_t s, bool stream);
// Element-wise local reduction io = op(io, in) (PMPI algorithm path).
cudaError_t launch_reduce_local(int op, int ec, const void *in, void *io, size_t n, int sm_count,
                                cudaStream_t s);

}  // namespace cail
