// Tensor-parallel exchange between the ranks of one node (one process per GPU): launch interfaces of tp.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qdec {

// How long an exchange polls for a peer's lines before it gives up (a peer this late is treated as gone).
constexpr unsigned long long EXCHANGE_WAIT_NS = 5000000000ull;

// One all-gather step in the low-latency line format: every 4 data bytes travel as one 8-byte line {data, tag},
// written and read with single 64-bit accesses (naturally aligned, so single-copy atomic: a reader sees either the
// whole old line or the whole new one), so a line that shows this step's tag holds its data -- no fences or
// separate flags.  Each rank writes the lines of its slice (`rows` rows of up to four byte ranges {seg_src,
// seg_dst, seg_len}, multiples of 16 bytes, from `src`) into every other rank's line buffer ll[k] at the position
// that mirrors the slice's place in the full rows (line index = byte offset / 4, row stride dst_ld), copies it
// straight into its own receive buffer `out`, then polls its own line buffer `ll_local` for the rest of the full
// rows (rows x dst_ld bytes) and unpacks them into `out`.  tag = epoch * 1024 + slot + 1 changes every step;
// consecutive steps alternate between two line buffers, and a rank cannot run two steps ahead of another, so a
// line is never overwritten before it is read.  The poll is bounded in time (wait_ns, 0 = EXCHANGE_WAIT_NS): on
// expiry the step records 0x10000 | slot in *err and returns.
struct XArgs {
    const uint8_t* src;
    long long src_ld;
    uint8_t* ll[8];          // every rank's line buffer for this step (ll[rank] unused)
    const uint8_t* ll_local;  // this rank's line buffer for this step
    uint8_t* out;            // this rank's receive buffer (full rows)
    long long dst_ld;
    int seg_src[4], seg_dst[4], seg_len[4];
    int nseg, rows;
    const unsigned* epoch;   // local: the session counter
    unsigned* err;
    unsigned long long* stats;  // local: {steps, ns until pushed, ns until all arrived, 0}
    int slot, rank, world;
    unsigned long long wait_ns;
};

cudaError_t launch_exchange(const XArgs& a, cudaStream_t s);
// Failure-handling self-test of the exchange poll on the current device, one process, no peer: a step whose peer
// lines carry the previous step's tag must give up after wait_ns with the slot's error word, leaving the context
// usable; the same step with the peer's lines in place must then complete with the full rows.  0, or a code naming
// the half that misbehaved.
int selftest_exchange(unsigned long long wait_ns);
// *epoch += 1: a new session (its exchanges reuse the slots from 0 with new tags)
cudaError_t launch_tp_epoch(unsigned* epoch, cudaStream_t s);
// out[row] = the first maximum over the ranks' (value, index) pairs, 16 bytes per rank per row, in rank order
// with the strict > rule (rank 0's pair is seeded with the row's element 0); pairs with index < 0 are skipped.
cudaError_t launch_argmax_combine(const uint8_t* pairs, int world, int rows, int32_t* out, cudaStream_t s);

}  // namespace qdec
