// Tensor-parallel exchange between the ranks of one node (one process per GPU): launch interfaces of tp.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

namespace qdec {

// One all-gather step.  Every rank copies `rows` rows of its slice -- up to four byte ranges per row, {seg_src,
// seg_dst, seg_len}, multiples of 16 bytes -- from `src` into every rank's receive buffer dst[k] (peer memory
// opened over CUDA IPC; dst[rank] is local), then raises its flag for `slot` in every rank's flag array
// (pflags[k][slot * 8 + rank] = the session epoch) and waits until all ranks' flags for `slot` have arrived in
// its own array (lflags).  The wait is bounded in time: on expiry it records 0x10000 | slot in *err and returns.
struct XArgs {
    const uint8_t* src;
    long long src_ld;
    uint8_t* dst[8];
    long long dst_ld;
    int seg_src[4], seg_dst[4], seg_len[4];
    int nseg, rows;
    unsigned* pflags[8];
    const unsigned* lflags;
    unsigned* cnt;          // local: CTAs of this slot that finished copying
    const unsigned* epoch;  // local: the session counter
    unsigned* err;
    int slot, rank, world;
};

cudaError_t launch_exchange(const XArgs& a, cudaStream_t s);
// *epoch += 1: a new session (its exchanges reuse the slots from 0 with a larger flag value)
cudaError_t launch_tp_epoch(unsigned* epoch, cudaStream_t s);
// out[row] = the first maximum over the ranks' (value, index) pairs, 16 bytes per rank per row, in rank order
// with the strict > rule (rank 0's pair is seeded with the row's element 0); pairs with index < 0 are skipped.
cudaError_t launch_argmax_combine(const uint8_t* pairs, int world, int rows, int32_t* out, cudaStream_t s);

}  // namespace qdec
