// Sampling on the device (crates/core/src/sample.rs): launch interfaces of sample.cu.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qdec {

struct SamplerCfg {
    float temperature = 0.0f;  // <= 0: greedy
    int top_k = 0;             // 0: off
    float top_p = 1.0f, min_p = 0.0f;
    uint64_t seed = 0;
};

// the RNG state (4 x u64) for `seed`: splitmix64 steps (sample.rs:21-33)
void sampler_seed_state(uint64_t seed, uint64_t out[4]);

// Scratch of one processed row: the sort's keys and ids (in and out) and the radix sort's temporary storage.
size_t sampler_sort_scratch_bytes(int vocab);

// process() of one logits row (sample.rs:182-243): the candidates sorted by (logit desc, id asc), then the
// temperature softmax, top-p, min-p and renormalisation in the reference's order.  Writes the kept set:
// ids[0..n), probs[0..n), *n_out.  scratch: sampler_sort_scratch_bytes(vocab) bytes.
cudaError_t launch_sample_process(const float* logits, int vocab, const SamplerCfg& cfg, void* scratch, int32_t* ids,
                                  float* probs, int* n_out, cudaStream_t s);
// draw() (sample.rs:246-257) from a kept set: one uniform from the RNG state, the first id whose running mass
// exceeds it; the id into *out.
cudaError_t launch_sample_draw(uint64_t* rng, const int32_t* ids, const float* probs, const int* n, int32_t* out,
                               cudaStream_t s);
// write_dense (sample.rs:266-275): q[vocab] = 0 except q[ids[i]] = probs[i].
cudaError_t launch_sample_dense(const int32_t* ids, const float* probs, const int* n, int vocab, float* q, cudaStream_t s);

// The sampled acceptance of a verify batch (spec.rs:367-379 with accept_or_resample, sample.rs:279-313) and the
// round bookkeeping of the greedy accept kernel: rows 0..k of the kept sets (ids/probs at row stride `ld`,
// counts n[row]) are the target's processed distributions, q_dense[i] the draft distribution of draft i
// (vids[1 + i]).  work: `ld` floats.
struct SpecAcceptArgs {
    uint64_t* rng;
    const int32_t* ids;
    const float* probs;
    const int* n;
    size_t ld;
    const float* q_dense;
    int vocab;
    const int32_t* vids;
    int k;
    int* pos;
    int* keep_out;
    int* mpos;
    int32_t* mids;
    int* sel;
    int32_t* emit;
    float* work;
};
cudaError_t launch_spec_accept_sampled(const SpecAcceptArgs& a, cudaStream_t s);

}  // namespace qdec
