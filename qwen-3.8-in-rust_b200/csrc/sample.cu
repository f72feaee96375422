// Sampling on the device, in the reference's order (crates/core/src/sample.rs): the candidate sort, the
// sequential softmax / top-p / min-p tail, the draw, and the speculative acceptance rule.  The arithmetic is
// scalar and ordered exactly as the reference's (every running sum is one thread's left-to-right chain); only
// the independent per-candidate exps and divisions run in parallel.
#include <cub/device/device_radix_sort.cuh>
#include <cuda_runtime.h>

#include <algorithm>

#include "common.cuh"
#include "sample.cuh"

namespace qdec {

namespace {

__device__ __forceinline__ uint64_t rotl64(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

// xoshiro256** (sample.rs:36-48)
__device__ __forceinline__ uint64_t rng_next(uint64_t* s) {
    const uint64_t result = rotl64(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl64(s[3], 45);
    return result;
}
// (next >> 40) * 2^-24: 24 random bits, exact in f32 (sample.rs:51-55)
__device__ __forceinline__ float rng_f32(uint64_t* s) { return __fmul_rn((float)(rng_next(s) >> 40), 1.0f / 16777216.0f); }

__device__ int32_t draw_from(uint64_t* rng, const int32_t* ids, const float* probs, int n) {  // sample.rs:246-257
    const float u = rng_f32(rng);
    float cum = 0.0f;
    for (int i = 0; i < n; i++) {
        cum = __fadd_rn(cum, probs[i]);
        if (u < cum) return ids[i];
    }
    return ids[n - 1];
}

// sort keys: the logits with -0 made +0 (the reference's comparator treats them as equal; the radix sort orders
// by bits), the ids 0..vocab-1 in ascending order (the stable sort keeps that order among equal keys)
__global__ void sort_keys_kernel(const float* __restrict__ logits, int vocab, float* __restrict__ keys, int32_t* __restrict__ ids) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < vocab; i += gridDim.x * blockDim.x) {
        const float v = logits[i];
        keys[i] = v == 0.0f ? 0.0f : v;
        ids[i] = i;
    }
}

__global__ void __launch_bounds__(1024) process_kernel(const float* __restrict__ logits, int vocab, SamplerCfg cfg,
                                                       const int32_t* __restrict__ sorted, int32_t* __restrict__ ids,
                                                       float* __restrict__ probs, int* __restrict__ n_out) {
    __shared__ float sh_sum, sh_t;
    __shared__ int sh_n;
    const int n_cand = (cfg.top_k > 0 && cfg.top_k < vocab) ? cfg.top_k : vocab;
    const float inv_t = __fdiv_rn(1.0f, cfg.temperature);
    const float m = __fmul_rn(logits[sorted[0]], inv_t);
    for (int i = threadIdx.x; i < n_cand; i += blockDim.x) {
        const int32_t id = sorted[i];
        ids[i] = id;
        probs[i] = exp_f32(__fsub_rn(__fmul_rn(logits[id], inv_t), m));
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float sum = 0.0f;
        for (int i = 0; i < n_cand; i++) sum = __fadd_rn(sum, probs[i]);
        sh_sum = sum;
    }
    __syncthreads();
    const float sum = sh_sum;
    for (int i = threadIdx.x; i < n_cand; i += blockDim.x) probs[i] = __fdiv_rn(probs[i], sum);
    __syncthreads();
    if (threadIdx.x == 0) {
        int n = n_cand;
        if (cfg.top_p < 1.0f) {  // keep while the mass above is below top_p; the crossing token stays
            float cum = 0.0f;
            n = 0;
            while (n < n_cand && cum < cfg.top_p) {
                cum = __fadd_rn(cum, probs[n]);
                n++;
            }
            n = max(n, 1);
        }
        if (cfg.min_p > 0.0f) {  // drop below min_p x the top probability; at least one stays
            const float thr = __fmul_rn(cfg.min_p, probs[0]);
            int keep = 1;
            while (keep < n && probs[keep] >= thr) keep++;
            n = keep;
        }
        float t = 0.0f;
        for (int i = 0; i < n; i++) t = __fadd_rn(t, probs[i]);
        sh_t = t;
        sh_n = n;
        *n_out = n;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < sh_n; i += blockDim.x) probs[i] = __fdiv_rn(probs[i], sh_t);
}

__global__ void draw_kernel(uint64_t* rng, const int32_t* ids, const float* probs, const int* n, int32_t* out) {
    if (threadIdx.x == 0 && blockIdx.x == 0) *out = draw_from(rng, ids, probs, *n);
}

__global__ void __launch_bounds__(1024) dense_kernel(const int32_t* ids, const float* probs, const int* n, int vocab, float* q) {
    for (int i = threadIdx.x; i < vocab; i += blockDim.x) q[i] = 0.0f;
    __syncthreads();
    for (int i = threadIdx.x; i < *n; i += blockDim.x) q[ids[i]] = probs[i];
}

__global__ void spec_accept_sampled_kernel(const SpecAcceptArgs a) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int32_t emitted[16];
    int m = 0, ne = 0;
    while (m < a.k) {  // accept_or_resample at position m (sample.rs:279-313)
        const int32_t* ids = a.ids + (size_t)m * a.ld;
        const float* probs = a.probs + (size_t)m * a.ld;
        const float* q = a.q_dense + (size_t)m * a.vocab;
        const int n = a.n[m];
        const int32_t d = a.vids[1 + m];
        float pd = 0.0f;
        for (int i = 0; i < n; i++)
            if (ids[i] == d) {
                pd = probs[i];
                break;
            }
        const float qd = q[d];
        const float u = rng_f32(a.rng);
        if (qd > 0.0f && (pd >= qd || u < __fdiv_rn(pd, qd))) {
            emitted[ne++] = d;
            m++;
            continue;
        }
        // the residual max(0, p - q) over the kept set of p, renormalised
        float sum = 0.0f;
        for (int i = 0; i < n; i++) {
            const float r = fmaxf(__fsub_rn(probs[i], q[ids[i]]), 0.0f);
            a.work[i] = r;
            sum = __fadd_rn(sum, r);
        }
        if (sum <= 0.0f) {
            emitted[ne++] = draw_from(a.rng, ids, probs, n);  // the processed distribution itself
        } else {
            for (int i = 0; i < n; i++) a.work[i] = __fdiv_rn(a.work[i], sum);
            emitted[ne++] = draw_from(a.rng, ids, a.work, n);
        }
        break;
    }
    if (m == a.k) emitted[ne++] = draw_from(a.rng, a.ids + (size_t)a.k * a.ld, a.probs + (size_t)a.k * a.ld, a.n[a.k]);
    // the round's bookkeeping (as the greedy accept kernel): keep, positions, the MTP re-feed ids
    const int keep = m + 1;
    const int p = *a.pos;
    a.emit[0] = keep;
    for (int i = 0; i <= a.k; i++) {
        const int32_t t = i < keep ? emitted[i] : emitted[keep - 1];
        if (i < keep) a.emit[1 + i] = t;
        a.mids[i] = t;
    }
    *a.keep_out = keep;
    *a.pos = p + keep;
    a.mpos[0] = p;
    for (int i = 1; i < a.k; i++) a.mpos[i] = p + keep + i - 1;
    *a.sel = keep - 1;
}

struct SortLayout {
    size_t keys_in, keys_out, ids_in, ids_out, temp, temp_bytes, total;
};

SortLayout sort_layout(int vocab) {
    SortLayout L{};
    size_t temp_bytes = 0;
    cub::DeviceRadixSort::SortPairsDescending(nullptr, temp_bytes, (const float*)nullptr, (float*)nullptr,
                                              (const int32_t*)nullptr, (int32_t*)nullptr, vocab);
    auto al = [](size_t x) { return (x + 255) & ~(size_t)255; };
    size_t o = 0;
    L.keys_in = o, o += al((size_t)vocab * 4);
    L.keys_out = o, o += al((size_t)vocab * 4);
    L.ids_in = o, o += al((size_t)vocab * 4);
    L.ids_out = o, o += al((size_t)vocab * 4);
    L.temp = o, o += al(temp_bytes);
    L.temp_bytes = temp_bytes;
    L.total = o;
    return L;
}

}  // namespace

void sampler_seed_state(uint64_t seed, uint64_t out[4]) {  // splitmix64 (sample.rs:21-33)
    uint64_t x = seed;
    for (int i = 0; i < 4; i++) {
        x += 0x9E3779B97F4A7C15ull;
        uint64_t z = x;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        out[i] = z ^ (z >> 31);
    }
}

size_t sampler_sort_scratch_bytes(int vocab) { return sort_layout(vocab).total; }

cudaError_t launch_sample_process(const float* logits, int vocab, const SamplerCfg& cfg, void* scratch, int32_t* ids,
                                  float* probs, int* n_out, cudaStream_t s) {
    if (vocab <= 0 || cfg.temperature <= 0.0f) return cudaErrorInvalidValue;
    const SortLayout L = sort_layout(vocab);
    uint8_t* b = static_cast<uint8_t*>(scratch);
    float* keys_in = reinterpret_cast<float*>(b + L.keys_in);
    float* keys_out = reinterpret_cast<float*>(b + L.keys_out);
    int32_t* ids_in = reinterpret_cast<int32_t*>(b + L.ids_in);
    int32_t* ids_out = reinterpret_cast<int32_t*>(b + L.ids_out);
    sort_keys_kernel<<<std::min((vocab + 255) / 256, 1024), 256, 0, s>>>(logits, vocab, keys_in, ids_in);
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    size_t tb = L.temp_bytes;
    e = cub::DeviceRadixSort::SortPairsDescending(b + L.temp, tb, keys_in, keys_out, ids_in, ids_out, vocab, 0, 32, s);
    if (e != cudaSuccess) return e;
    process_kernel<<<1, 1024, 0, s>>>(logits, vocab, cfg, ids_out, ids, probs, n_out);
    return cudaGetLastError();
}

cudaError_t launch_sample_draw(uint64_t* rng, const int32_t* ids, const float* probs, const int* n, int32_t* out,
                               cudaStream_t s) {
    draw_kernel<<<1, 32, 0, s>>>(rng, ids, probs, n, out);
    return cudaGetLastError();
}

cudaError_t launch_sample_dense(const int32_t* ids, const float* probs, const int* n, int vocab, float* q, cudaStream_t s) {
    dense_kernel<<<1, 1024, 0, s>>>(ids, probs, n, vocab, q);
    return cudaGetLastError();
}

cudaError_t launch_spec_accept_sampled(const SpecAcceptArgs& a, cudaStream_t s) {
    if (a.k < 1 || a.k > 15) return cudaErrorInvalidValue;
    spec_accept_sampled_kernel<<<1, 32, 0, s>>>(a);
    return cudaGetLastError();
}

}  // namespace qdec
