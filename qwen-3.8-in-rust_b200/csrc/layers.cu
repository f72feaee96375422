// Per-layer kernels of the decode step, each bit-exact with the reference's f32 order:
//
//   resid_norm_quant  h = a + b; y = rmsnorm(h, w); y -> Q8_K / Q8_0 rows   (layers/mod.rs:316-323,
//                     kernels/rmsnorm.rs:14-76, q8k.rs:76-114, q8.rs:81-103)
//   swiglu_quant      h = silu(g) * u; h -> Q8_K / Q8_0                     (layers/mlp.rs:53-64, act.rs:24)
//   conv_step         causal depthwise conv + SiLU, t rows, deferred commit  (kernels/conv.rs:11-36)
//   deltanet_heads    l2norm, gates, gated delta rule, gated RMSNorm per V head, t rows sequential, with the
//                     state commit of the previous round's accepted rows    (layers/gated_deltanet.rs:261-370,
//                     kernels/deltanet.rs:19-89, spec.rs:395-415)
//   qk_norm_rope      per-head q/k RMSNorm, partial rotate-half RoPE, K/V cache append
//                                                                           (layers/gqa_attention.rs:343-362)
//   attention         scores over the cache, softmax, V sum, sigmoid gate   (layers/gqa_attention.rs:376-409,
//                                                                            kernels/softmax.rs:22-50)
//   argmax            first index of the maximum                            (model.rs:505-513)
//
// "Bit-exact" holds with the transcendentals of common.cuh (exp/log1p evaluated in double, rounded once).

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "layers.cuh"

namespace qdec {

namespace {

// The reference's 8-lane sum of squares over x[0..n) (rmsnorm.rs:55-69): lane k accumulates x[k], x[k+8], ...
// left to right; then reduce8; then the n % 8 tail left to right.  `xs` is in shared memory; the 8 lanes run
// on threads 0..7 of the block; the result is returned on every thread (via shared memory).
__device__ float sum_squares_8lane_block(const float* xs, int n, float* red) {
    const int n8 = n / 8 * 8;
    if (threadIdx.x < 8) {
        float acc = 0.0f;
#pragma unroll 8
        for (int i = threadIdx.x; i < n8; i += 8) acc = __fadd_rn(acc, __fmul_rn(xs[i], xs[i]));
        red[threadIdx.x] = acc;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float ss = reduce8(red);
        for (int i = n8; i < n; i++) ss = __fadd_rn(ss, __fmul_rn(xs[i], xs[i]));
        red[8] = ss;
    }
    __syncthreads();
    const float r = red[8];
    __syncthreads();
    return r;
}

// 1 / sqrt(mean + eps) with mean = ss / n (rmsnorm.rs:49-53)
__device__ __forceinline__ float inv_rms_of(float ss, int n, float eps) {
    return __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(__fdiv_rn(ss, (float)n), eps)));
}

// Quantise the 256 values of one chunk held in shared memory: warp 0 writes the Q8_K image block
// (q8k.rs:76-114), warps 0..7 the chunk's eight Q8_0 blocks into the row's Q8_0 image (q8.rs:81-103), whose
// codes start at q80_row and {d, sum} entries after the row's n/32 blocks of codes.  Block of 256 threads.
__device__ void quant_chunk(const float* xs, uint8_t* img_blk, uint8_t* q80_row, int n, int chunk) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (img_blk && warp == 0) {
        float v[8];
#pragma unroll
        for (int i = 0; i < 8; i++) v[i] = xs[lane * 8 + i];
        q8k_quantize_to_image(v, img_blk);
    }
    if (q80_row && warp < 8) {
        const int blk = chunk * 8 + warp;
        q80_quantize_to_image(xs[warp * 32 + lane], q80_row + (size_t)blk * 32, q80_row + (size_t)(n / 32) * 32 + (size_t)blk * 8);
    }
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace

// Grid (n / 256 chunks, rows), 256 threads.  h = a + b (b may be null: h = a); the CTA of chunk c writes chunk c
// of h to h_out (which must not alias a or b: every CTA of the row reads the whole row); y = rmsnorm(h, w)
// (rmsnorm.rs:14-76, the 8-lane sum over the whole row, recomputed by every CTA of the row) for its chunk,
// written to y_out when given and quantised into the Q8_K image / Q8_0 rows when given.
constexpr int RN_REG_VECS = 8;  // float4 of a row held per thread (rows up to 8192 values at 256 threads)

__global__ void __launch_bounds__(256)
resid_norm_quant_kernel(const float* __restrict__ a, const float* __restrict__ b, float* __restrict__ h_out,
                        const float* __restrict__ w, float eps, int n, float* __restrict__ y_out,
                        uint8_t* __restrict__ img_out, uint8_t* __restrict__ q80_out) {
    extern __shared__ __align__(16) float sm[];
    float* sq = sm;             // squares of the row, lane-major: sq[l * (n / 8) + k] = h[8k + l]^2 (n % 256 == 0)
    float* red = sm + n;        // 16
    float* ys = red + 16;       // this chunk's normed values
    __shared__ float hc[256];   // this chunk of h
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.y, c0 = blockIdx.x * 256, per = n / 8;
    const float4* a4 = reinterpret_cast<const float4*>(a + (size_t)row * n);
    const float4* b4 = b ? reinterpret_cast<const float4*>(b + (size_t)row * n) : nullptr;
    auto put = [&](int i, float4 v) {
        // elements 4i .. 4i+3: lanes (4i) % 8 .. +3, position (4i) / 8 in each lane
        const int l0 = (4 * i) & 7, k = (4 * i) >> 3;
        sq[(l0 + 0) * per + k] = __fmul_rn(v.x, v.x);
        sq[(l0 + 1) * per + k] = __fmul_rn(v.y, v.y);
        sq[(l0 + 2) * per + k] = __fmul_rn(v.z, v.z);
        sq[(l0 + 3) * per + k] = __fmul_rn(v.w, v.w);
        if (4 * i >= c0 && 4 * i < c0 + 256) reinterpret_cast<float4*>(hc)[(4 * i - c0) >> 2] = v;
    };
    auto sum4 = [](float4 v, float4 u) {
        return make_float4(__fadd_rn(v.x, u.x), __fadd_rn(v.y, u.y), __fadd_rn(v.z, u.z), __fadd_rn(v.w, u.w));
    };
    if (n / 4 <= RN_REG_VECS * (int)blockDim.x) {
        // rows up to RN_REG_VECS float4 per thread: every load issued before the first use, so the row arrives
        // in one memory round trip rather than one per iteration
        float4 va[RN_REG_VECS], vb[RN_REG_VECS];
#pragma unroll
        for (int j = 0; j < RN_REG_VECS; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n / 4) {
                va[j] = a4[i];
                if (b4) vb[j] = b4[i];
            }
        }
#pragma unroll
        for (int j = 0; j < RN_REG_VECS; j++) {
            const int i = threadIdx.x + j * blockDim.x;
            if (i < n / 4) put(i, b4 ? sum4(va[j], vb[j]) : va[j]);
        }
    } else {
        for (int i = threadIdx.x; i < n / 4; i += blockDim.x) put(i, b4 ? sum4(a4[i], b4[i]) : a4[i]);
    }
    __syncthreads();
    if (h_out) h_out[(size_t)row * n + c0 + threadIdx.x] = hc[threadIdx.x];
    // the 8-lane sum of squares (rmsnorm.rs:55-76): lane l adds h[l]^2, h[l+8]^2, ... left to right
    if (threadIdx.x < 8) {
        const float4* q = reinterpret_cast<const float4*>(sq + threadIdx.x * per);
        float acc = 0.0f;
#pragma unroll 4
        for (int k = 0; k < per / 4; k++) {
            const float4 v = q[k];
            acc = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(acc, v.x), v.y), v.z), v.w);
        }
        red[threadIdx.x] = acc;
    }
    __syncthreads();
    const float inv = inv_rms_of(reduce8(red), n, eps);
    const float y = __fmul_rn(__fmul_rn(hc[threadIdx.x], inv), w[c0 + threadIdx.x]);
    ys[threadIdx.x] = y;
    if (y_out) y_out[(size_t)row * n + c0 + threadIdx.x] = y;
    __syncthreads();
    quant_chunk(ys, img_out ? img_out + ((size_t)row * (n / 256) + blockIdx.x) * Q8K_IMG_BYTES : nullptr,
                q80_out ? q80_out + (size_t)row * (n / 32) * Q80_IMG_BYTES : nullptr, n, blockIdx.x);
}

// One CTA per row: y[row * y_ld + i] = rmsnorm(x[row * x_ld ..], w)[i] (rmsnorm.rs:25-33).
__global__ void rmsnorm_rows_kernel(const float* __restrict__ x, int x_ld, const float* __restrict__ w, float eps, int n,
                                    float* __restrict__ y, int y_ld) {
    extern __shared__ __align__(16) float sm[];
    float* xs = sm;
    float* red = sm + n;
    const float* xr = x + (size_t)blockIdx.x * x_ld;
    for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = xr[i];
    __syncthreads();
    const float inv = inv_rms_of(sum_squares_8lane_block(xs, n, red), n, eps);
    for (int i = threadIdx.x; i < n; i += blockDim.x) y[(size_t)blockIdx.x * y_ld + i] = __fmul_rn(__fmul_rn(xs[i], inv), w[i]);
}

// Grid (n / 256, rows), 256 threads: h = silu(g) * u (act.rs:24) for one chunk, optionally written, quantised.
__global__ void __launch_bounds__(256)
swiglu_quant_kernel(const float* __restrict__ g, const float* __restrict__ u, int n, float* __restrict__ h_out,
                    uint8_t* __restrict__ img_out, uint8_t* __restrict__ q80_out) {
    __shared__ float hs[256];
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.y;
    const size_t i = (size_t)row * n + blockIdx.x * 256 + threadIdx.x;
    const float h = __fmul_rn(silu_f32(g[i]), u[i]);
    hs[threadIdx.x] = h;
    if (h_out) h_out[i] = h;
    __syncthreads();
    quant_chunk(hs, img_out ? img_out + ((size_t)row * (n / 256) + blockIdx.x) * Q8K_IMG_BYTES : nullptr,
                q80_out ? q80_out + (size_t)row * (n / 32) * Q80_IMG_BYTES : nullptr, n, blockIdx.x);
}

// Grid (n / 256, rows), 256 threads: quantise rows already in global memory (the mixer outputs).
__global__ void __launch_bounds__(256)
quant_rows_kernel(const float* __restrict__ x, int n, uint8_t* __restrict__ img_out, uint8_t* __restrict__ q80_out) {
    __shared__ float hs[256];
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.y;
    hs[threadIdx.x] = x[(size_t)row * n + blockIdx.x * 256 + threadIdx.x];
    __syncthreads();
    quant_chunk(hs, img_out ? img_out + ((size_t)row * (n / 256) + blockIdx.x) * Q8K_IMG_BYTES : nullptr,
                q80_out ? q80_out + (size_t)row * (n / 32) * Q80_IMG_BYTES : nullptr, n, blockIdx.x);
}

// Causal depthwise conv1d (+ SiLU) for t rows, one thread per channel (conv.rs:11-36).  The committed window
// `state` (channels x (K-1)) first absorbs the `keep` pending inputs of the previous call (the accepted rows of
// the previous round), then the t new rows are stepped from it; their inputs become the new pending rows.
// Launched as a programmatic dependent of the ssm_alpha/ssm_beta GEMV, whose outputs it does not read: x (the
// qkv projection) is three launches back, so the whole step runs before griddepcontrol.wait.
__device__ __forceinline__ void conv_done() {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__global__ void conv_step_kernel(float* __restrict__ state, const float* __restrict__ w, int K, int channels,
                                 const float* __restrict__ x, int t, float* __restrict__ out, float* __restrict__ pend_x,
                                 const int* __restrict__ keep_prev, int max_t) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) {
        conv_done();
        return;
    }
    float st[8];
    for (int j = 0; j < K - 1; j++) st[j] = state[(size_t)c * (K - 1) + j];
    const int keep = keep_prev ? *keep_prev : 0;
    for (int i = 0; i < keep; i++) {  // commit: shift in the accepted inputs (conv.rs:30-33)
        for (int j = 0; j < K - 2; j++) st[j] = st[j + 1];
        if (K >= 2) st[K - 2] = pend_x[(size_t)i * channels + c];
    }
    for (int j = 0; j < K - 1; j++) state[(size_t)c * (K - 1) + j] = st[j];
    const float* wc = w + (size_t)c * K;
    for (int i = 0; i < t; i++) {
        const float xn = x[(size_t)i * channels + c];
        float acc = 0.0f;
        for (int j = 0; j < K - 1; j++) acc = __fadd_rn(acc, __fmul_rn(wc[j], st[j]));
        acc = __fadd_rn(acc, __fmul_rn(wc[K - 1], xn));
        for (int j = 0; j < K - 2; j++) st[j] = st[j + 1];
        if (K >= 2) st[K - 2] = xn;
        out[(size_t)i * channels + c] = silu_f32(acc);
        if (i < max_t) pend_x[(size_t)i * channels + c] = xn;
    }
    conv_done();
}

// Gated DeltaNet recurrence of one call (t rows) for every V head p: one CTA per head, blockDim.x == 2 * dv.
// Steps:
//   1. load S (the committed state of the previous call) and apply its `keep` pending rows: S *= decay_i;
//      S += k_i (x) delta_i -- the same element operations, in the same order, as the reference's replay of the
//      accepted rows from a snapshot (spec.rs:395-415), so the state is bit-identical; store S back.
//   2. for each of the t new rows: l2norm q and k, scale q, gates, the delta rule, gated RMSNorm; record
//      (decay, k, delta) as the pending rows.  The state after the t rows is not stored: the next call commits
//      exactly the rows the accept step keeps.
// The two halves of each value column live in two different warps:
// warp w < dv/32 holds S[0, DK/2) of columns 32w .. 32w+31, warp w + dv/32 holds S[DK/2, DK) of the same
// columns, so every warp runs all 32 lanes on one half.  The k-ordered sums (kv, o) stay single left-to-right
// chains: the low-half warp sums its 64 terms from 0 and hands the partial sum through shared memory, the
// high-half warp continues from it.
// acc + sum_k S[k] * v[k] for k = 0 .. HK-1, left to right; v (shared memory, 16-byte aligned) is read four values
// at a time with the next quad requested one step ahead, so the dependent adds do not wait on each load
template <int HK>
__device__ __forceinline__ float chain_dot(const float (&S)[HK], const float* v, float acc) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float4 nx0 = v4[0], nx1 = v4[1];  // two quads ahead: a shared-memory load takes longer than four adds
#pragma unroll
    for (int q = 0; q < HK / 4; q++) {
        const float4 cur = nx0;
        nx0 = nx1;
        if (q + 2 < HK / 4) nx1 = v4[q + 2];
        acc = __fadd_rn(acc, __fmul_rn(S[4 * q], cur.x));
        acc = __fadd_rn(acc, __fmul_rn(S[4 * q + 1], cur.y));
        acc = __fadd_rn(acc, __fmul_rn(S[4 * q + 2], cur.z));
        acc = __fadd_rn(acc, __fmul_rn(S[4 * q + 3], cur.w));
    }
    return acc;
}
// acc + v[0]^2 + v[1]^2 + .. + v[N-1]^2 left to right, v in shared memory (16-byte aligned), quads two ahead
template <int N>
__device__ __forceinline__ float chain_sq(const float* v, float acc) {
    const float4* v4 = reinterpret_cast<const float4*>(v);
    float4 nx0 = v4[0], nx1 = v4[1];
#pragma unroll
    for (int q = 0; q < N / 4; q++) {
        const float4 cur = nx0;
        nx0 = nx1;
        if (q + 2 < N / 4) nx1 = v4[q + 2];
        acc = __fadd_rn(acc, __fmul_rn(cur.x, cur.x));
        acc = __fadd_rn(acc, __fmul_rn(cur.y, cur.y));
        acc = __fadd_rn(acc, __fmul_rn(cur.z, cur.z));
        acc = __fadd_rn(acc, __fmul_rn(cur.w, cur.w));
    }
    return acc;
}

template <int DK>
__global__ void __launch_bounds__(256) deltanet_halves_kernel(const DeltaArgs a) {
    constexpr int HK = DK / 2;
    constexpr int CH = 8;  // rows whose q/k norms and gates are computed together (they do not depend on S)
    const int p = blockIdx.x, t = threadIdx.x, lane = t & 31, warp = t >> 5;
    const int dv = a.dv, wph = dv / 32;  // warps per half
    const int h = warp >= wph ? 1 : 0, j = (warp - h * wph) * 32 + lane;
    const int k0 = h * HK;
    const int dk = DK;
    const int kh = p % a.n_k;
    __shared__ __align__(16) float qs_all[CH][DK], ks_all[CH][DK];
    __shared__ float gate[CH][2], nrm[CH][2];  // (decay, beta), (1/|q|, 1/|k|)
    __shared__ float red[16], outs[128], part[128], dlt[128];
    __shared__ __align__(16) float ab_part[2 * CH * 160];  // the in-kernel alpha / beta products
    __shared__ float ab_val[2][CH];
    __shared__ __align__(16) float vs_all[CH][128];  // the v rows of the chunk (dv <= 128)
    // Before griddepcontrol.wait: everything the conv kernel (launched right before) does not write -- the state
    // and the previous call's pending rows (this layer's own), the gates of the first rows (ssm_alpha/ssm_beta
    // two launches back, or their products from the normed rows, further back) and their z rows (attn_gate).
    const int nr0 = min(CH, a.t);
    if (a.w_alpha) {
        // alpha, beta of this head for the t rows: dot_f32 (dot.rs:180-198) of the F32 weight rows with the normed
        // rows -- 32-element partials left to right, then the partials chained in order plus the tail partial
        // thread jp: partial jp of both weight rows against every normed row (each weight segment read once)
        const int H = a.hid, np = (H + 31) / 32, nfull = H / 32;
        const float* wa = a.w_alpha + (size_t)p * H;
        const float* wb = a.w_beta + (size_t)p * H;
        for (int jp = t; jp < nfull; jp += blockDim.x) {
            float4 w4[2][8];
#pragma unroll
            for (int q = 0; q < 8; q++) {
                w4[0][q] = __ldg(reinterpret_cast<const float4*>(wa + jp * 32) + q);
                w4[1][q] = __ldg(reinterpret_cast<const float4*>(wb + jp * 32) + q);
            }
            for (int r = 0; r < nr0; r++) {
                float4 x4[8];
#pragma unroll
                for (int q = 0; q < 8; q++) x4[q] = __ldg(reinterpret_cast<const float4*>(a.xn + (size_t)r * H + jp * 32) + q);
#pragma unroll
                for (int which = 0; which < 2; which++) {
                    float acc = 0.0f;
#pragma unroll
                    for (int q = 0; q < 8; q++) {
                        acc = __fadd_rn(acc, __fmul_rn(w4[which][q].x, x4[q].x));
                        acc = __fadd_rn(acc, __fmul_rn(w4[which][q].y, x4[q].y));
                        acc = __fadd_rn(acc, __fmul_rn(w4[which][q].z, x4[q].z));
                        acc = __fadd_rn(acc, __fmul_rn(w4[which][q].w, x4[q].w));
                    }
                    ab_part[(which * CH + r) * 160 + jp] = acc;
                }
            }
        }
        if (t < 2 * nr0 && np > nfull) {  // the tail partial (hid % 32 elements)
            const int which = t / nr0, r = t % nr0;
            const float* wr = (which ? wb : wa);
            float acc = 0.0f;
            for (int i = nfull * 32; i < H; i++) acc = __fadd_rn(acc, __fmul_rn(wr[i], a.xn[(size_t)r * H + i]));
            ab_part[(which * CH + r) * 160 + nfull] = acc;
        }
        __syncthreads();
        if (t < 2 * nr0) {
            const int which = t / nr0, r = t % nr0;
            const float* pp = ab_part + (which * CH + r) * 160;
            float acc = 0.0f;
            int jp = 0;
            if (nfull >= 8) {  // the partials in order, their shared-memory quads loaded two ahead
                const float4* p4 = reinterpret_cast<const float4*>(pp);
                const int nq = nfull / 4;
                float4 nx0 = p4[0], nx1 = p4[1];
                for (int q = 0; q < nq; q++) {
                    const float4 cur = nx0;
                    nx0 = nx1;
                    if (q + 2 < nq) nx1 = p4[q + 2];
                    acc = __fadd_rn(acc, cur.x);
                    acc = __fadd_rn(acc, cur.y);
                    acc = __fadd_rn(acc, cur.z);
                    acc = __fadd_rn(acc, cur.w);
                }
                jp = nq * 4;
            }
            for (; jp < nfull; jp++) acc = __fadd_rn(acc, pp[jp]);
            ab_val[which][r] = __fadd_rn(acc, np > nfull ? pp[nfull] : 0.0f);
        }
        __syncthreads();
    }
    float S[HK];
    float* Sg = a.S + (size_t)p * dk * dv;
#pragma unroll
    for (int k = 0; k < HK; k++) S[k] = Sg[(size_t)(k0 + k) * dv + j];
    const int keep = a.keep_prev ? *a.keep_prev : 0;
    for (int i = 0; i < keep; i++) {  // commit the previous call's accepted rows (spec.rs:395-415 replay order)
        const float decay = a.pend_decay[(size_t)i * a.n_v + p];
        const float* kp = a.pend_k + ((size_t)i * a.n_v + p) * dk + k0;
        const float delta = a.pend_delta[((size_t)i * a.n_v + p) * dv + j];
#pragma unroll
        for (int k = 0; k < HK; k++) S[k] = __fmul_rn(S[k], decay);
#pragma unroll
        for (int k = 0; k < HK; k++) S[k] = __fadd_rn(S[k], __fmul_rn(kp[k], delta));
    }
    if (keep > 0) {
#pragma unroll
        for (int k = 0; k < HK; k++) Sg[(size_t)(k0 + k) * dv + j] = S[k];
    }
    // gates (g = a * softplus(alpha + dt_bias), decay = exp(g), beta = sigmoid(b)) of the first chunk's rows
    if (t < nr0) {
        const float al = a.w_alpha ? ab_val[0][t] : a.alpha[(size_t)t * a.n_v + p];
        const float be = a.w_alpha ? ab_val[1][t] : a.beta[(size_t)t * a.n_v + p];
        const float g = __fmul_rn(a.ssm_a[p], softplus_f32(__fadd_rn(al, a.dt_bias[p])));
        gate[t][0] = exp_f32(g);
        gate[t][1] = sigmoid_f32(be);
    }
    float zr[CH];
#pragma unroll
    for (int i = 0; i < CH; i++) zr[i] = (h == 1 && i < nr0) ? a.z[(size_t)i * a.n_v * dv + p * dv + j] : 0.0f;
    griddep_wait();
    griddep_launch();
    const float scale = __fdiv_rn(1.0f, __fsqrt_rn((float)dk));  // 1 / sqrt(dk) (gated_deltanet.rs:574)
    for (int c0 = 0; c0 < a.t; c0 += CH) {
        const int nr = min(CH, a.t - c0);
        for (int e = t; e < nr * DK; e += blockDim.x) {
            const int i = e / DK, k = e % DK;
            const float* row = a.conved + (size_t)(c0 + i) * a.conv_dim;
            qs_all[i][k] = row[kh * dk + k];
            ks_all[i][k] = row[a.kd + kh * dk + k];
        }
        for (int e = t; e < nr * dv; e += blockDim.x) {  // the v rows, off the delta's path
            const int i = e / dv, jj = e % dv;
            vs_all[i][jj] = a.conved[(size_t)(c0 + i) * a.conv_dim + 2 * a.kd + p * dv + jj];
        }
        __syncthreads();
        // l2norm (deltanet.rs:19-27, sums left to right): warp w normalises q of rows w, w + warps, .. on lane 0
        // and k on lane 16; the gates of later chunks on lane 8
        for (int i = warp; i < nr && (lane & 7) == 0; i += blockDim.x / 32) {
            if (lane == 8) {
                if (c0 == 0) continue;
                const int r = c0 + i;
                const float g = __fmul_rn(a.ssm_a[p], softplus_f32(__fadd_rn(a.alpha[(size_t)r * a.n_v + p], a.dt_bias[p])));
                gate[i][0] = exp_f32(g);
                gate[i][1] = sigmoid_f32(a.beta[(size_t)r * a.n_v + p]);
            } else if (lane != 24) {
                const float* vec = lane == 0 ? qs_all[i] : ks_all[i];
                const float ss = chain_sq<DK>(vec, 0.0f);
                nrm[i][lane == 0 ? 0 : 1] = __fdiv_rn(1.0f, __fsqrt_rn(__fadd_rn(ss, 1e-6f)));
            }
        }
        __syncthreads();
        for (int e = t; e < nr * DK; e += blockDim.x) {
            const int i = e / DK, k = e % DK;
            qs_all[i][k] = __fmul_rn(__fmul_rn(qs_all[i][k], nrm[i][0]), scale);
            ks_all[i][k] = __fmul_rn(ks_all[i][k], nrm[i][1]);
        }
        __syncthreads();
        for (int i = 0; i < nr; i++) {
            const int r = c0 + i;
            const float* qs = qs_all[i] + k0;
            const float* ks = ks_all[i] + k0;
            const float decay = gate[i][0], beta = gate[i][1];
#pragma unroll
            for (int k = 0; k < HK; k++) S[k] = __fmul_rn(S[k], decay);
            // kv = sum_k S[k] k[k]: the low half from 0, the high half from the low half's sum
            float kv = 0.0f;
            if (h == 0) {
                kv = chain_dot<HK>(S, ks, 0.0f);
                part[j] = kv;
            }
            __syncthreads();
            if (h == 1) {
                kv = chain_dot<HK>(S, ks, part[j]);
                dlt[j] = __fmul_rn(__fsub_rn(vs_all[i][j], kv), beta);
            }
            __syncthreads();
            const float delta = dlt[j];
#pragma unroll
            for (int q = 0; q < HK / 4; q++) {
                const float4 k4 = reinterpret_cast<const float4*>(ks)[q];
                S[4 * q] = __fadd_rn(S[4 * q], __fmul_rn(k4.x, delta));
                S[4 * q + 1] = __fadd_rn(S[4 * q + 1], __fmul_rn(k4.y, delta));
                S[4 * q + 2] = __fadd_rn(S[4 * q + 2], __fmul_rn(k4.z, delta));
                S[4 * q + 3] = __fadd_rn(S[4 * q + 3], __fmul_rn(k4.w, delta));
            }
            if (h == 0) part[j] = chain_dot<HK>(S, qs, 0.0f);
            if (r < a.max_t) {
                if (t == 0) a.pend_decay[(size_t)r * a.n_v + p] = decay;
                for (int k = t; k < dk; k += blockDim.x) a.pend_k[((size_t)r * a.n_v + p) * dk + k] = ks_all[i][k];
                if (h == 1) a.pend_delta[((size_t)r * a.n_v + p) * dv + j] = delta;
            }
            __syncthreads();
            float o = 0.0f;
            if (h == 1) {
                o = chain_dot<HK>(S, qs, part[j]);
                outs[j] = o;
            }
            __syncthreads();
            // gated RMSNorm over the head's dv outputs (rmsnorm.rs:36-47); the helper ends with a barrier, after
            // which outs, part, dlt and this chunk's rows may be overwritten
            const float inv = inv_rms_of(sum_squares_8lane_block(outs, dv, red), dv, a.eps);
            if (h == 1) {
                float z = 0.0f;
#pragma unroll
                for (int q = 0; q < CH; q++)
                    if (q == i) z = zr[q];
                if (c0 > 0) z = a.z[(size_t)r * a.n_v * dv + p * dv + j];
                a.heads[(size_t)r * a.n_v * dv + p * dv + j] = __fmul_rn(__fmul_rn(a.norm_w[j], __fmul_rn(o, inv)), silu_f32(z));
            }
        }
    }
    if (!a.img_q8k && !a.img_q80) return;
    // the out projection's input images of the t head rows (the quantise step of the layer, act.rs / q8k.rs)
    const int n = a.n_v * dv, nw = blockDim.x / 32;
    __threadfence();
    __syncthreads();
    if (a.img_q80) {  // this head's 32-value blocks, one warp each
        for (int e = warp; e < a.t * (dv / 32); e += nw) {
            const int r = e / (dv / 32), blk = p * (dv / 32) + e % (dv / 32);
            uint8_t* row = a.img_q80 + (size_t)r * (n / 32) * Q80_IMG_BYTES;
            q80_quantize_to_image(__ldcg(a.heads + (size_t)r * n + blk * 32 + lane), row + (size_t)blk * 32,
                                  row + (size_t)(n / 32) * 32 + (size_t)blk * 8);
        }
    }
    if (a.img_q8k) {
        const int hpb = 256 / dv, blk = p / hpb;
        __shared__ unsigned s_prev;
        if (t == 0) s_prev = atomicAdd(&a.blk_cnt[blk], 1u);
        __syncthreads();
        if (s_prev == (unsigned)(hpb - 1)) {  // the block's last head: quantise its rows
            __threadfence();
            for (int r = warp; r < a.t; r += nw) {
                const float4* hb = reinterpret_cast<const float4*>(a.heads + (size_t)r * n + (size_t)blk * 256 + lane * 8);
                const float4 u0 = __ldcg(hb), u1 = __ldcg(hb + 1);
                const float v[8] = {u0.x, u0.y, u0.z, u0.w, u1.x, u1.y, u1.z, u1.w};
                q8k_quantize_to_image(v, a.img_q8k + ((size_t)r * (n / 256) + blk) * Q8K_IMG_BYTES);
            }
            if (t == 0) a.blk_cnt[blk] = 0u;  // ready for the next call
        }
    }
}

// Per (row i, head): RMSNorm of q (heads 0..nh-1) or k (heads nh..nh+nkv-1) with the 8-lane order, then
// rotate-half RoPE on the first rope_dim dims (rope.rs:31-45); q written to q_out with its gate copied to
// gate_out; k and v appended to the cache at position pos0 + i (gqa_attention.rs:343-362).
__global__ void qk_norm_rope_kernel(const QkArgs a) {
    extern __shared__ __align__(16) float sm[];
    const int i = blockIdx.y, h = blockIdx.x;
    const int hd = a.head_dim, rd = a.rope_dim, half = rd / 2;
    const int pos = *a.pos + i;
    float* xs = sm;
    float* red = sm + hd;
    const bool is_q = h < a.n_head;
    const float* src = is_q ? a.qg + (size_t)i * 2 * a.n_head * hd + (size_t)h * 2 * hd
                            : a.k + (size_t)i * a.n_kv * hd + (size_t)(h - a.n_head) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) xs[d] = src[d];
    __syncthreads();
    const float inv = inv_rms_of(sum_squares_8lane_block(xs, hd, red), hd, a.eps);
    const float* nw = is_q ? a.q_norm : a.k_norm;
    const float* cs = a.cos + (size_t)pos * rd;
    const float* sn = a.sin + (size_t)pos * rd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) xs[d] = __fmul_rn(__fmul_rn(xs[d], inv), nw[d]);
    __syncthreads();
    float* dst;
    if (is_q) dst = a.q_out + (size_t)i * a.n_head * hd + (size_t)h * hd;
    else dst = a.k_cache + ((size_t)pos * a.n_kv + (h - a.n_head)) * hd;
    for (int d = threadIdx.x; d < hd; d += blockDim.x) {
        float val = xs[d];
        if (d < half) val = __fsub_rn(__fmul_rn(xs[d], cs[d]), __fmul_rn(xs[d + half], sn[d]));
        else if (d < rd) val = __fadd_rn(__fmul_rn(xs[d], cs[d]), __fmul_rn(xs[d - half], sn[d]));
        dst[d] = val;
    }
    if (is_q) {
        for (int d = threadIdx.x; d < hd; d += blockDim.x)
            a.gate_out[(size_t)i * a.n_head * hd + (size_t)h * hd + d] = src[hd + d];
    } else {
        const float* vsrc = a.v + (size_t)i * a.n_kv * hd + (size_t)(h - a.n_head) * hd;
        float* vdst = a.v_cache + ((size_t)pos * a.n_kv + (h - a.n_head)) * hd;
        for (int d = threadIdx.x; d < hd; d += blockDim.x) vdst[d] = vsrc[d];
    }
}

// Attention of row i and query head h (gqa_attention.rs:376-409): scores s[t] = (sum_d q[d] k_t[d]) * scaling
// over the cache positions 0..pos0+i (sum left to right over d), softmax (max, exp, 8-lane sum, divide),
// out[d] = sum_t p[t] v_t[d] (left to right over t), times sigmoid(gate) -- in three kernels.
// Scores: a CTA takes up to 8 (query head, row) pairs that read the same kv head (pair p = query head
// kvh * group + p % group of row p / group) and strides over 256-position chunks of the cache; each warp stages the
// keys of 32 positions 32 dims at a time in shared memory (coalesced loads; rows padded to 36 floats so the
// 16-byte reads of 8 lanes hit 32 distinct banks) and lane l continues the left-to-right dots of position l for
// all the pairs -- every score is the reference's sequential sum, and a key is read once per 8 pairs.
constexpr int ATT_KCH = 32;      // dims staged per pass
constexpr int ATT_SGRID = 32;    // CTAs per (kv head, pair group) over the positions
// ATT_PAIRS: (query head, row) pairs per CTA -- 8 for long caches (a key is read once per 8 pairs), 2 for short
// ones (4x the CTAs, so a short context still spreads over the SMs).  NW warps, 32 positions each, per chunk of
// the cache.  (Every pair of a kv head in one 4-warp CTA, so each key is read once, measured slower at 8K
// positions: 66 against 39 us per call, for want of warps.)
template <int ATT_PAIRS, int NW>
__global__ void __launch_bounds__(32 * NW) attn_scores_kernel(const AttnArgs a, int rows) {
    __shared__ __align__(16) float kt[NW][32][ATT_KCH + 4];
    __shared__ __align__(16) float qs[ATT_PAIRS][256];
    const int hd = a.head_dim, group = a.n_head / a.n_kv, npairs = group * rows;
    const int kvh = blockIdx.y, pg = blockIdx.z;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int pos = *a.pos;
    const int np = min(ATT_PAIRS, npairs - pg * ATT_PAIRS);
    for (int e = threadIdx.x; e < np * hd; e += blockDim.x) {
        const int j = e / hd, d = e % hd;
        const int pi = pg * ATT_PAIRS + j, h = kvh * group + pi % group, i = pi / group;
        qs[j][d] = a.q[(size_t)i * a.n_head * hd + (size_t)h * hd + d];
    }
    __syncthreads();
    const int len = pos + (pg * ATT_PAIRS + np - 1) / group + 1;  // the group's longest row (rows ascend with the pair)
    const size_t rstride = (size_t)a.n_kv * hd;
    for (int c = blockIdx.x; c * (32 * NW) < len; c += gridDim.x) {
        const int p0 = c * (32 * NW) + warp * 32;
        if (p0 >= len) continue;  // warp-uniform
        float acc[ATT_PAIRS];
#pragma unroll
        for (int j = 0; j < ATT_PAIRS; j++) acc[j] = 0.0f;
        for (int d0 = 0; d0 < hd; d0 += ATT_KCH) {
            // 32 positions x 32 dims: lane l loads 16-byte piece (l % 8) of positions l / 8 + 4j
#pragma unroll
            for (int j = 0; j < 8; j++) {
                const int pp = lane / 8 + 4 * j, t = p0 + pp;
                if (t < len) {
                    const float4 v = *reinterpret_cast<const float4*>(a.k_cache + (size_t)t * rstride + (size_t)kvh * hd + d0 + (lane % 8) * 4);
                    *reinterpret_cast<float4*>(&kt[warp][pp][(lane % 8) * 4]) = v;
                }
            }
            __syncwarp();
#pragma unroll
            for (int d = 0; d < ATT_KCH; d += 4) {
                const float4 k4 = *reinterpret_cast<const float4*>(&kt[warp][lane][d]);
#pragma unroll
                for (int j = 0; j < ATT_PAIRS; j++) {
                    const float4 q4 = *reinterpret_cast<const float4*>(&qs[j][d0 + d]);
                    acc[j] = __fadd_rn(acc[j], __fmul_rn(q4.x, k4.x));
                    acc[j] = __fadd_rn(acc[j], __fmul_rn(q4.y, k4.y));
                    acc[j] = __fadd_rn(acc[j], __fmul_rn(q4.z, k4.z));
                    acc[j] = __fadd_rn(acc[j], __fmul_rn(q4.w, k4.w));
                }
            }
            __syncwarp();
        }
        const int t = p0 + lane;
#pragma unroll
        for (int j = 0; j < ATT_PAIRS; j++) {
            const int pi = pg * ATT_PAIRS + j, i = pi / group, h = kvh * group + pi % group;
            if (j < np && t < pos + i + 1)
                a.scores[((size_t)i * a.n_head + h) * ((a.max_len + 3) & ~3) + t] = __fmul_rn(acc[j], a.scaling);
        }
    }
}

// Softmax of each (head, row) score row in place (softmax.rs:22-50): m = max, e = exp(x - m), the 8-lane sum
// (lane l adds e[l], e[l+8], ... left to right; reduce8; the tail), p = e / sum.  One CTA of 256 per row.  The
// exps are kept in shared memory (`es`, when the launch gave it room for the row), so the 8 serial chains read
// them at shared-memory latency rather than from L2.
__global__ void __launch_bounds__(256) attn_softmax_kernel(const AttnArgs a, int staged) {
    extern __shared__ __align__(16) float es_dyn[];
    __shared__ float red[16];
    const int h = blockIdx.x, i = blockIdx.y, tid = threadIdx.x, lane = tid & 31;
    const int len = *a.pos + i + 1;
    float* p = a.scores + ((size_t)i * a.n_head + h) * ((a.max_len + 3) & ~3);
    float* e = staged ? es_dyn : p;
    float m = -INFINITY;
    for (int t = tid; t < len; t += 256) m = fmaxf(m, p[t]);
    for (int off = 16; off > 0; off >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, off));
    if (lane == 0) red[tid >> 5] = m;
    __syncthreads();
    if (tid == 0) {
        float mm = red[0];
        for (int w = 1; w < 8; w++) mm = fmaxf(mm, red[w]);
        red[15] = mm;
    }
    __syncthreads();
    m = red[15];
    for (int t = tid; t < len; t += 256) e[t] = exp_f32(__fsub_rn(p[t], m));
    __syncthreads();  // this CTA's writes are visible to its own threads after the barrier
    const int n8 = len / 8 * 8;
    if (tid < 8) {
        float acc = 0.0f;
        for (int t = tid; t < n8; t += 8) acc = __fadd_rn(acc, e[t]);
        red[tid] = acc;
    }
    __syncthreads();
    if (tid == 0) {
        float sum = reduce8(red);
        for (int t = n8; t < len; t++) sum = __fadd_rn(sum, e[t]);
        red[8] = sum;
    }
    __syncthreads();
    const float ssum = red[8];
    for (int t = tid; t < len; t += 256) p[t] = __fdiv_rn(e[t], ssum);
}

// The value sum: one CTA per (32 output dims, kv head, group of ATT_VP (query head, row) pairs reading that kv
// head), warp j = pair j, lane = output dim: out[d] = sum_t p[t] * v_t[d] left to right over t, times
// sigmoid(gate) (gqa_attention.rs:376-409).  The value rows (32 dims) and the pairs' probabilities stream through
// a 4-stage ring of cp.async copies, 64 positions per stage, so a value row is read once for the group's 4 pairs
// (12 pairs per CTA measured slower at 8K positions: 110 against 95 us per call).
constexpr int ATT_VT = 64, ATT_VS = 4;

__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"((uint32_t)__cvta_generic_to_shared(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_stages() { asm volatile("cp.async.wait_group %0;" ::"n"(ATT_VS - 2) : "memory"); }

template <int ATT_VP>
__global__ void __launch_bounds__(32 * ATT_VP) attn_pv_kernel(const AttnArgs a, int rows) {
    __shared__ __align__(16) float vs[ATT_VS][ATT_VT][32];
    __shared__ __align__(16) float ps[ATT_VS][ATT_VP][ATT_VT];
    const int dc = blockIdx.x, kvh = blockIdx.y, pg = blockIdx.z, hd = a.head_dim;
    const int group = a.n_head / a.n_kv, npairs = group * rows;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int np = min(ATT_VP, npairs - pg * ATT_VP);
    const int pos = *a.pos;
    const int sld = (a.max_len + 3) & ~3;
    const int pw = pg * ATT_VP + min(warp, np - 1);  // this warp's pair
    const int h = kvh * group + pw % group, i = pw / group;
    const int len = pos + i + 1;
    const int lenmax = pos + (pg * ATT_VP + np - 1) / group + 1;  // the group's longest row (rows ascend)
    const size_t rstride = (size_t)a.n_kv * hd;
    const float* vbase = a.v_cache + (size_t)kvh * hd + dc * 32;
    const int ntiles = (lenmax + ATT_VT - 1) / ATT_VT;
    auto issue = [&](int k) {
        const int st = k % ATT_VS;
        for (int e = tid; e < ATT_VT * 8; e += 32 * ATT_VP) {  // 64 positions x 8 pieces of 16 bytes
            const int tt = e / 8, cc = e % 8, t = k * ATT_VT + tt;
            if (t < lenmax) cp_async16(&vs[st][tt][cc * 4], vbase + (size_t)t * rstride + cc * 4);
        }
        for (int e = tid; e < np * (ATT_VT / 4); e += 32 * ATT_VP) {  // the pairs' probabilities, 16 per row
            const int j = e / (ATT_VT / 4), cc = e % (ATT_VT / 4), t = k * ATT_VT + cc * 4;
            const int pj = pg * ATT_VP + j, hj = kvh * group + pj % group, ij = pj / group;
            if (t < pos + ij + 1) cp_async16(&ps[st][j][cc * 4], a.scores + ((size_t)ij * a.n_head + hj) * sld + t);
        }
    };
#pragma unroll
    for (int s = 0; s < ATT_VS - 1; s++) {
        if (s < ntiles) issue(s);
        cp_async_commit();
    }
    float o = 0.0f;
    for (int k = 0; k < ntiles; k++) {
        cp_async_wait_stages();
        __syncthreads();  // tile k landed for every thread; every thread is done with tile k - 1
        if (k + ATT_VS - 1 < ntiles) issue(k + ATT_VS - 1);
        cp_async_commit();
        const int st = k % ATT_VS;
        const int tn = min(ATT_VT, len - k * ATT_VT);  // warp-uniform: the pair's own length
        if (tn == ATT_VT) {
#pragma unroll
            for (int tt = 0; tt < ATT_VT; tt++) o = __fadd_rn(o, __fmul_rn(ps[st][warp][tt], vs[st][tt][lane]));
        } else {
            for (int tt = 0; tt < tn; tt++) o = __fadd_rn(o, __fmul_rn(ps[st][warp][tt], vs[st][tt][lane]));
        }
    }
    asm volatile("cp.async.wait_all;" ::: "memory");
    if (warp < np) {
        const int d = dc * 32 + lane;
        const float g = a.gate[(size_t)i * a.n_head * hd + (size_t)h * hd + d];
        a.out[(size_t)i * a.n_head * hd + (size_t)h * hd + d] = __fmul_rn(o, sigmoid_f32(g));
    }
}

// out[row] = the first index of the maximum (model.rs:505-513: best = x[0], then a strict > scan; NaN is never
// taken, and a NaN x[0] is kept).  Grid (chunks, rows): each CTA reduces ARGMAX_CHUNK values to its first
// maximum (ties -> smaller index; NaN skipped), writes it, and the last CTA of the row to finish combines the
// chunk results in chunk order with the strict > rule and resets the row's counter.
constexpr int ARGMAX_CHUNK = 8192;

// With `pairs` (a tensor-parallel rank's vocabulary slice starting at index `base`): the row's result is
// written as {float value, int index + base} at pairs + 16 * row, and the seed x[0] is used only when `seed`
// (rank 0); otherwise the slice's own first maximum (index -1 when it holds only NaN).
__global__ void __launch_bounds__(256) argmax_kernel(const float* __restrict__ x, int n, int32_t* __restrict__ out,
                                                     float* __restrict__ pval, int* __restrict__ pidx,
                                                     unsigned* __restrict__ counter, uint8_t* __restrict__ pairs, int base,
                                                     int seed) {
    griddep_wait();
    griddep_launch();
    const int row = blockIdx.y, chunks = gridDim.x, c = blockIdx.x;
    const float* r = x + (size_t)row * n;
    const int lo = c * ARGMAX_CHUNK, hi = min(n, lo + ARGMAX_CHUNK);
    float best = -INFINITY;
    int bi = -1;
    for (int i = lo + threadIdx.x; i < hi; i += blockDim.x) {
        const float v = r[i];
        if (v > best || (bi < 0 && v == best)) best = v, bi = i;  // the first -inf counts as a candidate too
    }
    for (int off = 16; off > 0; off >>= 1) {
        const float ov = __shfl_xor_sync(0xffffffffu, best, off);
        const int oi = __shfl_xor_sync(0xffffffffu, bi, off);
        if (oi >= 0 && (bi < 0 || ov > best || (ov == best && oi < bi))) best = ov, bi = oi;
    }
    __shared__ float bv[8];
    __shared__ int bx[8];
    __shared__ bool last;
    if ((threadIdx.x & 31) == 0) bv[threadIdx.x >> 5] = best, bx[threadIdx.x >> 5] = bi;
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < (int)(blockDim.x >> 5); w++)
            if (bx[w] >= 0 && (bi < 0 || bv[w] > best || (bv[w] == best && bx[w] < bi))) best = bv[w], bi = bx[w];
        pval[(size_t)row * chunks + c] = best;
        pidx[(size_t)row * chunks + c] = bi;
        __threadfence();
        last = atomicAdd(&counter[row], 1u) == (unsigned)chunks - 1;
    }
    __syncthreads();
    if (last && threadIdx.x == 0) {
        __threadfence();
        float g = seed ? r[0] : -INFINITY;  // the reference's seed: x[0] at index 0
        int gi = seed ? 0 : -1;
        for (int k = 0; k < chunks; k++) {
            const volatile float* pv = pval + (size_t)row * chunks;
            const volatile int* pi = pidx + (size_t)row * chunks;
            if (pi[k] >= 0 && (gi < 0 || pv[k] > g)) g = pv[k], gi = pi[k];
        }
        if (pairs) {
            *reinterpret_cast<float*>(pairs + 16 * (size_t)row) = g;
            *reinterpret_cast<int*>(pairs + 16 * (size_t)row + 4) = gi < 0 ? -1 : gi + base;
        } else {
            out[row] = gi;
        }
        counter[row] = 0u;
    }
}

// ------------------------------------------------------------------------------------------- launchers

namespace {
// Launch with the programmatic-dependent attribute: the kernel calls griddepcontrol.wait before touching
// anything its predecessor writes, and triggers its own dependents at once.
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t s, Args... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}
}  // namespace

cudaError_t launch_resid_norm_quant(const float* a, const float* b, float* h_out, const float* w, float eps, int n, int rows,
                                    float* y_out, uint8_t* img_out, uint8_t* q80_out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    if (n % 256) return cudaErrorInvalidValue;
    if (h_out && (h_out == a || h_out == b)) return cudaErrorInvalidValue;
    const size_t smem = (size_t)(n + 16 + 256) * sizeof(float);
    if (n % 256 || smem > 200 * 1024) return cudaErrorInvalidValue;
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(resid_norm_quant_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    return launch_pdl(resid_norm_quant_kernel, dim3(n / 256, rows), dim3(256), smem, s, a, b, h_out, w, eps, n, y_out, img_out,
                      q80_out);
}

cudaError_t launch_rmsnorm_rows(const float* x, int x_ld, const float* w, float eps, int n, int rows, float* y, int y_ld,
                               cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const size_t smem = (size_t)(n + 16) * sizeof(float);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(rmsnorm_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    rmsnorm_rows_kernel<<<rows, 512, smem, s>>>(x, x_ld, w, eps, n, y, y_ld);
    return cudaGetLastError();
}

cudaError_t launch_swiglu_quant(const float* g, const float* u, int n, int rows, float* h_out, uint8_t* img_out,
                                uint8_t* q80_out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    if (n % 256) return cudaErrorInvalidValue;
    return launch_pdl(swiglu_quant_kernel, dim3(n / 256, rows), dim3(256), 0, s, g, u, n, h_out, img_out, q80_out);
}

cudaError_t launch_quant_rows(const float* x, int n, int rows, uint8_t* img_out, uint8_t* q80_out, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    if (n % 256) return cudaErrorInvalidValue;
    return launch_pdl(quant_rows_kernel, dim3(n / 256, rows), dim3(256), 0, s, x, n, img_out, q80_out);
}

cudaError_t launch_conv_step(float* state, const float* w, int K, int channels, const float* x, int t, float* out,
                             float* pend_x, const int* keep_prev, int max_t, cudaStream_t s) {
    const cudaError_t e = launch_pdl(conv_step_kernel, dim3((channels + 255) / 256), dim3(256), 0, s, state, w, K, channels, x, t,
                                     out, pend_x, keep_prev, max_t);
    return e == cudaSuccess ? cudaGetLastError() : e;
}

cudaError_t launch_deltanet_heads(const DeltaArgs& a, cudaStream_t s) {
    if (!deltanet_dims_supported(a.dk, a.dv)) return cudaErrorInvalidValue;
    cudaError_t e = a.dk == 128 ? launch_pdl(deltanet_halves_kernel<128>, dim3(a.n_v), dim3(2 * a.dv), 0, s, a)
                                : launch_pdl(deltanet_halves_kernel<64>, dim3(a.n_v), dim3(2 * a.dv), 0, s, a);
    return e == cudaSuccess ? cudaGetLastError() : e;
}

cudaError_t launch_qk_norm_rope(const QkArgs& a, int t, cudaStream_t s) {
    const dim3 grid(a.n_head + a.n_kv, t);
    const size_t smem = (size_t)(a.head_dim + 16) * sizeof(float);
    qk_norm_rope_kernel<<<grid, 128, smem, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_attention(const AttnArgs& a, int t, cudaStream_t s) {
    if (!a.scores || !attention_dims_supported(a.head_dim)) return cudaErrorInvalidValue;
    const int group = a.n_head / a.n_kv, npairs = group * t;
    const bool lng = a.max_len > 2048;  // a long cache: read every key and value row once per call
    if (lng) {
        const dim3 sgrid(std::min((a.max_len + 255) / 256, ATT_SGRID), a.n_kv, (npairs + 7) / 8);
        attn_scores_kernel<8, 8><<<sgrid, 256, 0, s>>>(a, t);
    } else {
        const dim3 sgrid(std::min((a.max_len + 255) / 256, ATT_SGRID), a.n_kv, (npairs + 1) / 2);
        attn_scores_kernel<2, 8><<<sgrid, 256, 0, s>>>(a, t);
    }
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    // the exps of a score row in shared memory when it fits (up to 48K positions)
    const size_t row_bytes = (size_t)((a.max_len + 3) & ~3) * sizeof(float);
    const bool staged = row_bytes <= 192 * 1024;
    static size_t sm_attr = 48 * 1024;  // raised once, before any graph capture reaches a longer cache
    if (staged && row_bytes > sm_attr) {
        e = cudaFuncSetAttribute(attn_softmax_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)row_bytes);
        if (e != cudaSuccess) return e;
        sm_attr = row_bytes;
    }
    attn_softmax_kernel<<<dim3(a.n_head, t), 256, staged ? row_bytes : 0, s>>>(a, staged ? 1 : 0);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
    attn_pv_kernel<4><<<dim3(a.head_dim / 32, a.n_kv, (npairs + 3) / 4), 32 * 4, 0, s>>>(a, t);
    return cudaGetLastError();
}

size_t argmax_scratch_bytes(int n, int rows) {
    const int chunks = (n + ARGMAX_CHUNK - 1) / ARGMAX_CHUNK;
    return (size_t)rows * chunks * 8 + (size_t)rows * 4 + 64;
}

cudaError_t launch_argmax(const float* x, int n, int rows, int32_t* out, void* scratch, cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const int chunks = (n + ARGMAX_CHUNK - 1) / ARGMAX_CHUNK;
    // scratch: counters (zero at rest: every launch leaves them zero), then the per-chunk values and indices
    unsigned* counter = (unsigned*)scratch;
    float* pval = (float*)((uint8_t*)scratch + ((size_t)rows * 4 + 15) / 16 * 16);
    int* pidx = (int*)(pval + (size_t)rows * chunks);
    return launch_pdl(argmax_kernel, dim3(chunks, rows), dim3(256), 0, s, x, n, out, pval, pidx, counter, (uint8_t*)nullptr, 0, 1);
}

cudaError_t launch_argmax_pairs(const float* x, int n, int rows, uint8_t* pairs, int base, bool seed, void* scratch,
                                cudaStream_t s) {
    if (rows == 0) return cudaSuccess;
    const int chunks = (n + ARGMAX_CHUNK - 1) / ARGMAX_CHUNK;
    unsigned* counter = (unsigned*)scratch;
    float* pval = (float*)((uint8_t*)scratch + ((size_t)rows * 4 + 15) / 16 * 16);
    int* pidx = (int*)(pval + (size_t)rows * chunks);
    return launch_pdl(argmax_kernel, dim3(chunks, rows), dim3(256), 0, s, x, n, (int32_t*)nullptr, pval, pidx, counter, pairs,
                      base, seed ? 1 : 0);
}

}  // namespace qdec
