// K-quant GEMV with bulk-copy staging (Q4_K, Q5_K, and Q6_K in the split layout) x Q8_K activations,
// bit-exact with crates/core/src/kernels/kdot.rs:37-141 and its blocked form :176-333.
//
// Work split.  LPR lanes share one weight row; each owns 8/LPR of the reference's eight i32 lanes (lane g =
// positions 4g..4g+3 of every 32-element sub-block) and the matching min lanes, walks the row's super-blocks in
// order and keeps its f32 accumulators in registers -- the reference's "per lane, sequential over
// super-blocks" chain, with no cross-lane traffic until one final reduce8 + reduce4 in the reference's order.
// LPR is chosen per matrix so that short matrices (5120 output rows) still give every SM enough warps.
//
// Data movement.  A warp owns 32/LPR rows.  Per stage it copies SC = LPR super-blocks of each of its rows from
// HBM into that row's shared-memory slot with one cp.async.bulk per row (completion on the stage's mbarrier);
// STAGES stages are in flight per warp.  Slot strides are odd multiples of 16 bytes, so lanes of different rows
// read distinct banks.  The activation columns are staged once per CTA; all lanes of a warp walk the same
// super-block together, so their activation reads hit at most LPR distinct 32-byte runs.
//
// Q6_K split layout: the engine stores each Q6_K super-block as its 208 bytes [ql 128 | qh 64 | scales 16]
// (16-byte aligned) followed, after all blocks of the tensor, by the f16 scales d (2 bytes per block) -- the
// same total bytes as ggml's 210-byte blocks, repacked once at load (repack_q6k_kernel).
//
// Waits are bounded: a wait that gives up records a code in the library's device error word and the warp
// leaves its row loop; the host reports QDEC_ETIMEOUT.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

__device__ unsigned int g_kernel_error = 0;  // first timeout code recorded by a bounded wait

namespace {

constexpr int V4_WARPS = 4;     // warps per CTA
constexpr int V4_STAGES = 4;    // chunks in flight per warp
constexpr uint32_t WAIT_LIMIT = 1u << 26;

template <int TYPE>
struct BlkBytes {
    static constexpr int value = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 208;  // Q6_K: split layout
};

template <int TYPE, int LPR>
struct V4Geo {
    static constexpr int BB = BlkBytes<TYPE>::value;
    static constexpr int SC = LPR;                                          // super-blocks per chunk
    static constexpr int RW = 32 / LPR;                                     // rows per warp
    static constexpr int CHUNK = SC * BB;
    static constexpr int SLOT = ((CHUNK / 16) % 2 == 0) ? CHUNK + 16 : CHUNK;  // odd number of 16-byte units
    static constexpr int STAGE = RW * SLOT;
    static constexpr size_t BAR_BYTES = ((size_t)V4_WARPS * V4_STAGES * 8 + 127) / 128 * 128;
    static constexpr size_t FIXED = BAR_BYTES + (size_t)V4_WARPS * V4_STAGES * STAGE;
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity, unsigned code) {
    for (uint32_t it = 0; it < WAIT_LIMIT; it++)
        if (mbar_try_wait(bar, parity)) return true;
    atomicCAS(&g_kernel_error, 0u, code);
    return false;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
__device__ __forceinline__ uint32_t prmt_byte(uint32_t w, int i) { return __byte_perm(w, 0u, 0x4440 | i); }

// Activation image: per (column, super-block): 256 code bytes in block order, f32 d, and 16 int32 sums
// (q8s[s] = bsums[2s] + bsums[2s+1] in [0..8) for Q4_K/Q5_K; the 16 bsums for Q6_K).
struct ActGeo {
    static __host__ __device__ size_t off_d(int nc, int nb) { return (size_t)nc * nb * 256; }
    static __host__ __device__ size_t off_s(int nc, int nb) { return (off_d(nc, nb) + (size_t)nc * nb * 4 + 15) & ~(size_t)15; }
    static __host__ __device__ size_t bytes(int nc, int nb) { return off_s(nc, nb) + (size_t)nc * nb * 64; }
};

template <bool Q6>
__device__ void stage_act(const uint8_t* __restrict__ act, int nc, int nb, uint8_t* sm) {
    uint32_t* xq = reinterpret_cast<uint32_t*>(sm);
    float* xd = reinterpret_cast<float*>(sm + ActGeo::off_d(nc, nb));
    int* xs = reinterpret_cast<int*>(sm + ActGeo::off_s(nc, nb));
    for (int i = threadIdx.x; i < nc * nb * 73; i += blockDim.x) {
        const int blk = i / 73, wi = i % 73;
        const uint32_t v = reinterpret_cast<const uint32_t*>(act + (size_t)blk * Q8K_BLOCK_BYTES)[wi];
        if (wi == 0) {
            xd[blk] = __uint_as_float(v);
        } else if (wi <= 64) {
            xq[(size_t)blk * 64 + (wi - 1)] = v;
        } else {
            const int g2 = wi - 65, lo = (int)(int16_t)(v & 0xffff), hi = (int)(int16_t)(v >> 16);
            if (Q6) {
                xs[blk * 16 + 2 * g2] = lo;
                xs[blk * 16 + 2 * g2 + 1] = hi;
            } else {
                xs[blk * 16 + g2] = (int)(int16_t)(lo + hi);  // q8k.rs:185-193
            }
        }
    }
}

template <int N>
__device__ __forceinline__ void lds_words(const uint8_t* p, uint32_t (&w)[N]) {
    if constexpr (N == 8) {
        const uint4 a = *reinterpret_cast<const uint4*>(p), b = *reinterpret_cast<const uint4*>(p + 16);
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w, w[4] = b.x, w[5] = b.y, w[6] = b.z, w[7] = b.w;
    } else if constexpr (N == 4) {
        const uint4 a = *reinterpret_cast<const uint4*>(p);
        w[0] = a.x, w[1] = a.y, w[2] = a.z, w[3] = a.w;
    } else if constexpr (N == 2) {
        const uint2 a = *reinterpret_cast<const uint2*>(p);
        w[0] = a.x, w[1] = a.y;
    } else {
        w[0] = *reinterpret_cast<const uint32_t*>(p);
    }
}

template <int TYPE, int NC, int LPR>
__global__ void __launch_bounds__(V4_WARPS * 32)
kq_gemv_v4_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ dsplit, int rows, int nb,
                  const uint8_t* __restrict__ act, float* __restrict__ y) {
    using G = V4Geo<TYPE, LPR>;
    constexpr int GL = 8 / LPR;  // reference lanes per thread
    constexpr bool Q6 = TYPE == T_Q6_K;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rlane = lane / LPR, part = lane % LPR, g0 = part * GL;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    uint8_t* wst = smem + G::BAR_BYTES;
    uint8_t* asm_ = wst + (size_t)V4_WARPS * V4_STAGES * G::STAGE;
    if (threadIdx.x < V4_WARPS * V4_STAGES) mbar_init(&bars[threadIdx.x], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    stage_act<Q6>(act, NC, nb, asm_);
    __syncthreads();
    const uint8_t* xq = asm_;
    const float* xd = reinterpret_cast<const float*>(asm_ + ActGeo::off_d(NC, nb));
    const int* xs = reinterpret_cast<const int*>(asm_ + ActGeo::off_s(NC, nb));
    uint64_t* wbar = bars + warp * V4_STAGES;
    uint8_t* wbuf = wst + (size_t)warp * V4_STAGES * G::STAGE;
    const size_t row_bytes = (size_t)nb * G::BB;
    const int nchunks = (nb + G::SC - 1) / G::SC;
    uint32_t phase_bits = 0;
    bool alive = true;

    const int groups = (rows + G::RW - 1) / G::RW;
    for (int grp = blockIdx.x * V4_WARPS + warp; grp < groups && alive; grp += gridDim.x * V4_WARPS) {
        const int row = grp * G::RW + rlane;
        const int crow = min(row, rows - 1);
        const uint8_t* wrow = w + (size_t)crow * row_bytes;
        auto issue = [&](int c) {
            const int st = c % V4_STAGES, sb0 = c * G::SC;
            const uint32_t bytes = (uint32_t)(min(G::SC, nb - sb0) * G::BB);
            if (lane == 0) mbar_expect_tx(&wbar[st], G::RW * bytes);
            __syncwarp();
            if (part == 0) bulk_g2s(wbuf + (size_t)st * G::STAGE + rlane * G::SLOT, wrow + (size_t)sb0 * G::BB, bytes, &wbar[st]);
        };
        for (int c = 0; c < min(V4_STAGES, nchunks); c++) issue(c);

        float acc[NC][GL], accm[NC][4];
#pragma unroll
        for (int n = 0; n < NC; n++) {
#pragma unroll
            for (int g = 0; g < GL; g++) acc[n][g] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) accm[n][i] = 0.0f;
        }
        for (int c = 0; c < nchunks; c++) {
            const int st = c % V4_STAGES;
            if (!mbar_wait_bounded(&wbar[st], (phase_bits >> st) & 1u, 0x200u | (unsigned)TYPE)) {
                alive = false;
                break;
            }
            phase_bits ^= 1u << st;
            const uint8_t* slot = wbuf + (size_t)st * G::STAGE + rlane * G::SLOT;
            const int nsb = min(G::SC, nb - c * G::SC);
            for (int j = 0; j < nsb; j++) {
                const int sb = c * G::SC + j;
                const uint8_t* blk = slot + j * G::BB;
                int sumi[NC][GL];
#pragma unroll
                for (int n = 0; n < NC; n++)
#pragma unroll
                    for (int g = 0; g < GL; g++) sumi[n][g] = 0;
                if constexpr (!Q6) {
                    const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
                    const uint32_t sc03 = hdr.y & 0x3F3F3F3Fu;
                    const uint32_t sc47 = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
                    const float dw = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
                    const float dminw = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
                    uint32_t qh[GL];
                    if constexpr (TYPE == T_Q5_K) lds_words<GL>(blk + 16 + 4 * g0, qh);
#pragma unroll
                    for (int p = 0; p < 4; p++) {  // sub-blocks 2p (low nibbles), 2p+1 (high nibbles)
                        constexpr int QO = TYPE == T_Q4_K ? 16 : 48;
                        uint32_t raw[GL];
                        lds_words<GL>(blk + QO + 32 * p + 4 * g0, raw);
                        const int scA = (int)prmt_byte(p < 2 ? sc03 : sc47, (2 * p) & 3);
                        const int scB = (int)prmt_byte(p < 2 ? sc03 : sc47, (2 * p + 1) & 3);
                        uint32_t lo[GL], hi[GL];
#pragma unroll
                        for (int g = 0; g < GL; g++) {
                            lo[g] = raw[g] & 0x0F0F0F0Fu;
                            hi[g] = (raw[g] >> 4) & 0x0F0F0F0Fu;
                            if constexpr (TYPE == T_Q5_K) {
                                lo[g] |= ((qh[g] >> (2 * p)) & 0x01010101u) << 4;
                                hi[g] |= ((qh[g] >> (2 * p + 1)) & 0x01010101u) << 4;
                            }
                        }
#pragma unroll
                        for (int n = 0; n < NC; n++) {
                            const uint8_t* xb = xq + ((size_t)n * nb + sb) * 256;
                            uint32_t xA[GL], xB[GL];
                            lds_words<GL>(xb + (2 * p) * 32 + 4 * g0, xA);
                            lds_words<GL>(xb + (2 * p + 1) * 32 + 4 * g0, xB);
#pragma unroll
                            for (int g = 0; g < GL; g++) {
                                sumi[n][g] += scA * __dp4a((int)lo[g], (int)xA[g], 0);
                                sumi[n][g] += scB * __dp4a((int)hi[g], (int)xB[g], 0);
                            }
                        }
                    }
                    const uint32_t m03 = hdr.z & 0x3F3F3F3Fu;
                    const uint32_t m47 = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const float dx = xd[n * nb + sb];
                        const float d = __fmul_rn(dx, dw);
#pragma unroll
                        for (int g = 0; g < GL; g++) acc[n][g] = __fadd_rn(acc[n][g], __fmul_rn(d, (float)sumi[n][g]));
                        const float dmin = __fmul_rn(-dx, dminw);
                        const int* q8 = xs + ((size_t)n * nb + sb) * 16;
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            if ((i * LPR) / 4 != part) continue;  // min lane i belongs to this part
                            const uint32_t mw = i < 2 ? m03 : m47;
                            const int prod = (int)prmt_byte(mw, (2 * i) & 3) * q8[2 * i] + (int)prmt_byte(mw, (2 * i + 1) & 3) * q8[2 * i + 1];
                            accm[n][i] = __fadd_rn(accm[n][i], __fmul_rn(dmin, (float)prod));
                        }
                    }
                } else {
                    // Q6_K: ql (128), qh (64), int8 scales (16); d from the split array (kdot.rs:97-141)
                    const float dw = f16_bits_to_f32(__ldg(dsplit + (size_t)crow * nb + sb));
                    const uint4 scv = *reinterpret_cast<const uint4*>(blk + 192);
                    const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
                    uint32_t ql[4][GL], qh[2][GL];
#pragma unroll
                    for (int i = 0; i < 4; i++) lds_words<GL>(blk + 32 * i + 4 * g0, ql[i]);
#pragma unroll
                    for (int h = 0; h < 2; h++) lds_words<GL>(blk + 128 + 32 * h + 4 * g0, qh[h]);
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int k = 0; k < 4; k++) {
                            const int c32 = 4 * h + k;  // 32-element chunk
#pragma unroll
                            for (int n = 0; n < NC; n++) {
                                uint32_t xw[GL];
                                lds_words<GL>(xq + ((size_t)n * nb + sb) * 256 + c32 * 32 + 4 * g0, xw);
#pragma unroll
                                for (int g = 0; g < GL; g++) {
                                    const uint32_t lo = (ql[2 * h + (k & 1)][g] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
                                    const uint32_t hi = ((qh[h][g] >> (2 * k)) & 0x03030303u) << 4;
                                    const int si = h * 8 + 2 * k + ((g0 + g) >> 2);  // sc[2k + l/16] of half h
                                    const int scale = (int)(int8_t)prmt_byte(scw[si >> 2], si & 3);
                                    sumi[n][g] += scale * __dp4a((int)(lo | hi), (int)xw[g], 0);
                                }
                            }
                        }
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const int* bs = xs + ((size_t)n * nb + sb) * 16;
                        const float d = __fmul_rn(xd[n * nb + sb], dw);
#pragma unroll
                        for (int g = 0; g < GL; g++) {
                            const int l = g0 + g;
                            const int s0 = (int)(int8_t)prmt_byte(scw[(2 * l) >> 2], (2 * l) & 3);
                            const int s1 = (int)(int8_t)prmt_byte(scw[(2 * l + 1) >> 2], (2 * l + 1) & 3);
                            const int corr = 32 * (bs[2 * l] * s0 + bs[2 * l + 1] * s1);
                            acc[n][g] = __fadd_rn(acc[n][g], __fmul_rn(d, (float)(sumi[n][g] - corr)));
                        }
                    }
                }
            }
            __syncwarp();
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (c + V4_STAGES < nchunks) issue(c + V4_STAGES);
        }
        if (!alive) break;
        // gather the 8 main and 4 min lanes of the row in its part-0 lane; reduce in the reference's order
        const int base = rlane * LPR;
#pragma unroll
        for (int n = 0; n < NC; n++) {
            float l8[8], m4[4];
#pragma unroll
            for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[n][g % GL], base + g / GL);
#pragma unroll
            for (int i = 0; i < 4; i++) m4[i] = __shfl_sync(0xffffffffu, accm[n][i], base + (i * LPR) / 4);
            if (part == 0 && row < rows) {
                float v = reduce8(l8);
                if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
                y[(size_t)n * rows + row] = v;
            }
        }
    }
}

constexpr size_t SMEM_LIMIT = 227 * 1024;

template <int TYPE, int NC, int LPR>
cudaError_t launch_v4(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, float* y, cudaStream_t s) {
    using G = V4Geo<TYPE, LPR>;
    const size_t smem = G::FIXED + ActGeo::bytes(NC, nb);
    if (smem > SMEM_LIMIT) return cudaErrorInvalidConfiguration;
    auto kern = kq_gemv_v4_kernel<TYPE, NC, LPR>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, V4_WARPS * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int groups = (rows + G::RW - 1) / G::RW;
    const int grid = std::max(1, std::min((groups + V4_WARPS - 1) / V4_WARPS, num_sms() * per_sm));
    kern<<<grid, V4_WARPS * 32, smem, s>>>(w, dsplit, rows, nb, (const uint8_t*)act, y);
    return cudaGetLastError();
}

int g_forced_lpr = [] {
    const char* e = getenv("QDEC_GEMV_LANES_PER_ROW");  // tuning override: 1, 2, 4 or 8
    return e ? atoi(e) : 0;
}();

// Lanes per row: the smallest that still gives ~32 warps per SM, so short matrices spread over the GPU.
int pick_lpr(int rows) {
    const int forced = g_forced_lpr;
    if (forced == 1 || forced == 2 || forced == 4 || forced == 8) return forced;
    const long want_threads = (long)num_sms() * 32 * 32;
    for (int lpr = 1; lpr < 8; lpr *= 2)
        if ((long)rows * lpr >= want_threads) return lpr;
    return 8;
}

template <int TYPE, int NC>
cudaError_t launch_v4_nc(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, float* y, cudaStream_t s) {
    switch (pick_lpr(rows)) {
    case 1: return launch_v4<TYPE, NC, 1>(w, dsplit, rows, nb, act, y, s);
    case 2: return launch_v4<TYPE, NC, 2>(w, dsplit, rows, nb, act, y, s);
    case 4: return launch_v4<TYPE, NC, 4>(w, dsplit, rows, nb, act, y, s);
    default: return launch_v4<TYPE, NC, 8>(w, dsplit, rows, nb, act, y, s);
    }
}

template <int TYPE>
cudaError_t launch_v4_type(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, int ncols, float* y,
                           cudaStream_t s) {
    switch (ncols) {
    case 1: return launch_v4_nc<TYPE, 1>(w, dsplit, rows, nb, act, y, s);
    case 2: return launch_v4_nc<TYPE, 2>(w, dsplit, rows, nb, act, y, s);
    case 3: return launch_v4_nc<TYPE, 3>(w, dsplit, rows, nb, act, y, s);
    default: return launch_v4_nc<TYPE, 4>(w, dsplit, rows, nb, act, y, s);
    }
}

// ggml Q6_K (210-byte blocks) -> split layout: 208-byte blocks [ql | qh | scales], then every block's f16 d.
__global__ void repack_q6k_kernel(const uint8_t* __restrict__ src, size_t nblocks, uint8_t* __restrict__ dst) {
    uint16_t* dsplit = reinterpret_cast<uint16_t*>(dst + nblocks * 208);
    for (size_t b = blockIdx.x; b < nblocks; b += gridDim.x) {
        const uint8_t* s = src + b * 210;
        uint8_t* d = dst + b * 208;
        for (int i = threadIdx.x; i < 104; i += blockDim.x)
            reinterpret_cast<uint16_t*>(d)[i] = (uint16_t)(s[2 * i] | (s[2 * i + 1] << 8));
        if (threadIdx.x == 0) dsplit[b] = (uint16_t)(s[208] | (s[209] << 8));
    }
}

template <int TYPE>
constexpr size_t max_fixed() {
    return std::max(std::max(V4Geo<TYPE, 1>::FIXED, V4Geo<TYPE, 2>::FIXED), std::max(V4Geo<TYPE, 4>::FIXED, V4Geo<TYPE, 8>::FIXED));
}

}  // namespace

bool tma_gemv_supported(int type, int cols, int ncols) {
    if (type != T_Q4_K && type != T_Q5_K && type != T_Q6_K_SPLIT) return false;
    if (ncols < 1 || ncols > 4 || cols % QK_K) return false;
    const int nb = cols / QK_K;
    size_t fixed = 0;
    if (type == T_Q4_K) fixed = max_fixed<T_Q4_K>();
    else if (type == T_Q5_K) fixed = max_fixed<T_Q5_K>();
    else fixed = max_fixed<T_Q6_K>();
    return fixed + ActGeo::bytes(ncols, nb) <= SMEM_LIMIT;
}

cudaError_t launch_gemv_tma(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y, cudaStream_t s) {
    const int nb = cols / QK_K;
    if (type == T_Q4_K) return launch_v4_type<T_Q4_K>(w, nullptr, rows, nb, act, ncols, y, s);
    if (type == T_Q5_K) return launch_v4_type<T_Q5_K>(w, nullptr, rows, nb, act, ncols, y, s);
    // Q6_K split: the d array follows the blocks
    const uint16_t* dsplit = reinterpret_cast<const uint16_t*>(w + (size_t)rows * nb * 208);
    return launch_v4_type<T_Q6_K>(w, dsplit, rows, nb, act, ncols, y, s);
}

cudaError_t launch_repack_q6k(const uint8_t* src, size_t nblocks, uint8_t* dst, cudaStream_t s) {
    if (nblocks == 0) return cudaSuccess;
    const int grid = (int)std::min<size_t>(nblocks, (size_t)num_sms() * 32);
    repack_q6k_kernel<<<grid, 128, 0, s>>>(src, nblocks, dst);
    return cudaGetLastError();
}

void set_gemv_lanes_per_row(int lpr) { g_forced_lpr = lpr; }

unsigned read_kernel_error(bool clear) {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof v);
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_kernel_error, &z, sizeof z);
    }
    return v;
}

}  // namespace qdec
