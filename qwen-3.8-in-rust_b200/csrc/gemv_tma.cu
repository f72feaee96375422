// K-quant GEMV, bulk-copy pipeline (Q4_K / Q5_K weights x Q8_K activations), bit-exact with
// crates/core/src/kernels/kdot.rs:37-95 and the blocked form :176-270.
//
// Layout.  One lane owns one weight row and walks its super-blocks in order, so the reference's eight i32
// lanes, four min lanes, their f32 accumulators and the final reduce8 + reduce4 all live in that thread and
// follow the reference's order with no cross-lane traffic.  A warp owns 32 consecutive rows.  Weight bytes
// reach shared memory through cp.async.bulk (one copy per row and chunk of SC super-blocks, completion on an
// mbarrier, STAGES chunks in flight per warp); each row gets its own shared slot whose stride is an odd
// number of 16-byte units, so the 32 lanes' 16-byte reads hit distinct banks.  The activation columns are
// staged once per CTA; every lane of a warp reads the same activation word at the same time (the warp walks
// the super-blocks in lockstep), which shared memory serves as a broadcast.
//
// Waits are bounded: a wait that gives up sets the library's device error word and the kernel leaves the
// row loop; the host reports QDEC_ETIMEOUT.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

__device__ unsigned int g_kernel_error = 0;  // first timeout code recorded by a bounded wait

namespace {

constexpr int TMA_WARPS = 8;       // warps per CTA, 32 rows each
constexpr int TMA_SC = 1;          // super-blocks per copy chunk
constexpr uint32_t WAIT_LIMIT = 1u << 26;

template <int TYPE>
struct TmaGeo {
    static constexpr int BB = TYPE == T_Q4_K ? 144 : 176;
    static constexpr int CHUNK = TMA_SC * BB;                                  // bytes per row per chunk
    static constexpr int SLOT = ((CHUNK / 16) % 2 == 0) ? CHUNK + 16 : CHUNK;   // odd number of 16-byte units
    static constexpr int STAGE_BYTES = 32 * SLOT;                               // one warp's stage
};

// shared memory in front of the stages: one 8-byte mbarrier per (warp, stage), rounded to 128 bytes
template <int STAGES>
__host__ __device__ constexpr size_t tma_bar_bytes() {
    return ((size_t)TMA_WARPS * STAGES * 8 + 127) / 128 * 128;
}

template <int TYPE, int STAGES>
__host__ __device__ constexpr size_t tma_smem_bytes_fixed() {
    return tma_bar_bytes<STAGES>() + (size_t)TMA_WARPS * STAGES * TmaGeo<TYPE>::STAGE_BYTES;
}

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
// Bounded wait; returns false (and records the error) if the phase never completes.
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

// Activation image for this kernel: per (column, super-block): the 256 code bytes in block order, the f32 d,
// and the 8 sub-block sums q8s = bsums[2s] + bsums[2s+1] (q8k.rs:185-193).
struct ActGeo {
    static __host__ __device__ size_t off_d(int nc, int nb) { return (size_t)nc * nb * 256; }
    static __host__ __device__ size_t off_s(int nc, int nb) { return (off_d(nc, nb) + (size_t)nc * nb * 4 + 15) & ~(size_t)15; }
    static __host__ __device__ size_t bytes(int nc, int nb) { return off_s(nc, nb) + (size_t)nc * nb * 32; }
};

__device__ void stage_act(const uint8_t* __restrict__ act, int nc, int nb, uint8_t* sm) {
    uint32_t* xq = reinterpret_cast<uint32_t*>(sm);
    float* xd = reinterpret_cast<float*>(sm + ActGeo::off_d(nc, nb));
    int* xs = reinterpret_cast<int*>(sm + ActGeo::off_s(nc, nb));
    for (int i = threadIdx.x; i < nc * nb * 73; i += blockDim.x) {
        const int blk = i / 73, wi = i % 73;
        const uint32_t v = reinterpret_cast<const uint32_t*>(act + (size_t)blk * Q8K_BLOCK_BYTES)[wi];
        if (wi == 0) xd[blk] = __uint_as_float(v);
        else if (wi <= 64) xq[(size_t)blk * 64 + (wi - 1)] = v;
        else xs[blk * 8 + (wi - 65)] = (int)(int16_t)(((int)(int16_t)(v & 0xffff)) + ((int)(int16_t)(v >> 16)));
    }
}

template <int TYPE, int NC, int TMA_STAGES>
__global__ void __launch_bounds__(TMA_WARPS * 32, 1)
kq_gemv_tma_kernel(const uint8_t* __restrict__ w, int rows, int nb, const uint8_t* __restrict__ act, float* __restrict__ y) {
    using G = TmaGeo<TYPE>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);                      // [TMA_WARPS][TMA_STAGES]
    uint8_t* wst = smem + tma_bar_bytes<TMA_STAGES>();                        // [TMA_WARPS][TMA_STAGES][STAGE_BYTES]
    static_assert(tma_bar_bytes<TMA_STAGES>() >= (size_t)TMA_WARPS * TMA_STAGES * sizeof(uint64_t), "barrier region");
    uint8_t* asm_ = wst + (size_t)TMA_WARPS * TMA_STAGES * G::STAGE_BYTES;   // activation image
    if (threadIdx.x < TMA_WARPS * TMA_STAGES) mbar_init(&bars[threadIdx.x], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    stage_act(act, NC, nb, asm_);
    __syncthreads();

    const uint32_t* xq = reinterpret_cast<const uint32_t*>(asm_);
    const float* xd = reinterpret_cast<const float*>(asm_ + ActGeo::off_d(NC, nb));
    const int* xs = reinterpret_cast<const int*>(asm_ + ActGeo::off_s(NC, nb));
    uint64_t* wbar = bars + warp * TMA_STAGES;
    uint8_t* wbuf = wst + (size_t)warp * TMA_STAGES * G::STAGE_BYTES;
    const size_t row_bytes = (size_t)nb * G::BB;
    const int nchunks = (nb + TMA_SC - 1) / TMA_SC;
    uint32_t phase_bits = 0;  // parity per stage
    bool alive = true;

    const int tiles = (rows + 31) / 32;
    for (int tile = blockIdx.x * TMA_WARPS + warp; tile < tiles && alive; tile += gridDim.x * TMA_WARPS) {
        const int row = tile * 32 + lane;
        const uint8_t* wrow = w + (size_t)min(row, rows - 1) * row_bytes;
        auto issue = [&](int c) {
            const int st = c % TMA_STAGES;
            const int sb0 = c * TMA_SC;
            const uint32_t bytes = (uint32_t)(min(TMA_SC, nb - sb0) * G::BB);
            if (lane == 0) mbar_expect_tx(&wbar[st], 32 * bytes);
            __syncwarp();
            bulk_g2s(wbuf + (size_t)st * G::STAGE_BYTES + lane * G::SLOT, wrow + (size_t)sb0 * G::BB, bytes, &wbar[st]);
        };
        for (int c = 0; c < min(TMA_STAGES, nchunks); c++) issue(c);

        float acc[NC][8], accm[NC][4];
#pragma unroll
        for (int n = 0; n < NC; n++) {
#pragma unroll
            for (int g = 0; g < 8; g++) acc[n][g] = 0.0f;
#pragma unroll
            for (int i = 0; i < 4; i++) accm[n][i] = 0.0f;
        }
        for (int c = 0; c < nchunks; c++) {
            const int st = c % TMA_STAGES;
            if (!mbar_wait_bounded(&wbar[st], (phase_bits >> st) & 1u, 0x100u | (unsigned)TYPE)) {
                alive = false;
                break;
            }
            phase_bits ^= 1u << st;
            const uint8_t* slot = wbuf + (size_t)st * G::STAGE_BYTES + lane * G::SLOT;
            const int nsb = min(TMA_SC, nb - c * TMA_SC);
            for (int j = 0; j < nsb; j++) {
                const int sb = c * TMA_SC + j;
                const uint8_t* blk = slot + j * G::BB;
                const uint4 hdr = *reinterpret_cast<const uint4*>(blk);
                // get_scale_min_k4 (quant.rs:45-51), packed one byte per sub-block
                const uint32_t sc03 = hdr.y & 0x3F3F3F3Fu;
                const uint32_t m03 = hdr.z & 0x3F3F3F3Fu;
                const uint32_t sc47 = (hdr.w & 0x0F0F0F0Fu) | ((hdr.y >> 2) & 0x30303030u);
                const uint32_t m47 = ((hdr.w >> 4) & 0x0F0F0F0Fu) | ((hdr.z >> 2) & 0x30303030u);
                const float dw = f16_bits_to_f32((uint16_t)(hdr.x & 0xffff));
                const float dminw = f16_bits_to_f32((uint16_t)(hdr.x >> 16));
                uint4 qh0, qh1;
                if constexpr (TYPE == T_Q5_K) {
                    qh0 = *reinterpret_cast<const uint4*>(blk + 16);
                    qh1 = *reinterpret_cast<const uint4*>(blk + 32);
                }
                int sumi[NC][8];
#pragma unroll
                for (int n = 0; n < NC; n++)
#pragma unroll
                    for (int g = 0; g < 8; g++) sumi[n][g] = 0;
#pragma unroll
                for (int p = 0; p < 4; p++) {  // sub-blocks 2p (low nibbles) and 2p+1 (high nibbles)
                    constexpr int QO = TYPE == T_Q4_K ? 16 : 48;
                    const uint4 r0 = *reinterpret_cast<const uint4*>(blk + QO + 32 * p);
                    const uint4 r1 = *reinterpret_cast<const uint4*>(blk + QO + 32 * p + 16);
                    const uint32_t raw[8] = {r0.x, r0.y, r0.z, r0.w, r1.x, r1.y, r1.z, r1.w};
                    const int scA = (int)prmt_byte(p < 2 ? sc03 : sc47, (2 * p) & 3);
                    const int scB = (int)prmt_byte(p < 2 ? sc03 : sc47, (2 * p + 1) & 3);
                    uint32_t lo[8], hi[8];
#pragma unroll
                    for (int g = 0; g < 8; g++) {
                        lo[g] = raw[g] & 0x0F0F0F0Fu;
                        hi[g] = (raw[g] >> 4) & 0x0F0F0F0Fu;
                    }
                    if constexpr (TYPE == T_Q5_K) {
                        const uint32_t qh[8] = {qh0.x, qh0.y, qh0.z, qh0.w, qh1.x, qh1.y, qh1.z, qh1.w};
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            lo[g] |= ((qh[g] >> (2 * p)) & 0x01010101u) << 4;
                            hi[g] |= ((qh[g] >> (2 * p + 1)) & 0x01010101u) << 4;
                        }
                    }
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const uint4* xa = reinterpret_cast<const uint4*>(xq + ((size_t)n * nb + sb) * 64 + (2 * p) * 8);
                        const uint4 a0 = xa[0], a1 = xa[1], b0 = xa[2], b1 = xa[3];
                        const uint32_t xA[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                        const uint32_t xB[8] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w};
#pragma unroll
                        for (int g = 0; g < 8; g++) {
                            sumi[n][g] += scA * __dp4a((int)lo[g], (int)xA[g], 0);
                            sumi[n][g] += scB * __dp4a((int)hi[g], (int)xB[g], 0);
                        }
                    }
                }
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const float dx = xd[n * nb + sb];
                    const float d = __fmul_rn(dx, dw);
                    const float dmin = __fmul_rn(-dx, dminw);
#pragma unroll
                    for (int g = 0; g < 8; g++) acc[n][g] = __fadd_rn(acc[n][g], __fmul_rn(d, (float)sumi[n][g]));
                    const int4 q0 = *reinterpret_cast<const int4*>(xs + ((size_t)n * nb + sb) * 8);
                    const int4 q1 = *reinterpret_cast<const int4*>(xs + ((size_t)n * nb + sb) * 8 + 4);
                    const int q8s[8] = {q0.x, q0.y, q0.z, q0.w, q1.x, q1.y, q1.z, q1.w};
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        const uint32_t mw = i < 2 ? m03 : m47;
                        const int prod = (int)prmt_byte(mw, (2 * i) & 3) * q8s[2 * i] + (int)prmt_byte(mw, (2 * i + 1) & 3) * q8s[2 * i + 1];
                        accm[n][i] = __fadd_rn(accm[n][i], __fmul_rn(dmin, (float)prod));
                    }
                }
            }
            __syncwarp();
            // the stage's generic-proxy reads are done; order them before the async-proxy refill
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            if (c + TMA_STAGES < nchunks) issue(c + TMA_STAGES);
        }
        if (!alive) break;
        if (row < rows) {
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const float m = __fadd_rn(__fadd_rn(accm[n][0], accm[n][2]), __fadd_rn(accm[n][1], accm[n][3]));
                y[(size_t)n * rows + row] = __fadd_rn(reduce8(acc[n]), m);
            }
        }
    }
}

template <int TYPE, int NC, int STAGES>
cudaError_t launch_tma_st(const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    const int nb = cols / QK_K;
    const size_t smem = tma_smem_bytes_fixed<TYPE, STAGES>() + ActGeo::bytes(NC, nb);
    auto kern = kq_gemv_tma_kernel<TYPE, NC, STAGES>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, TMA_WARPS * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    const int tiles = (rows + 31) / 32;
    const int grid = std::max(1, std::min((tiles + TMA_WARPS - 1) / TMA_WARPS, num_sms() * per_sm));
    kern<<<grid, TMA_WARPS * 32, smem, s>>>(w, rows, nb, (const uint8_t*)act, y);
    return cudaGetLastError();
}

constexpr size_t SMEM_LIMIT = 227 * 1024;

template <int TYPE, int NC>
cudaError_t launch_tma(const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    const int nb = cols / QK_K;
    if (tma_smem_bytes_fixed<TYPE, 4>() + ActGeo::bytes(NC, nb) <= SMEM_LIMIT)
        return launch_tma_st<TYPE, NC, 4>(w, rows, cols, act, y, s);
    return launch_tma_st<TYPE, NC, 2>(w, rows, cols, act, y, s);
}

}  // namespace

bool tma_gemv_supported(int type, int cols, int ncols) {
    if (type != T_Q4_K && type != T_Q5_K) return false;
    if (ncols < 1 || ncols > 4) return false;
    const int nb = cols / QK_K;
    const size_t fixed = type == T_Q4_K ? tma_smem_bytes_fixed<T_Q4_K, 2>() : tma_smem_bytes_fixed<T_Q5_K, 2>();
    return fixed + ActGeo::bytes(ncols, nb) <= SMEM_LIMIT;
}

cudaError_t launch_gemv_tma(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y, cudaStream_t s) {
    if (type == T_Q4_K) {
        switch (ncols) {
        case 1: return launch_tma<T_Q4_K, 1>(w, rows, cols, act, y, s);
        case 2: return launch_tma<T_Q4_K, 2>(w, rows, cols, act, y, s);
        case 3: return launch_tma<T_Q4_K, 3>(w, rows, cols, act, y, s);
        default: return launch_tma<T_Q4_K, 4>(w, rows, cols, act, y, s);
        }
    }
    switch (ncols) {
    case 1: return launch_tma<T_Q5_K, 1>(w, rows, cols, act, y, s);
    case 2: return launch_tma<T_Q5_K, 2>(w, rows, cols, act, y, s);
    case 3: return launch_tma<T_Q5_K, 3>(w, rows, cols, act, y, s);
    default: return launch_tma<T_Q5_K, 4>(w, rows, cols, act, y, s);
    }
}

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
