// The decode GEMV of K-quant tile matrices (Q4_K, Q5_K, Q6_K in the tile layout) against 1..4 Q8_K image
// columns: the verify pass's ffn / attention / DeltaNet projections and the drafts' lm_head.  Bit-exact with
// crates/core/src/kernels/kdot.rs:37-141 (single row) and :176-333 (blocked), which is what matvec / matmul_t
// compute per row and column.
//
// Arithmetic.  The reference keeps, per row, column and super-block, eight exact i32 lanes (lane g = positions
// 4g..4g+3 of every 32-element chunk) with the chunk scale multiplied in, converts each lane once to f32, and
// accumulates d * lane into an 8-lane f32 chain over the super-blocks (plus, for Q4_K / Q5_K, four min lanes
// -dx * dmin * (mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1])); the row's value is reduce8 + reduce4 of the chains.
// Here each lane's integer sum is built with 8 dp4a (one per 32-element chunk, exact), the eight chunk results
// packed two per register as 16-bit halves (PRMT) and scaled by their chunk scales with 4 dp2a straight from
// the packed scale bytes -- two multiply-adds per instruction, and no per-scale unpacking.  Q4_K / Q5_K chunk
// results are biased by 2^15 into unsigned halves and the bias (2^15 * sum of the scales) is folded into the
// accumulator's start; Q6_K results fit signed halves.  For Q4_K the start also carries 1.5 * 2^23, so the
// finished sum read as a float minus 1.5 * 2^23 is the lane as f32 (|lane| < 2^22); Q5_K and Q6_K lanes (which
// may exceed that) are converted with a rounding I2F, as the reference's `as f32`.  All integer steps are exact,
// so the f32 operations are the reference's, in its order.
//
// Four Q4_K columns take the warp-MMA forms instead (kq_gemv7m_kernel, kq_gemv7mw_kernel): the same lanes as
// exact i32 accumulators of mma.sync.m16n8k32 (s8), with the chunk scale split into two byte parts on the weight
// operand and the activation operand masked per lane, so the per-column integer work -- most of the dp4a form's
// instructions at four columns -- runs on the tensor pipe; the f32 chains are unchanged.
//
// Work split.  Four threads share a weight row (thread tg holds lanes 2tg, 2tg+1 and min lane tg), eight rows
// make a tile (one tile block per super-block: 8 x the block bytes, contiguous, in the order the threads read
// it), a warp owns R tiles.  A CTA is G x S warps: G groups of R tiles each, and S warps per group splitting the
// super-block range (warp phase p takes super-blocks p, p+S, ...).  S = 1: every chain stays in the owning
// thread's registers.  S > 1: each warp writes its f32 lane terms (d * lane) to shared memory and, after every
// window of S super-blocks, one owner thread per (tile, column, row, lane) adds the window's terms in
// super-block order -- the reference's own chain of additions.  Short matrices (5120 rows) take S > 1 so that
// enough warps share the work.
//
// Data movement.  One thread keeps D windows in flight with bulk asynchronous copies (cp.async.bulk, no
// multicast) into a ring of shared-memory stages, each completing on its own mbarrier: per window a copy of S
// contiguous tile blocks per tile and a copy of S contiguous image blocks per column, so the bytes in flight cost
// no registers and the activation words are fetched once per CTA.  The weight copies of the first D windows are
// issued before griddepcontrol.wait (weights are never written after load), overlapping the kernel that
// produces the activations; the image copies after it.  A stage is refilled after a CTA barrier; every wait is
// bounded in time, and a CTA whose copy never arrived records an error word, lets its other copies land and
// returns.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

namespace {

constexpr uint32_t G7_MAGIC_I = 0x4B400000u;  // bits of 12582912.0f = 1.5 * 2^23
constexpr float G7_MAGIC_F = 12582912.0f;

template <int TYPE>
struct G7 {
    static constexpr int TB = TYPE == T_Q4_K ? 1152 : TYPE == T_Q5_K ? 1408 : 1680;  // tile block bytes
    static constexpr bool MINS = TYPE != T_Q6_K;
    static constexpr int LPC = MINS ? 12 : 8;  // f32 chains per (row, column): 8 lanes (+ 4 min lanes)
};

// One thread's share of a tile block (tile layout, gemv_v6.cu): thread L = 4 * row + tg.
template <int TYPE>
struct W7;
template <>
struct W7<T_Q4_K> {
    uint4 c0, c1, hdr;  // code chunks (qs groups 0,1 | 2,3: 8 bytes of each at 8tg), header of the row
};
template <>
struct W7<T_Q5_K> {
    uint4 c0, c1, hdr;
    uint2 qh;  // qh bytes 16 + 8tg .. +8 (bit s: the fifth bit of chunk s)
};
template <>
struct W7<T_Q6_K> {
    uint4 c0, c1, c2, sc;  // ql 8tg | ql 32+8tg; ql 64+8tg | ql 96+8tg; qh 128+8tg | qh 160+8tg; the row's scales
    uint32_t d;           // the row's f16 d (low half)
};

// The row-dependent decode of one super-block, shared by every column.
template <int TYPE>
struct Dec7 {
    uint32_t code[8][2];  // chunk s, lane 2tg+gi: four codes as bytes
    uint32_t scw[2];      // chunk scales as bytes: Q4_K/Q5_K sc0..3 | sc4..7; Q6_K this thread's chunk scales per half
    uint32_t start;       // the lane accumulator's start (bias terms)
    uint32_t spair;       // Q6_K: the row's scale bytes 4tg .. 4tg+3 (the -32 bsum correction of lanes 2tg, 2tg+1)
    uint32_t mpair;       // Q4_K/Q5_K: the mins of chunks 2tg, 2tg+1 in bytes 0, 1
    float dw, dminw;
};

template <int TYPE>
__device__ __forceinline__ void decode7(const W7<TYPE>& f, int tg, Dec7<TYPE>& o) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const uint32_t qs[4][2] = {{f.c0.x, f.c0.y}, {f.c0.z, f.c0.w}, {f.c1.x, f.c1.y}, {f.c1.z, f.c1.w}};
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int gi = 0; gi < 2; gi++) {
                o.code[2 * p][gi] = qs[p][gi] & 0x0F0F0F0Fu;
                o.code[2 * p + 1][gi] = (qs[p][gi] >> 4) & 0x0F0F0F0Fu;
            }
        if constexpr (TYPE == T_Q5_K) {
            const uint32_t qh[2] = {f.qh.x, f.qh.y};
#pragma unroll
            for (int s = 0; s < 8; s++)
#pragma unroll
                for (int gi = 0; gi < 2; gi++) o.code[s][gi] |= ((qh[gi] >> s) & 0x01010101u) << 4;
        }
        // get_scale_min_k4 (quant.rs:45-51) on all eight chunks at once: hdr bytes 4..15 are q[0..11]
        o.scw[0] = f.hdr.y & 0x3F3F3F3Fu;
        o.scw[1] = (f.hdr.w & 0x0F0F0F0Fu) | ((f.hdr.y >> 2) & 0x30303030u);
        const uint32_t mw = tg < 2 ? (f.hdr.z & 0x3F3F3F3Fu) : (((f.hdr.w >> 4) & 0x0F0F0F0Fu) | ((f.hdr.z >> 2) & 0x30303030u));
        o.mpair = mw >> (16 * (tg & 1));
        const uint32_t ssum = (uint32_t)__dp4a((int)o.scw[0], 0x01010101, __dp4a((int)o.scw[1], 0x01010101, 0));
        o.start = (TYPE == T_Q4_K ? G7_MAGIC_I : 0u) - 32768u * ssum;  // mod 2^32
        o.dw = f16_bits_to_f32((uint16_t)(f.hdr.x & 0xffff));
        o.dminw = f16_bits_to_f32((uint16_t)(f.hdr.x >> 16));
    } else {
        const uint32_t ql[4][2] = {{f.c0.x, f.c0.y}, {f.c0.z, f.c0.w}, {f.c1.x, f.c1.y}, {f.c1.z, f.c1.w}};
        const uint32_t qh[2][2] = {{f.c2.x, f.c2.y}, {f.c2.z, f.c2.w}};
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int gi = 0; gi < 2; gi++) {
                    const uint32_t lo = (ql[2 * h + (k & 1)][gi] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
                    const uint32_t hi = ((qh[h][gi] >> (2 * k)) & 0x03030303u) << 4;
                    o.code[4 * h + k][gi] = lo | hi;
                }
        // chunk (h, k) of lane 2tg+gi takes scale byte 8h + 2k + (tg >> 1) (kdot.rs:117, sc[2k + l/16])
        const uint32_t sel = (tg >> 1) ? 0x7531u : 0x6420u;
        o.scw[0] = __byte_perm(f.sc.x, f.sc.y, sel);
        o.scw[1] = __byte_perm(f.sc.z, f.sc.w, sel);
        const uint32_t scv[4] = {f.sc.x, f.sc.y, f.sc.z, f.sc.w};
        o.spair = scv[tg];
        o.start = 0u;
        o.dw = f16_bits_to_f32((uint16_t)(f.d & 0xffff));
    }
}

__device__ __forceinline__ uint32_t dp2a_lo_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("dp2a.lo.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ uint32_t dp2a_hi_u(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("dp2a.hi.u32.u32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ int dp2a_lo_s(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}
__device__ __forceinline__ int dp2a_hi_s(uint32_t a, uint32_t b, int c) {
    int r;
    asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// The exact integer lane gi of one row, super-block and column, as f32 (the reference's `sumi[g] as f32`).
template <int TYPE>
__device__ __forceinline__ float lane7(const Dec7<TYPE>& o, const uint32_t* xw, int gi, uint32_t bsp) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        uint32_t pk[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int a = __dp4a((int)o.code[2 * p][gi], (int)xw[gi * 8 + 2 * p], 32768);
            const int b = __dp4a((int)o.code[2 * p + 1][gi], (int)xw[gi * 8 + 2 * p + 1], 32768);
            pk[p] = __byte_perm((uint32_t)a, (uint32_t)b, 0x5410);
        }
        uint32_t s = dp2a_lo_u(pk[0], o.scw[0], o.start);
        s = dp2a_hi_u(pk[1], o.scw[0], s);
        s = dp2a_lo_u(pk[2], o.scw[1], s);
        s = dp2a_hi_u(pk[3], o.scw[1], s);
        if constexpr (TYPE == T_Q4_K) return __fsub_rn(__uint_as_float(s), G7_MAGIC_F);
        else return __int2float_rn((int)s);
    } else {
        uint32_t pk[4];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            const int a = __dp4a((int)o.code[2 * p][gi], (int)xw[gi * 8 + 2 * p], 0);
            const int b = __dp4a((int)o.code[2 * p + 1][gi], (int)xw[gi * 8 + 2 * p + 1], 0);
            pk[p] = __byte_perm((uint32_t)a, (uint32_t)b, 0x5410);
        }
        // chunks (h, 2j), (h, 2j+1) pair with the scale bytes 2j, 2j+1 of half h
        int s = dp2a_lo_s(pk[0], o.scw[0], 0);
        s = dp2a_hi_s(pk[1], o.scw[0], s);
        s = dp2a_lo_s(pk[2], o.scw[1], s);
        s = dp2a_hi_s(pk[3], o.scw[1], s);
        // - 32 * (bsums[2g] sc[2g] + bsums[2g+1] sc[2g+1])  (kdot.rs:128-133)
        const int corr = gi == 0 ? dp2a_lo_s(bsp, o.spair, 0) : dp2a_hi_s(bsp, o.spair, 0);
        return __int2float_rn(s - 32 * corr);
    }
}

__device__ __forceinline__ void gd_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void gd_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }
__device__ __forceinline__ void mbar_init7(uint64_t* bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(smem_addr(bar)));
}
__device__ __forceinline__ void mbar_expect7(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_test7(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// How long a stage wait lasts before it gives up (device clock), and a test knob: extra bytes the first window's
// barrier expects, which never arrive -- the failure-handling self-test's "data nothing sends".
__device__ unsigned long long g7_wait_ns = 2000000000ull;
__device__ unsigned g7_test_extra_tx = 0;

__device__ __forceinline__ unsigned long long gtimer7() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// A wait that gives up after g7_wait_ns and returns false.
__device__ __forceinline__ bool mbar_wait7(uint64_t* bar, uint32_t parity) {
    if (mbar_test7(bar, parity)) return true;
    const unsigned long long t0 = gtimer7(), lim = g7_wait_ns;
    while (!mbar_test7(bar, parity))
        if (gtimer7() - t0 > lim) return false;
    return true;
}
// bytes global -> shared, completing on `bar` (no multicast); 16-byte aligned addresses, size a multiple of 16
__device__ __forceinline__ void bulk7(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(smem_addr(dst)),
                 "l"(src), "r"(bytes), "r"(smem_addr(bar))
                 : "memory");
}

__device__ unsigned int g7_error = 0;  // set when a bounded wait of this file's kernels gave up

// Shared memory of a CTA: D stage buffers, each one window of S super-blocks for the CTA's G x R tiles (a copy of
// S contiguous tile blocks per tile) and the NC activation columns (a copy of S contiguous image blocks per
// column); then, with S > 1, the double-buffered lane terms and the final chains.
template <int TYPE, int NC, int G, int S, int R, int D, bool X2>
struct Geo7 {
    static constexpr int TB = G7<TYPE>::TB;
    static constexpr int WST = G * R * S * TB;
    // X2: the window's image blocks twice -- threads tg < 2 read copy A, tg >= 2 copy B, which sits 16 bytes off
    // the 128-byte bank period from A, so the four threads of a row read four different bank groups
    static constexpr int XW = NC * S * Q8K_IMG_BYTES;
    static constexpr int XOFF = X2 ? (XW + 127) / 128 * 128 + 16 : 0;
    static constexpr int STAGE = WST + XOFF + XW;
    static constexpr int PER_SB = R * NC * 8 * 12;  // one warp's terms of one super-block
    static constexpr size_t BAR = 128;
    static constexpr size_t ST0 = BAR;
    static constexpr size_t TERMS = ST0 + (size_t)D * STAGE;
    static constexpr size_t FIN = TERMS + (S > 1 ? (size_t)2 * G * S * PER_SB * 4 : 0);
    static constexpr size_t BYTES = FIN + (S > 1 ? (size_t)G * R * NC * 8 * 12 * 4 : 0);
    static_assert(D <= 16, "mbarriers");
    static_assert(STAGE % 16 == 0, "stage alignment");
};

// One thread's share of a tile block held in shared memory (the same offsets as the global tile layout).
template <int TYPE>
__device__ __forceinline__ void lds_w7(const uint8_t* ts, int L, int rs, W7<TYPE>& f) {
    auto v4 = [](const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); };
    f.c0 = v4(ts + L * 16);
    f.c1 = v4(ts + 512 + L * 16);
    if constexpr (TYPE == T_Q4_K) {
        f.hdr = v4(ts + 1024 + rs * 16);
    } else if constexpr (TYPE == T_Q5_K) {
        f.qh = *reinterpret_cast<const uint2*>(ts + 1024 + L * 8);
        f.hdr = v4(ts + 1280 + rs * 16);
    } else {
        f.c2 = v4(ts + 1024 + L * 16);
        f.sc = v4(ts + 1536 + rs * 16);
        f.d = *reinterpret_cast<const uint16_t*>(ts + 1664 + rs * 2);
    }
}

// Streaming form for matrices with enough tiles to fill the GPU with one warp per R tiles (S = 1): every warp
// streams its own tiles' super-blocks through a private ring of D stages of P super-blocks (one bulk copy of P
// contiguous tile blocks per tile and stage, completing on the warp's own mbarrier), so warps never wait for one
// another.  The activation image of all NC columns and super-blocks is staged once per CTA and stays resident,
// its code words rearranged so that the four threads of a row read them without bank conflicts: the 16-byte
// quad q = 4 tg + c of a block (thread tg's quad c) is stored at 4 c + tg.  Chains stay in the owning thread's
// registers, in super-block order.
template <int TYPE, int NC, int G, int R, int D, int P>
struct GeoS7 {
    static constexpr int TB = G7<TYPE>::TB;
    static constexpr size_t BAR = 1024;                   // G x D stage barriers
    static constexpr size_t STAGE = (size_t)R * P * TB;  // one warp's stage
    static constexpr size_t RING = (size_t)G * D * STAGE;
    static size_t bytes(int nb) { return BAR + RING + (size_t)NC * nb * Q8K_IMG_BYTES; }
    static_assert(8 * G * D <= BAR, "barriers");
    static_assert(STAGE % 16 == 0, "stage alignment");
};

// SWIGLU (the MLP's gate and up, R = 2): a warp's two tiles are tile t of w_a (gate) and tile t of w_b (up), so it
// ends holding both values of its 8 rows; it writes h = silu(g) * u (act.rs:24) to y_a, and the warp that
// finishes last among the 32 tiles of a 256-row block (a counter per block, reset by that warp) quantises the
// block of every column into the Q8_K image img_out -- the swiglu and quantise step of mlp.rs:114-132 without a
// launch of its own.
template <int TYPE, int NC, int G, int R, int D, int P, bool SWIGLU = false>
__global__ void __launch_bounds__(32 * G)
kq_gemv7s_kernel(const uint8_t* __restrict__ w_a, int rows_a, float* __restrict__ y_a, const uint8_t* __restrict__ w_b,
                 int rows_b, float* __restrict__ y_b, int nb, const uint8_t* __restrict__ img, uint8_t* __restrict__ img_out,
                 unsigned* __restrict__ blk_cnt) {
    static_assert(!SWIGLU || R == 2, "the gate/up pairing holds one tile of each matrix");
    using G_ = G7<TYPE>;
    using Geo = GeoS7<TYPE, NC, G, R, D, P>;
    constexpr int TB = G_::TB;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int rs = lane >> 2, tg = lane & 3;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem) + wid * D;
    uint8_t* ring = smem + Geo::BAR + (size_t)wid * D * Geo::STAGE;
    uint8_t* xs = smem + Geo::BAR + Geo::RING;
    constexpr int TPW = SWIGLU ? 1 : R;  // tile indices per warp
    const int ctas_a = (rows_a / 8 + G * TPW - 1) / (G * TPW);
    const bool second = !SWIGLU && (int)blockIdx.x >= ctas_a;
    const uint8_t* w = second ? w_b : w_a;
    const int rows = second ? rows_b : rows_a;
    float* y = second ? y_b : y_a;
    const int bid = second ? (int)blockIdx.x - ctas_a : (int)blockIdx.x;
    const int tiles = rows / 8;
    const int t0 = (bid * G + wid) * TPW;  // this warp's first tile
    const bool active = t0 < tiles;
    const int nwin = (nb + P - 1) / P;

    auto issue = [&](int win) {  // lane 0: the tile blocks of window `win` (P super-blocks) of this warp's tiles
        uint8_t* st = ring + (size_t)(win % D) * Geo::STAGE;
        const int n = min(P, nb - win * P);
        mbar_expect7(&bar[win % D], (uint32_t)(R * n * TB) + (win == 0 && wid == 0 ? g7_test_extra_tx : 0u));
        for (int j = 0; j < R; j++) {
            const int t = SWIGLU ? t0 : min(t0 + j, tiles - 1);
            const uint8_t* wm = SWIGLU && j == 1 ? w_b : w;
            bulk7(st + (size_t)j * P * TB, wm + ((size_t)t * nb + (size_t)win * P) * TB, (uint32_t)(n * TB), &bar[win % D]);
        }
    };
    if (lane == 0 && active) {
        for (int d = 0; d < D; d++) mbar_init7(&bar[d]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0 && active)
        for (int d = 0; d < D && d < nwin; d++) issue(d);  // weights are never written after load: before the wait
    gd_wait();  // the activation image is the previous kernel's output
    gd_launch();
    {  // stage the image, code quads rearranged (q = 4 tg + c -> 4 c + tg)
        const uint4* src = reinterpret_cast<const uint4*>(img);
        uint4* dst = reinterpret_cast<uint4*>(xs);
        const int nq = NC * nb * (Q8K_IMG_BYTES / 16);
        for (int i = tid; i < nq; i += 32 * G) {
            const int blk = i / (Q8K_IMG_BYTES / 16), q = i % (Q8K_IMG_BYTES / 16);
            const int qd = q < 16 ? 4 * (q & 3) + (q >> 2) : q;
            dst[blk * (Q8K_IMG_BYTES / 16) + qd] = src[i];
        }
    }
    __syncthreads();
    if (!active) return;
    float acc[R][NC][2], accm[R][NC];
#pragma unroll
    for (int j = 0; j < R; j++)
#pragma unroll
        for (int n = 0; n < NC; n++) acc[j][n][0] = acc[j][n][1] = accm[j][n] = 0.0f;

    bool ok = true;
    int win = 0;
    for (; win < nwin; win++) {
        const int slot = win % D;
        if (!__all_sync(0xffffffffu, mbar_wait7(&bar[slot], (uint32_t)((win / D) & 1)))) {
            ok = false;
            break;
        }
        const uint8_t* st = ring + (size_t)slot * Geo::STAGE;
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int sb = win * P + p;
            if (P > 1 && sb >= nb) break;
            Dec7<TYPE> dec[R];
#pragma unroll
            for (int j = 0; j < R; j++) {
                W7<TYPE> f;
                lds_w7<TYPE>(st + (size_t)(j * P + p) * TB, lane, rs, f);
                decode7<TYPE>(f, tg, dec[j]);
            }
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const uint8_t* xb = xs + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
                uint32_t xw[16];
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const uint4 v = reinterpret_cast<const uint4*>(xb)[4 * c + tg];
                    xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                }
                const float dx = *reinterpret_cast<const float*>(xb + Q8K_IMG_D);
                uint32_t q8s = 0;
                uint2 bsp2 = make_uint2(0, 0);
                if constexpr (G_::MINS) q8s = reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S)[tg];
                else bsp2 = reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP)[tg];
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const float dd = __fmul_rn(dx, dec[j].dw);  // d = dx * d_w (kdot.rs:50)
                    acc[j][n][0] = __fadd_rn(acc[j][n][0], __fmul_rn(dd, lane7<TYPE>(dec[j], xw, 0, bsp2.x)));
                    acc[j][n][1] = __fadd_rn(acc[j][n][1], __fmul_rn(dd, lane7<TYPE>(dec[j], xw, 1, bsp2.y)));
                    if constexpr (G_::MINS) {  // (-dx * dmin) * (mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1]), i = tg
                        const float prod = __fsub_rn(__int_as_float(dp2a_lo_s(q8s, dec[j].mpair, (int)G7_MAGIC_I)), G7_MAGIC_F);
                        accm[j][n] = __fadd_rn(accm[j][n], __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod));
                    }
                }
            }
        }
        __syncwarp();  // every lane is done with this slot
        if (lane == 0 && win + D < nwin) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's reads before the async refill
            issue(win + D);
        }
    }
    if (!ok) {
        // a copy never arrived: record it, let this warp's copies still in flight land (each wait bounded), stop
        if (lane == 0) {
            atomicCAS(&g7_error, 0u, 0x700u | (unsigned)TYPE);
            for (int k = win; k < nwin && k < win + D; k++) mbar_wait7(&bar[k % D], (uint32_t)((k / D) & 1));
        }
        return;
    }
    // per (tile, column, row): reduce8 of the 8 main lanes + reduce4 of the 4 min lanes (kdot.rs:75)
    const int base = rs * 4;
    float vr[R][NC];
#pragma unroll
    for (int j = 0; j < R; j++)
#pragma unroll
        for (int n = 0; n < NC; n++) {
            float l8[8], m4[4];
#pragma unroll
            for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[j][n][g & 1], base + (g >> 1));
#pragma unroll
            for (int m = 0; m < 4; m++) m4[m] = __shfl_sync(0xffffffffu, accm[j][n], base + m);
            float v = reduce8(l8);
            if constexpr (G_::MINS) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
            vr[j][n] = v;
            const int tile = t0 + j;
            if (!SWIGLU && tg == 0 && tile < tiles) y[(size_t)n * rows + tile * 8 + rs] = v;
        }
    if constexpr (SWIGLU) {
        if (tg == 0)
#pragma unroll
            for (int n = 0; n < NC; n++) y_a[(size_t)n * rows + t0 * 8 + rs] = __fmul_rn(silu_f32(vr[0][n]), vr[1][n]);
        __threadfence();  // the h rows before the block counter
        __syncwarp();
        const int blk = t0 / 32, nblk = rows / 256;
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&blk_cnt[blk], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == 31) {  // the block's last tile: quantise its 256 h values of every column
            __threadfence();
            float v[NC][8];  // every column's values first: one round trip to L2
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const float4* hb = reinterpret_cast<const float4*>(y_a + (size_t)n * rows + (size_t)blk * 256 + lane * 8);
                const float4 a = __ldcg(hb), b = __ldcg(hb + 1);
                v[n][0] = a.x, v[n][1] = a.y, v[n][2] = a.z, v[n][3] = a.w;
                v[n][4] = b.x, v[n][5] = b.y, v[n][6] = b.z, v[n][7] = b.w;
            }
#pragma unroll
            for (int n = 0; n < NC; n++) q8k_quantize_to_image(v[n], img_out + ((size_t)n * nblk + blk) * Q8K_IMG_BYTES);
            if (lane == 0) blk_cnt[blk] = 0u;  // ready for the next launch
        }
    }
}

// The same streaming form for Q4_K tile pairs with the integer lanes on the tensor cores: mma.sync m16n8k32 (s8)
// per reference lane pair.  A warp's two tiles are the MMA's 16 rows (row g of tile 0, row g of tile 1); the K
// dimension of one MMA is 4 chunks x 2 lanes (lanes 2u, 2u+1 of chunks 4q..4q+3), the activation codes are the B
// operand masked per lane (B column 2n + s holds column n's codes at lane 2u+s's K words, zeros at the other lane's),
// so D[row][2n+s] is exactly the reference's lane sum of lane 2u+s over those chunks; the chunk scale is folded
// into A split in two byte parts (q * (sc >> 3), q * (sc & 7): every product of a 4-bit code fits a byte) and
// sumi = 8 D0 + D1 in i32.  Thread (g = lane / 4, c = lane % 4) builds A words of chunk 4q + c for both its rows
// and ends holding column c's lanes and mins of both rows: the f32 chains (kdot.rs:37-95) run in its registers in
// super-block order, and the final reduce8 + reduce4 needs no shuffles.  The activation image is staged once per
// CTA as [column][super-block][u][q][s][c] words with a column stride of 8 banks mod 32, so the B loads of a
// warp hit 32 different banks.
template <int NC>
struct GeoM7 {
    static constexpr int TB = G7<T_Q4_K>::TB;
    __host__ __device__ static int col_words(int nb) { return nb * (Q8K_IMG_BYTES / 4) + ((8 - (nb * (Q8K_IMG_BYTES / 4)) % 32) + 32) % 32; }
};

__device__ __forceinline__ void mma_s8_16832(int (&d)[4], const uint32_t (&a)[4], uint32_t b0, uint32_t b1) {
    asm volatile("mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, {%0, %1, %2, %3};"
                 : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
                 : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// One super-block of a warp's two Q4_K tiles (tile blocks tb0, tb1 in shared memory) against the B column of
// thread (g, c): activation column g / 2 at lane parity g % 2, its image block at xb (zeros when !bval).  Leaves in
// thread (g, c), for column c and row g of tile j, the eight exact lane sums (biased: the bits of 1.5 * 2^23 + sumi
// as a float) and the row's d, dmin and min pairs
// (get_scale_min_k4, quant.rs:45-51).  PERM: the block's code words are stored [u][q][s][c] (the streaming kernel's
// staging) instead of the image's [lane][chunk].
template <bool PERM>
__device__ __forceinline__ void q4k_mma_sb(const uint8_t* tb0, const uint8_t* tb1, const uint32_t* xb, bool bval, int g, int c,
                                           int (&sumi)[2][8], float (&dw)[2], float (&dminw)[2], uint32_t (&mp)[2][4]) {
    const uint8_t* tb[2] = {tb0, tb1};
    uint32_t shi[2][2], slo[2][2];  // the scale parts of chunks c and 4 + c
#pragma unroll
    for (int j = 0; j < 2; j++) {
        const uint4 hd = *reinterpret_cast<const uint4*>(tb[j] + 1024 + g * 16);
        const uint32_t sw0 = hd.y & 0x3F3F3F3Fu, sw1 = (hd.w & 0x0F0F0F0Fu) | ((hd.y >> 2) & 0x30303030u);
        const uint32_t s0 = (sw0 >> (8 * c)) & 0xFFu, s1 = (sw1 >> (8 * c)) & 0xFFu;
        shi[j][0] = s0 >> 3, slo[j][0] = s0 & 7u, shi[j][1] = s1 >> 3, slo[j][1] = s1 & 7u;
        const uint32_t mlo = hd.z & 0x3F3F3F3Fu, mhi = ((hd.w >> 4) & 0x0F0F0F0Fu) | ((hd.z >> 2) & 0x30303030u);
        mp[j][0] = mlo, mp[j][1] = mlo >> 16, mp[j][2] = mhi, mp[j][3] = mhi >> 16;
        dw[j] = f16_bits_to_f32((uint16_t)(hd.x & 0xffff));
        dminw[j] = f16_bits_to_f32((uint16_t)(hd.x >> 16));
    }
    const int s = g & 1, sh = 4 * (c & 1);
#pragma unroll
    for (int u = 0; u < 4; u++) {  // lanes 2u, 2u + 1
        // the low part accumulates onto 1.5 * 2^23's bits, so 8 D0 + D1 read as a float is 1.5 * 2^23 + sumi
        // (|sumi| < 2^22): the lane as f32 with one subtraction
        int d0[4] = {0, 0, 0, 0}, d1[4] = {(int)G7_MAGIC_I, (int)G7_MAGIC_I, (int)G7_MAGIC_I, (int)G7_MAGIC_I};
#pragma unroll
        for (int q = 0; q < 2; q++) {
            // chunk 4q + c = pair 2q + c/2, nibble c % 2: the 8 bytes of lanes 2u, 2u + 1 of both rows
            const uint2 w0 = *reinterpret_cast<const uint2*>(tb0 + q * 512 + (g * 4 + u) * 16 + (c >> 1) * 8);
            const uint2 w1 = *reinterpret_cast<const uint2*>(tb1 + q * 512 + (g * 4 + u) * 16 + (c >> 1) * 8);
            const uint32_t n00 = (w0.x >> sh) & 0x0F0F0F0Fu, n01 = (w0.y >> sh) & 0x0F0F0F0Fu;
            const uint32_t n10 = (w1.x >> sh) & 0x0F0F0F0Fu, n11 = (w1.y >> sh) & 0x0F0F0F0Fu;
            // A: a0 row g (tile 0) K word c (lane 2u), a1 row g + 8 (tile 1), a2 / a3 K word c + 4 (lane 2u + 1)
            const uint32_t ah[4] = {n00 * shi[0][q], n10 * shi[1][q], n01 * shi[0][q], n11 * shi[1][q]};
            const uint32_t al[4] = {n00 * slo[0][q], n10 * slo[1][q], n01 * slo[0][q], n11 * slo[1][q]};
            // B: lane 2u + s of chunk 4q + c, in the K half of that lane
            const uint32_t xw = bval ? xb[PERM ? (u * 2 + q) * 8 + s * 4 + c : (2 * u + s) * 8 + 4 * q + c] : 0u;
            const uint32_t b0 = s ? 0u : xw, b1 = s ? xw : 0u;
            mma_s8_16832(d0, ah, b0, b1);
            mma_s8_16832(d1, al, b0, b1);
        }
        // d[0], d[1]: row g of tile 0, column c, lanes 2u, 2u + 1; d[2], d[3]: tile 1
#pragma unroll
        for (int j = 0; j < 2; j++)
#pragma unroll
            for (int e = 0; e < 2; e++) sumi[j][2 * u + e] = 8 * d0[2 * j + e] + d1[2 * j + e];
    }
}

// (-dx * dmin) * (mn[2k] q8s[2k] + mn[2k+1] q8s[2k+1]) of min group k (exact integer, then the reference's products)
__device__ __forceinline__ float q4k_min_term(float dx, float dminw, uint32_t q8w, uint32_t mpair) {
    const float prod = __fsub_rn(__int_as_float(dp2a_lo_s(q8w, mpair, (int)G7_MAGIC_I)), G7_MAGIC_F);
    return __fmul_rn(__fmul_rn(-dx, dminw), prod);
}

template <int NC, int G, int D, int P, bool SWIGLU = false>
__global__ void __launch_bounds__(32 * G)
kq_gemv7m_kernel(const uint8_t* __restrict__ w_a, int rows_a, float* __restrict__ y_a, const uint8_t* __restrict__ w_b,
                 int rows_b, float* __restrict__ y_b, int nb, const uint8_t* __restrict__ img, uint8_t* __restrict__ img_out,
                 unsigned* __restrict__ blk_cnt) {
    constexpr int TYPE = T_Q4_K, R = 2;
    using Geo = GeoS7<TYPE, NC, G, R, D, P>;
    constexpr int TB = G7<TYPE>::TB;
    extern __shared__ __align__(128) uint8_t smem[];
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
    const int g = lane >> 2, c = lane & 3;  // MMA group (row g of each tile; B column g) and thread in group
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem) + wid * D;
    uint8_t* ring = smem + Geo::BAR + (size_t)wid * D * Geo::STAGE;
    uint32_t* xs = reinterpret_cast<uint32_t*>(smem + Geo::BAR + Geo::RING);
    const int cw = GeoM7<NC>::col_words(nb);
    constexpr int TPW = SWIGLU ? 1 : R;
    const int ctas_a = (rows_a / 8 + G * TPW - 1) / (G * TPW);
    const bool second = !SWIGLU && (int)blockIdx.x >= ctas_a;
    const uint8_t* w = second ? w_b : w_a;
    const int rows = second ? rows_b : rows_a;
    float* y = second ? y_b : y_a;
    const int bid = second ? (int)blockIdx.x - ctas_a : (int)blockIdx.x;
    const int tiles = rows / 8;
    const int t0 = (bid * G + wid) * TPW;
    const bool active = t0 < tiles;
    const int nwin = (nb + P - 1) / P;

    auto issue = [&](int win) {
        uint8_t* st = ring + (size_t)(win % D) * Geo::STAGE;
        const int n = min(P, nb - win * P);
        mbar_expect7(&bar[win % D], (uint32_t)(R * n * TB) + (win == 0 && wid == 0 ? g7_test_extra_tx : 0u));
        for (int j = 0; j < R; j++) {
            const int t = SWIGLU ? t0 : min(t0 + j, tiles - 1);
            const uint8_t* wm = SWIGLU && j == 1 ? w_b : w;
            bulk7(st + (size_t)j * P * TB, wm + ((size_t)t * nb + (size_t)win * P) * TB, (uint32_t)(n * TB), &bar[win % D]);
        }
    };
    if (lane == 0 && active) {
        for (int d = 0; d < D; d++) mbar_init7(&bar[d]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    if (lane == 0 && active)
        for (int d = 0; d < D && d < nwin; d++) issue(d);  // weights are never written after load: before the wait
    gd_wait();  // the activation image is the previous kernel's output
    gd_launch();
    {  // stage the image: code quad Q = 2 L + q (lane L = 2u + s, chunks 4q..4q+3) goes to quad (2u + q) * 2 + s
        const uint4* src = reinterpret_cast<const uint4*>(img);
        const int nq = NC * nb * (Q8K_IMG_BYTES / 16);
        for (int i = tid; i < nq; i += 32 * G) {
            const int blk = i / (Q8K_IMG_BYTES / 16), Q = i % (Q8K_IMG_BYTES / 16);
            const int L = Q >> 1, q = Q & 1;
            const int qd = Q < 16 ? ((L >> 1) * 2 + q) * 2 + (L & 1) : Q;
            const int n = blk / nb, sb = blk % nb;
            reinterpret_cast<uint4*>(xs + (size_t)n * cw + (size_t)sb * (Q8K_IMG_BYTES / 4))[qd] = src[i];
        }
    }
    __syncthreads();
    if (!active) return;
    float acc[R][8], accm[R][4];  // column c of rows g (tile 0) and g (tile 1): the 8 lanes and the 4 mins groups
#pragma unroll
    for (int j = 0; j < R; j++) {
#pragma unroll
        for (int l = 0; l < 8; l++) acc[j][l] = 0.0f;
#pragma unroll
        for (int m = 0; m < 4; m++) accm[j][m] = 0.0f;
    }
    const int bn = g >> 1;  // this thread's B column: activation column bn (lane parity g % 2)
    const bool bval = bn < NC, cval = c < NC;
    bool ok = true;
    int win = 0;
    for (; win < nwin; win++) {
        const int slot = win % D;
        if (!__all_sync(0xffffffffu, mbar_wait7(&bar[slot], (uint32_t)((win / D) & 1)))) {
            ok = false;
            break;
        }
        const uint8_t* st = ring + (size_t)slot * Geo::STAGE;
#pragma unroll
        for (int p = 0; p < P; p++) {
            const int sb = win * P + p;
            if (P > 1 && sb >= nb) break;
            int sumi[R][8];
            float dw[R], dminw[R];
            uint32_t mp[R][4];
            const uint32_t* xb = xs + (size_t)(bval ? bn : 0) * cw + (size_t)sb * (Q8K_IMG_BYTES / 4);
            q4k_mma_sb<true>(st + (size_t)p * TB, st + (size_t)(P + p) * TB, xb, bval, g, c, sumi, dw, dminw, mp);
            // column c's scale and chunk sums
            const uint32_t* xc = xs + (size_t)(cval ? c : 0) * cw + (size_t)sb * (Q8K_IMG_BYTES / 4);
            const float dx = cval ? __uint_as_float(xc[Q8K_IMG_D / 4]) : 0.0f;
            const uint4 q8 = cval ? *reinterpret_cast<const uint4*>(xc + Q8K_IMG_Q8S / 4) : make_uint4(0, 0, 0, 0);
            const uint32_t q8w[4] = {q8.x, q8.y, q8.z, q8.w};
#pragma unroll
            for (int j = 0; j < R; j++) {
                const float dd = __fmul_rn(dx, dw[j]);  // d = dx * d_w (kdot.rs:50)
#pragma unroll
                for (int l = 0; l < 8; l++) acc[j][l] = __fadd_rn(acc[j][l], __fmul_rn(dd, __fsub_rn(__int_as_float(sumi[j][l]), G7_MAGIC_F)));
#pragma unroll
                for (int k = 0; k < 4; k++) accm[j][k] = __fadd_rn(accm[j][k], q4k_min_term(dx, dminw[j], q8w[k], mp[j][k]));
            }
        }
        __syncwarp();  // every lane is done with this slot
        if (lane == 0 && win + D < nwin) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's reads before the async refill
            issue(win + D);
        }
    }
    if (!ok) {
        if (lane == 0) {
            atomicCAS(&g7_error, 0u, 0x700u | (unsigned)TYPE);
            for (int k = win; k < nwin && k < win + D; k++) mbar_wait7(&bar[k % D], (uint32_t)((k / D) & 1));
        }
        return;
    }
    // per (tile, column c, row g): reduce8 of the 8 lanes + reduce4 of the 4 mins groups (kdot.rs:75)
    float vr[R];
#pragma unroll
    for (int j = 0; j < R; j++) {
        const float v = reduce8(acc[j]);
        vr[j] = __fadd_rn(v, __fadd_rn(__fadd_rn(accm[j][0], accm[j][2]), __fadd_rn(accm[j][1], accm[j][3])));
        const int tile = t0 + j;
        if (!SWIGLU && cval && tile < tiles) y[(size_t)c * rows + tile * 8 + g] = vr[j];
    }
    if constexpr (SWIGLU) {
        if (cval) y_a[(size_t)c * rows + t0 * 8 + g] = __fmul_rn(silu_f32(vr[0]), vr[1]);
        __threadfence();  // the h rows before the block counter
        __syncwarp();
        const int blk = t0 / 32, nblk = rows / 256;
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(&blk_cnt[blk], 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == 31) {  // the block's last tile: quantise its 256 h values of every column
            __threadfence();
            float v[NC][8];
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const float4* hb = reinterpret_cast<const float4*>(y_a + (size_t)n * rows + (size_t)blk * 256 + lane * 8);
                const float4 a = __ldcg(hb), b = __ldcg(hb + 1);
                v[n][0] = a.x, v[n][1] = a.y, v[n][2] = a.z, v[n][3] = a.w;
                v[n][4] = b.x, v[n][5] = b.y, v[n][6] = b.z, v[n][7] = b.w;
            }
#pragma unroll
            for (int n = 0; n < NC; n++) q8k_quantize_to_image(v[n], img_out + ((size_t)n * nblk + blk) * Q8K_IMG_BYTES);
            if (lane == 0) blk_cnt[blk] = 0u;  // ready for the next launch
        }
    }
}

// CTA = G x S warps: warp w serves tile group w % G (R tiles of 8 rows) and super-block phase w / G, i.e.
// super-blocks w/G, w/G + S, ... of its tiles.  Thread 0 keeps D windows of S super-blocks in flight.
template <int TYPE, int NC, int G, int S, int R, int D, bool X2>
__global__ void __launch_bounds__(32 * G * S)
kq_gemv7_kernel(const uint8_t* __restrict__ w_a, int rows_a, float* __restrict__ y_a, const uint8_t* __restrict__ w_b,
                int rows_b, float* __restrict__ y_b, int nb, const uint8_t* __restrict__ img) {
    using G_ = G7<TYPE>;
    using Geo = Geo7<TYPE, NC, G, S, R, D, X2>;
    constexpr int TB = G_::TB, LPC = G_::LPC, PER_SB = Geo::PER_SB;
    constexpr int CHAINS = G * R * NC * 8 * LPC;
    constexpr int NT = 32 * G * S;
    constexpr int CPT = (CHAINS + NT - 1) / NT;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    uint8_t* stages = smem + Geo::ST0;
    float* terms = reinterpret_cast<float*>(smem + Geo::TERMS);
    float* fin = reinterpret_cast<float*>(smem + Geo::FIN);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, gi = wid % G, si = wid / G;
    const int rs = lane >> 2, tg = lane & 3;
    const int ctas_a = (rows_a / 8 + G * R - 1) / (G * R);
    const bool second = (int)blockIdx.x >= ctas_a;
    const uint8_t* w = second ? w_b : w_a;
    const int rows = second ? rows_b : rows_a;
    float* y = second ? y_b : y_a;
    const int bid = second ? (int)blockIdx.x - ctas_a : (int)blockIdx.x;
    const int tiles = rows / 8;
    const int nwin = (nb + S - 1) / S;

    // window `win` into slot win % D: the weights (G*R copies of up to S tile blocks), then -- separately, after
    // the activations exist -- the NC image copies; one expect_tx for both
    auto win_sbs = [&](int win) { return min(S, nb - win * S); };
    auto issue_w = [&](int win) {
        uint8_t* st = stages + (size_t)(win % D) * Geo::STAGE;
        const int n = win_sbs(win);
        mbar_expect7(&bar[win % D], (uint32_t)(n * (G * R * TB + (X2 ? 2 : 1) * NC * Q8K_IMG_BYTES)) + (win == 0 ? g7_test_extra_tx : 0u));
        for (int k = 0; k < G * R; k++) {
            const int t = min(bid * G * R + k, tiles - 1);
            bulk7(st + (size_t)k * S * TB, w + ((size_t)t * nb + (size_t)win * S) * TB, (uint32_t)(n * TB), &bar[win % D]);
        }
    };
    auto issue_x = [&](int win) {
        uint8_t* st = stages + (size_t)(win % D) * Geo::STAGE + Geo::WST;
        const int n = win_sbs(win);
        for (int c = 0; c < NC; c++)
            for (int copy = 0; copy < (X2 ? 2 : 1); copy++)
                bulk7(st + (copy ? Geo::XOFF : 0) + (size_t)c * S * Q8K_IMG_BYTES,
                      img + ((size_t)c * nb + (size_t)win * S) * Q8K_IMG_BYTES, (uint32_t)(n * Q8K_IMG_BYTES), &bar[win % D]);
    };
    if (tid == 0) {
        s_abort = 0;
        for (int d = 0; d < D; d++) mbar_init7(&bar[d]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int d = 0; d < D && d < nwin; d++) issue_w(d);  // weights are never written after load: before the wait
    }
    gd_wait();  // the activation image is the previous kernel's output
    gd_launch();
    if (tid == 0)
        for (int d = 0; d < D && d < nwin; d++) issue_x(d);
    __syncthreads();

    float acc[R][NC][2], accm[R][NC];  // S == 1: this thread's chains
    float cacc[CPT];                   // S > 1: the chains this thread owns
#pragma unroll
    for (int j = 0; j < R; j++)
#pragma unroll
        for (int n = 0; n < NC; n++) acc[j][n][0] = acc[j][n][1] = accm[j][n] = 0.0f;
#pragma unroll
    for (int c = 0; c < CPT; c++) cacc[c] = 0.0f;

    for (int win = 0; win < nwin; win++) {
        const int slot = win % D;
        const bool ok = mbar_wait7(&bar[slot], (uint32_t)((win / D) & 1));
        if (!ok) s_abort = 1;
        const int sb = win * S + si;
        if (ok && sb < nb) {
            const uint8_t* st = stages + (size_t)slot * Geo::STAGE;
            Dec7<TYPE> dec[R];
#pragma unroll
            for (int j = 0; j < R; j++) {
                W7<TYPE> f;
                lds_w7<TYPE>(st + ((size_t)(gi * R + j) * S + si) * TB, lane, rs, f);
                decode7<TYPE>(f, tg, dec[j]);
            }
            float* tb = terms + (size_t)(((win & 1) * S + si) * G + gi) * PER_SB;
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const uint8_t* xb = st + Geo::WST + (X2 && tg >= 2 ? Geo::XOFF : 0) + (size_t)(n * S + si) * Q8K_IMG_BYTES;
                uint32_t xw[16];
#pragma unroll
                for (int c = 0; c < 4; c++) {
                    const uint4 v = reinterpret_cast<const uint4*>(xb + 64 * tg)[c];
                    xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                }
                const float dx = *reinterpret_cast<const float*>(xb + Q8K_IMG_D);
                uint32_t q8s = 0;
                uint2 bsp2 = make_uint2(0, 0);
                if constexpr (G_::MINS) q8s = reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S)[tg];
                else bsp2 = reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP)[tg];
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const float dd = __fmul_rn(dx, dec[j].dw);  // d = dx * d_w (kdot.rs:50)
                    const float t0 = __fmul_rn(dd, lane7<TYPE>(dec[j], xw, 0, bsp2.x));
                    const float t1 = __fmul_rn(dd, lane7<TYPE>(dec[j], xw, 1, bsp2.y));
                    float tm = 0.0f;
                    if constexpr (G_::MINS) {  // (-dx * dmin) * (mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1]), i = tg
                        const float prod = __fsub_rn(__int_as_float(dp2a_lo_s(q8s, dec[j].mpair, (int)G7_MAGIC_I)), G7_MAGIC_F);
                        tm = __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod);
                    }
                    if constexpr (S == 1) {
                        acc[j][n][0] = __fadd_rn(acc[j][n][0], t0);
                        acc[j][n][1] = __fadd_rn(acc[j][n][1], t1);
                        if constexpr (G_::MINS) accm[j][n] = __fadd_rn(accm[j][n], tm);
                    } else {
                        float* t = tb + ((j * NC + n) * 8 + rs) * 12;
                        *reinterpret_cast<float2*>(t + 2 * tg) = make_float2(t0, t1);
                        if constexpr (G_::MINS) t[8 + tg] = tm;
                    }
                }
            }
        }
        __syncthreads();  // every warp is done with this slot (and has written its terms)
        if (s_abort) {
            // a copy never arrived: record it, let the copies still in flight (this window's included) land, each wait
                // bounded, and stop
            if (tid == 0) {
                atomicCAS(&g7_error, 0u, 0x700u | (unsigned)TYPE);
                for (int k = win; k < nwin && k < win + D; k++) mbar_wait7(&bar[k % D], (uint32_t)((k / D) & 1));
            }
            return;
        }
        if (tid == 0 && win + D < nwin) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's reads before the async refill
            issue_w(win + D);
            issue_x(win + D);
        }
        if constexpr (S > 1) {  // the owners add this window's terms in super-block order
            const int nsb = win_sbs(win);
#pragma unroll
            for (int c = 0; c < CPT; c++) {
                const int ci = tid + c * NT;
                if (ci < CHAINS) {
                    const int g = ci / (R * NC * 8 * LPC), r = ci % (R * NC * 8 * LPC);
                    const int slot_i = (r / LPC) * 12 + r % LPC;
                    const float* tw = terms + (size_t)((win & 1) * S * G + g) * PER_SB + slot_i;
                    float a = cacc[c];
#pragma unroll
                    for (int k = 0; k < S; k++)
                        if (k < nsb) a = __fadd_rn(a, tw[(size_t)k * G * PER_SB]);
                    cacc[c] = a;
                }
            }
        }
    }
    // per (tile, column, row): reduce8 of the 8 main lanes + reduce4 of the 4 min lanes (kdot.rs:75)
    if constexpr (S == 1) {
        const int base = rs * 4;
#pragma unroll
        for (int j = 0; j < R; j++)
#pragma unroll
            for (int n = 0; n < NC; n++) {
                float l8[8], m4[4];
#pragma unroll
                for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[j][n][g & 1], base + (g >> 1));
#pragma unroll
                for (int m = 0; m < 4; m++) m4[m] = __shfl_sync(0xffffffffu, accm[j][n], base + m);
                const int tile = (bid * G + gi) * R + j;
                if (tg == 0 && tile < tiles) {
                    float v = reduce8(l8);
                    if constexpr (G_::MINS) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
                    y[(size_t)n * rows + tile * 8 + rs] = v;
                }
            }
    } else {
#pragma unroll
        for (int c = 0; c < CPT; c++) {
            const int ci = tid + c * NT;
            if (ci < CHAINS) {
                const int g = ci / (R * NC * 8 * LPC), r = ci % (R * NC * 8 * LPC);
                fin[(size_t)g * R * NC * 8 * 12 + (r / LPC) * 12 + r % LPC] = cacc[c];
            }
        }
        __syncthreads();
        for (int o = tid; o < G * R * NC * 8; o += NT) {
            const int r = o % 8, n = (o / 8) % NC, j = (o / (8 * NC)) % R, g = o / (8 * NC * R);
            const float* f = fin + (size_t)o * 12;
            float v = reduce8(f);
            if constexpr (G_::MINS) v = __fadd_rn(v, __fadd_rn(__fadd_rn(f[8], f[10]), __fadd_rn(f[9], f[11])));
            const int tile = (bid * G + g) * R + j;
            if (tile < tiles) y[(size_t)n * rows + tile * 8 + r] = v;
        }
    }
}

// The windowed form with the integer lanes on the tensor cores (Q4_K): warp w of the CTA serves the two tiles of
// tile group w % G (the MMA's 16 rows) and super-block phase w / G; per super-block each thread writes its
// column's 8 lane terms d * sumi and 4 min terms for its row of both tiles, and the owners add them in
// super-block order as in kq_gemv7_kernel.  A window's image blocks of column n start at n * XC + {0, 16, 64, 80}
// bytes (XC a multiple of 128), so the B loads of a warp (8 (lane parity) + 4 n' + c banks) hit 32 different banks;
// the term rows of a column are padded to 104 floats so the 16-byte term stores of a quarter warp do not collide.
template <int NC, int G, int S, int D>
struct GeoMW7 {
    static constexpr int TB = G7<T_Q4_K>::TB, R = 2;
    static constexpr int WST = G * R * S * TB;
    static constexpr int XC = (S * Q8K_IMG_BYTES + 127) / 128 * 128;
    __host__ __device__ static constexpr int xoff(int n) { return n * XC + (n & 1) * 16 + (n >> 1) * 64; }
    static constexpr int XW = xoff(NC - 1) + S * Q8K_IMG_BYTES;
    static constexpr int STAGE = (WST + XW + 127) / 128 * 128;
    static constexpr int CW = 8 * 12 + 8;  // one (tile, column)'s 8 rows of 12 terms, padded
    static constexpr int PER_SB = R * NC * CW;
    static constexpr size_t BAR = 128;
    static constexpr size_t ST0 = BAR;
    static constexpr size_t TERMS = ST0 + (size_t)D * STAGE;
    static constexpr size_t FIN = TERMS + (size_t)2 * G * S * PER_SB * 4;
    static constexpr size_t BYTES = FIN + (size_t)G * R * NC * 8 * 12 * 4;
    static_assert(S > 1 && D <= 16 && NC <= 4, "geometry");
};

template <int NC, int G, int S, int D>
__global__ void __launch_bounds__(32 * G * S)
kq_gemv7mw_kernel(const uint8_t* __restrict__ w_a, int rows_a, float* __restrict__ y_a, const uint8_t* __restrict__ w_b,
                  int rows_b, float* __restrict__ y_b, int nb, const uint8_t* __restrict__ img) {
    constexpr int TYPE = T_Q4_K, R = 2, LPC = 12;
    using Geo = GeoMW7<NC, G, S, D>;
    constexpr int TB = Geo::TB, PER_SB = Geo::PER_SB, CW = Geo::CW;
    constexpr int CHAINS = G * R * NC * 8 * LPC;
    constexpr int NT = 32 * G * S;
    constexpr int CPT = (CHAINS + NT - 1) / NT;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ int s_abort;
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem);
    uint8_t* stages = smem + Geo::ST0;
    float* terms = reinterpret_cast<float*>(smem + Geo::TERMS);
    float* fin = reinterpret_cast<float*>(smem + Geo::FIN);
    const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5, gi = wid % G, si = wid / G;
    const int g = lane >> 2, c = lane & 3;
    const int ctas_a = (rows_a / 8 + G * R - 1) / (G * R);
    const bool second = (int)blockIdx.x >= ctas_a;
    const uint8_t* w = second ? w_b : w_a;
    const int rows = second ? rows_b : rows_a;
    float* y = second ? y_b : y_a;
    const int bid = second ? (int)blockIdx.x - ctas_a : (int)blockIdx.x;
    const int tiles = rows / 8;
    const int nwin = (nb + S - 1) / S;

    auto win_sbs = [&](int win) { return min(S, nb - win * S); };
    auto issue_w = [&](int win) {
        uint8_t* st = stages + (size_t)(win % D) * Geo::STAGE;
        const int n = win_sbs(win);
        mbar_expect7(&bar[win % D], (uint32_t)(n * (G * R * TB + NC * Q8K_IMG_BYTES)) + (win == 0 ? g7_test_extra_tx : 0u));
        for (int k = 0; k < G * R; k++) {
            const int t = min(bid * G * R + k, tiles - 1);
            bulk7(st + (size_t)k * S * TB, w + ((size_t)t * nb + (size_t)win * S) * TB, (uint32_t)(n * TB), &bar[win % D]);
        }
    };
    auto issue_x = [&](int win) {
        uint8_t* st = stages + (size_t)(win % D) * Geo::STAGE + Geo::WST;
        const int n = win_sbs(win);
        for (int col = 0; col < NC; col++)
            bulk7(st + Geo::xoff(col), img + ((size_t)col * nb + (size_t)win * S) * Q8K_IMG_BYTES, (uint32_t)(n * Q8K_IMG_BYTES),
                  &bar[win % D]);
    };
    if (tid == 0) {
        s_abort = 0;
        for (int d = 0; d < D; d++) mbar_init7(&bar[d]);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        for (int d = 0; d < D && d < nwin; d++) issue_w(d);  // weights are never written after load: before the wait
    }
    gd_wait();  // the activation image is the previous kernel's output
    gd_launch();
    if (tid == 0)
        for (int d = 0; d < D && d < nwin; d++) issue_x(d);
    __syncthreads();

    float cacc[CPT];
#pragma unroll
    for (int k = 0; k < CPT; k++) cacc[k] = 0.0f;
    const int bn = g >> 1;
    const bool bval = bn < NC, cval = c < NC;

    for (int win = 0; win < nwin; win++) {
        const int slot = win % D;
        const bool ok = __all_sync(0xffffffffu, mbar_wait7(&bar[slot], (uint32_t)((win / D) & 1)));
        if (!ok && lane == 0) s_abort = 1;
        const int sb = win * S + si;
        if (ok && sb < nb) {
            const uint8_t* st = stages + (size_t)slot * Geo::STAGE;
            const uint8_t* xw = st + Geo::WST + (size_t)si * Q8K_IMG_BYTES;
            int sumi[R][8];
            float dw[R], dminw[R];
            uint32_t mp[R][4];
            q4k_mma_sb<false>(st + ((size_t)(gi * R) * S + si) * TB, st + ((size_t)(gi * R + 1) * S + si) * TB,
                              reinterpret_cast<const uint32_t*>(xw + Geo::xoff(bval ? bn : 0)), bval, g, c, sumi, dw, dminw, mp);
            if (cval) {
                const uint8_t* xc = xw + Geo::xoff(c);
                const float dx = *reinterpret_cast<const float*>(xc + Q8K_IMG_D);
                const uint4 q8 = *reinterpret_cast<const uint4*>(xc + Q8K_IMG_Q8S);
                const uint32_t q8w[4] = {q8.x, q8.y, q8.z, q8.w};
                float* tb = terms + (size_t)(((win & 1) * S + si) * G + gi) * PER_SB;
#pragma unroll
                for (int j = 0; j < R; j++) {
                    const float dd = __fmul_rn(dx, dw[j]);  // d = dx * d_w (kdot.rs:50)
                    float t[12];
#pragma unroll
                    for (int l = 0; l < 8; l++) t[l] = __fmul_rn(dd, __fsub_rn(__int_as_float(sumi[j][l]), G7_MAGIC_F));
#pragma unroll
                    for (int k = 0; k < 4; k++) t[8 + k] = q4k_min_term(dx, dminw[j], q8w[k], mp[j][k]);
                    float4* tp = reinterpret_cast<float4*>(tb + (j * NC + c) * CW + g * 12);
                    tp[0] = make_float4(t[0], t[1], t[2], t[3]);
                    tp[1] = make_float4(t[4], t[5], t[6], t[7]);
                    tp[2] = make_float4(t[8], t[9], t[10], t[11]);
                }
            }
        }
        __syncthreads();  // every warp is done with this slot (and has written its terms)
        if (s_abort) {
            if (tid == 0) {
                atomicCAS(&g7_error, 0u, 0x700u | (unsigned)TYPE);
                for (int k = win; k < nwin && k < win + D; k++) mbar_wait7(&bar[k % D], (uint32_t)((k / D) & 1));
            }
            return;
        }
        if (tid == 0 && win + D < nwin) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the slot's reads before the async refill
            issue_w(win + D);
            issue_x(win + D);
        }
        const int nsb = win_sbs(win);  // the owners add this window's terms in super-block order
#pragma unroll
        for (int k = 0; k < CPT; k++) {
            const int ci = tid + k * NT;
            if (ci < CHAINS) {
                const int gg = ci / (R * NC * 8 * LPC), r = ci % (R * NC * 8 * LPC);
                const int row = r / LPC, jn = row / 8;  // row = (j * NC + n) * 8 + row in tile
                const float* tw = terms + (size_t)((win & 1) * S * G + gg) * PER_SB + jn * CW + (row % 8) * 12 + r % LPC;
                float a = cacc[k];
#pragma unroll
                for (int p = 0; p < S; p++)
                    if (p < nsb) a = __fadd_rn(a, tw[(size_t)p * G * PER_SB]);
                cacc[k] = a;
            }
        }
    }
#pragma unroll
    for (int k = 0; k < CPT; k++) {
        const int ci = tid + k * NT;
        if (ci < CHAINS) fin[ci] = cacc[k];  // fin[gg][(j * NC + n) * 8 + row][12]
    }
    __syncthreads();
    // per (tile, column, row): reduce8 of the 8 main lanes + reduce4 of the 4 min lanes (kdot.rs:75)
    for (int o = tid; o < G * R * NC * 8; o += NT) {
        const int r = o % 8, n = (o / 8) % NC, j = (o / (8 * NC)) % R, gg = o / (8 * NC * R);
        const float* f = fin + (size_t)o * 12;
        const float v = __fadd_rn(reduce8(f), __fadd_rn(__fadd_rn(f[8], f[10]), __fadd_rn(f[9], f[11])));
        const int tile = (bid * G + gg) * R + j;
        if (tile < tiles) y[(size_t)n * rows + tile * 8 + r] = v;
    }
}

template <int NC, int G, int S, int D>
cudaError_t launch7mw(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                      const void* img, cudaStream_t s, bool pdl) {
    using Geo = GeoMW7<NC, G, S, D>;
    auto kern = kq_gemv7mw_kernel<NC, G, S, D>;
    static bool attr_done = false;  // per instantiation
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Geo::BYTES);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows_a / 8 + G * 2 - 1) / (G * 2) + (w_b ? (rows_b / 8 + G * 2 - 1) / (G * 2) : 0));
    cfg.blockDim = dim3(32 * G * S);
    cfg.dynamicSmemBytes = Geo::BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, (const uint8_t*)img);
}

template <int TYPE, int NC, int G, int S, int R, int D, bool X2 = false>
cudaError_t launch7(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                    const void* img, cudaStream_t s, bool pdl) {
    using Geo = Geo7<TYPE, NC, G, S, R, D, X2>;
    auto kern = kq_gemv7_kernel<TYPE, NC, G, S, R, D, X2>;
    static bool attr_done = false;  // per instantiation
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)Geo::BYTES);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows_a / 8 + G * R - 1) / (G * R) + (w_b ? (rows_b / 8 + G * R - 1) / (G * R) : 0));
    cfg.blockDim = dim3(32 * G * S);
    cfg.dynamicSmemBytes = Geo::BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, (const uint8_t*)img);
}

template <int TYPE, int NC, int G, int R, int D, int P, bool SWIGLU = false>
cudaError_t launch7s(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                     const void* img, cudaStream_t s, bool pdl, uint8_t* img_out = nullptr, unsigned* blk_cnt = nullptr) {
    using Geo = GeoS7<TYPE, NC, G, R, D, P>;
    auto kern = kq_gemv7s_kernel<TYPE, NC, G, R, D, P, SWIGLU>;
    const size_t bytes = Geo::bytes(nb);
    static size_t attr_bytes = 0;  // per instantiation: the largest dynamic shared memory enabled so far
    if (bytes > 48 * 1024 && bytes > attr_bytes) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        attr_bytes = bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = SWIGLU ? dim3((rows_a / 8 + G - 1) / G)
                         : dim3((rows_a / 8 + G * R - 1) / (G * R) + (w_b ? (rows_b / 8 + G * R - 1) / (G * R) : 0));
    cfg.blockDim = dim3(32 * G);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, (const uint8_t*)img, img_out, blk_cnt);
}

template <int NC, int G, int D, int P, bool SWIGLU = false>
cudaError_t launch7m(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                     const void* img, cudaStream_t s, bool pdl, uint8_t* img_out = nullptr, unsigned* blk_cnt = nullptr) {
    static_assert(NC <= 4, "the MMA's 8 B columns hold 4 activation columns x 2 lanes");
    using Geo = GeoS7<T_Q4_K, NC, G, 2, D, P>;
    auto kern = kq_gemv7m_kernel<NC, G, D, P, SWIGLU>;
    const size_t bytes = Geo::BAR + Geo::RING + (size_t)NC * GeoM7<NC>::col_words(nb) * 4;
    static size_t attr_bytes = 0;
    if (bytes > 48 * 1024 && bytes > attr_bytes) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes);
        if (e != cudaSuccess) return e;
        attr_bytes = bytes;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = SWIGLU ? dim3((rows_a / 8 + G - 1) / G)
                         : dim3((rows_a / 8 + G * 2 - 1) / (G * 2) + (w_b ? (rows_b / 8 + G * 2 - 1) / (G * 2) : 0));
    cfg.blockDim = dim3(32 * G);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, (const uint8_t*)img, img_out, blk_cnt);
}

int g_mma7_min_cols = 4;  // the smallest column group that takes the warp-MMA form for Q4_K (0 = never)

int g_cfg7 = [] {
    const char* e = getenv("QDEC_GEMV7_CFG");
    return e ? atoi(e) : 0;
}();

// Configurations: the streaming kernel (G warps of R tiles, D stages of P super-blocks per warp) for matrices with
// enough tiles, the windowed kernel (G tile groups x S super-block phases, R tiles per warp, D windows) otherwise.
template <int TYPE, int NC>
cudaError_t launch7_cfg(int cfg, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                        const void* img, cudaStream_t s, bool pdl) {
    if (cfg == 0) {  // by the rows of the launch (both matrices of a pair) and the column count, as measured
        const int rows = rows_a + (w_b ? rows_b : 0);
        if (rows >= 100000) cfg = NC == 1 ? 1 : 5;
        else if (rows >= 24576) cfg = 4;
        else if (rows >= 16384) cfg = 3;
        else if (rows >= 8192) cfg = rows / 80 <= num_sms() ? 6 : 2;  // 10-warp CTAs while they fit one wave
        else cfg = 7;
    }
    switch (cfg) {  // streaming: <warps, tiles per warp, stages, super-blocks per stage>; windowed: <tile groups,
                    // super-block phases, tiles per warp, windows, shifted image copy>
    case 1: return launch7s<TYPE, NC, 4, 1, 4, 1>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 2: return launch7s<TYPE, NC, 4, 1, 3, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 3:
        if (TYPE == T_Q4_K && g_mma7_min_cols > 0 && NC >= g_mma7_min_cols) return launch7m<NC, 4, 2, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
        return launch7s<TYPE, NC, 4, 2, 2, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 4:
        if (TYPE == T_Q4_K && g_mma7_min_cols > 0 && NC >= g_mma7_min_cols) return launch7m<NC, 5, 2, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
        return launch7s<TYPE, NC, 5, 2, 2, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 5:
        if (TYPE == T_Q4_K && g_mma7_min_cols > 0 && NC >= g_mma7_min_cols) return launch7m<NC, 6, 2, 1>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
        return launch7s<TYPE, NC, 6, 2, 2, 1>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 6: return launch7s<TYPE, NC, 10, 1, 2, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 7:
        if (TYPE == T_Q4_K && g_mma7_min_cols > 0 && NC >= g_mma7_min_cols) return launch7mw<NC, 1, 4, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
        return launch7<TYPE, NC, 1, 4, 2, 2, true>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    default: return launch7<TYPE, NC, 1, 4, 2, 3>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    }
}

template <int TYPE>
cudaError_t launch7_type(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                         const void* img, int nc, cudaStream_t s, bool pdl) {
    switch (nc) {
    case 1: return launch7_cfg<TYPE, 1>(g_cfg7, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 2: return launch7_cfg<TYPE, 2>(g_cfg7, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 3: return launch7_cfg<TYPE, 3>(g_cfg7, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    default: return launch7_cfg<TYPE, 4>(g_cfg7, w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    }
}

template <int TYPE>
cudaError_t launch7_swiglu_type(const uint8_t* w_g, const uint8_t* w_u, int rows, float* h, int nb, const void* img, int nc,
                                uint8_t* img_out, unsigned* cnt, cudaStream_t s, bool pdl) {
    if (TYPE == T_Q4_K && g_mma7_min_cols > 0 && nc >= g_mma7_min_cols) switch (nc) {
        case 1: return launch7m<1, 5, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
        case 2: return launch7m<2, 5, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
        case 3: return launch7m<3, 5, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
        default: return launch7m<4, 5, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
        }
    switch (nc) {  // the pair's default geometry: 5 warps of one gate and one up tile, 2 stages of 2 super-blocks
    case 1: return launch7s<TYPE, 1, 5, 2, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
    case 2: return launch7s<TYPE, 2, 5, 2, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
    case 3: return launch7s<TYPE, 3, 5, 2, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
    default: return launch7s<TYPE, 4, 5, 2, 2, 2, true>(w_g, rows, h, w_u, rows, nullptr, nb, img, s, pdl, img_out, cnt);
    }
}

}  // namespace

cudaError_t launch_gemv7_swiglu(int type, const uint8_t* w_gate, const uint8_t* w_up, int rows, int cols, const void* img,
                                int ncols, float* h_out, uint8_t* img_out, unsigned* blk_cnt, cudaStream_t s, bool pdl) {
    if (rows % 256 || cols % QK_K || !gemv7_supported(type)) return cudaErrorInvalidValue;
    if (((uintptr_t)w_gate | (uintptr_t)w_up | (uintptr_t)img) & 15) return cudaErrorMisalignedAddress;
    if (rows <= 0 || ncols <= 0) return cudaSuccess;
    const int nb = cols / QK_K, nblk = rows / 256;
    for (int c0 = 0; c0 < ncols; c0 += 4) {  // columns beyond 4 in groups of at most 4
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * nb * Q8K_IMG_BYTES;
        float* hh = h_out + (size_t)c0 * rows;
        uint8_t* io = img_out + (size_t)c0 * nblk * Q8K_IMG_BYTES;
        cudaError_t e;
        if (type == T_Q4_K_TILE) e = launch7_swiglu_type<T_Q4_K>(w_gate, w_up, rows, hh, nb, im, nc, io, blk_cnt, s, pdl);
        else if (type == T_Q5_K_TILE) e = launch7_swiglu_type<T_Q5_K>(w_gate, w_up, rows, hh, nb, im, nc, io, blk_cnt, s, pdl);
        else e = launch7_swiglu_type<T_Q6_K>(w_gate, w_up, rows, hh, nb, im, nc, io, blk_cnt, s, pdl);
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

bool gemv7_supported(int type) { return type == T_Q4_K_TILE || type == T_Q5_K_TILE || type == T_Q6_K_TILE; }

void set_gemv7_config(int cfg) { g_cfg7 = cfg; }
void set_gemv7_mma_min_cols(int n) { g_mma7_min_cols = n; }

cudaError_t enqueue_gemv7_error_read(unsigned* host_dst, cudaStream_t s) {
    return cudaMemcpyFromSymbolAsync(host_dst, g7_error, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, s);
}

unsigned read_gemv7_error(bool clear) {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, g7_error, sizeof v);
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g7_error, &z, sizeof z);
    }
    return v;
}

// Failure-handling self-test: a decode GEMV whose first stage waits for bytes nothing sends must give up after
// wait_ns, record its error word and leave the context usable; the same GEMV run normally afterwards must give the
// right result (zero weights: zeros).  Returns 0, or a code naming the half that misbehaved.
int selftest_gemv7_timeout(unsigned long long wait_ns) {
    const int rows = 64, cols = 256, maxc = 4;
    uint8_t *w = nullptr, *img = nullptr;
    float* y = nullptr;
    cudaStream_t st = nullptr;
    int rc = 0;
    if (cudaMalloc(&w, (size_t)rows / 8 * 1152) || cudaMalloc(&img, maxc * Q8K_IMG_BYTES) || cudaMalloc(&y, maxc * rows * 4) ||
        cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking))
        rc = 1;
    if (!rc) {
        cudaMemset(w, 0, (size_t)rows / 8 * 1152);
        cudaMemset(img, 0, maxc * Q8K_IMG_BYTES);
        cudaMemset(y, 0xff, maxc * rows * 4);
        read_gemv7_error(true);
    }
    const int saved_cfg = g_cfg7, saved_mma = g_mma7_min_cols;
    // the streaming kernel's first weight stage and the windowed kernel's first window, each in the dp4a form (one
    // column) and the warp-MMA form (four columns)
    const int cases[4][2] = {{1, 1}, {8, 1}, {4, 4}, {7, 4}};
    for (const auto& cs : cases) {
        if (rc) break;
        g_cfg7 = cs[0];
        g_mma7_min_cols = 4;
        const int nc = cs[1];
        const unsigned extra = 16;
        cudaMemcpyToSymbol(g7_test_extra_tx, &extra, sizeof extra);
        cudaMemcpyToSymbol(g7_wait_ns, &wait_ns, sizeof wait_ns);
        if (launch_gemv7(T_Q4_K_TILE, w, rows, y, nullptr, 0, nullptr, cols, img, nc, st, false) != cudaSuccess ||
            cudaStreamSynchronize(st) != cudaSuccess)
            rc = 2;  // the timed-out run must still complete as a kernel
        else if ((read_gemv7_error(true) & 0xff00u) != 0x700u)
            rc = 3;  // the wait did not report that it gave up
        const unsigned zero = 0;
        const unsigned long long dflt = 2000000000ull;
        cudaMemcpyToSymbol(g7_test_extra_tx, &zero, sizeof zero);
        cudaMemcpyToSymbol(g7_wait_ns, &dflt, sizeof dflt);
        if (!rc) {
            float h[maxc * 64];
            if (cudaMemset(y, 0xff, maxc * rows * 4) != cudaSuccess ||
                launch_gemv7(T_Q4_K_TILE, w, rows, y, nullptr, 0, nullptr, cols, img, nc, st, false) != cudaSuccess ||
                cudaStreamSynchronize(st) != cudaSuccess ||
                cudaMemcpy(h, y, (size_t)nc * rows * 4, cudaMemcpyDeviceToHost) != cudaSuccess)
                rc = 4;
            else if (read_gemv7_error(true) != 0)
                rc = 5;
            else
                for (int i = 0; i < nc * rows && !rc; i++)
                    if (h[i] != 0.0f) rc = 6;  // the normal run after the timeout gives the right result
        }
    }
    g_mma7_min_cols = saved_mma;
    g_cfg7 = saved_cfg;
    if (st) cudaStreamDestroy(st);
    cudaFree(w);
    cudaFree(img);
    cudaFree(y);
    return rc;
}

cudaError_t launch_gemv7(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                         int cols, const void* img, int ncols, cudaStream_t s, bool pdl) {
    if (rows_a % 8 || (w_b && rows_b % 8) || cols % QK_K) return cudaErrorInvalidValue;
    // the bulk copies need 16-byte aligned weights and activation image
    if (((uintptr_t)w_a | (uintptr_t)w_b | (uintptr_t)img) & 15) return cudaErrorMisalignedAddress;
    if (rows_a <= 0 || ncols <= 0) return cudaSuccess;
    const int nb = cols / QK_K;
    for (int c0 = 0; c0 < ncols; c0 += 4) {  // columns beyond 4 in groups of at most 4
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * nb * Q8K_IMG_BYTES;
        float* ya = y_a + (size_t)c0 * rows_a;
        float* yb = w_b ? y_b + (size_t)c0 * rows_b : nullptr;
        cudaError_t e;
        if (type == T_Q4_K_TILE) e = launch7_type<T_Q4_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else if (type == T_Q5_K_TILE) e = launch7_type<T_Q5_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else if (type == T_Q6_K_TILE) e = launch7_type<T_Q6_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else return cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

}  // namespace qdec
