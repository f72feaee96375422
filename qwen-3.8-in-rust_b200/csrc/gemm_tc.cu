// Prompt prefill GEMM on the 5th-generation tensor cores (tcgen05): K-quant weights in the tile layout against
// t >= 16 activation columns of the Q8_K device image, bit-exact with the reference's per-column dot
// (crates/core/src/kernels/kdot.rs:37-141, reached from Model::prefill model.rs:443 through the blocked matmul
// matvec.rs:446-467).  Decode (t <= 4 verify columns) stays on the CUDA-core GEMV.
//
// Exactness.  The reference accumulates, per row, column and super-block, eight exact i32 lane sums
// (lane g = positions 4g..4g+3 of each 32-element chunk, chunk scale folded in), then per lane an f32 chain
// acc[g] += d * f32(sumi[g]) over the super-blocks.  Here the integer part runs on the tensor cores: the weights
// are dequantised with their chunk scale folded in (sc * q: <= 1953 for Q4_K/Q5_K, exact in f16; Q6_K splits
// q = lo4 + 16 * hi2 so that sc * lo4 and sc * hi2 stay exact), the activation codes are exact in f16, every
// product is an integer below 2^18 and every partial sum of a lane an integer below 2^23, so the f32
// accumulation of `tcgen05.mma.kind::f16` is exact.  Each lane gets its own accumulator: the K dimension of one
// MMA is one lane's 16 positions of half a super-block, so eight MMAs per half super-block write eight
// accumulators (Q6_K: eight for the low parts, eight for the high parts).  The f32 chains (d * sumi, the
// Q4_K/Q5_K mins term, the Q6_K -32 * bsum correction) then run on the CUDA cores in the reference's order, in
// registers, across super-blocks.
//
// Work split.  A CTA owns 128 weight rows (the MMA's M, one TMEM lane each) and 16 activation columns (N).  Its
// 16 compute warps walk the super-blocks in steps of one MMA operand tile (half a super-block; for Q6_K half a
// super-block of the low or of the high parts); a 17th warp issues the copies and the MMAs.  The raw bytes of a
// super-block -- its 16 tile blocks (8 rows each, contiguous in the tile layout) and the 16 columns' image blocks
// -- arrive by two 2-D TMA tensor copies (completing on an mbarrier) into a ring of four stages, at least three
// steps ahead.  Per step the issuing warp starts the step's eight MMAs (operands from one of two shared-memory
// buffers, accumulators in the TMEM buffer of this super-block), commits them to an mbarrier and waits for them;
// meanwhile the compute warps run their share of the previous super-block's epilogue from the other TMEM buffer
// (warp w: TMEM lanes 32*(w%4).., i.e. rows, and one or two of its columns 4*(w/4)..+3) and dequantise the next
// step into the other operand buffer; one barrier ends the step.  Every wait is bounded: after about a second
// the kernel records an error code, drains its copies, frees its TMEM and returns.  Column groups are the
// fastest grid dimension, so the CTAs that share a weight tile run together and the tile is read from HBM once.
#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"
#include "tcgen05.cuh"

namespace qdec {

namespace {

__device__ unsigned int g_tc_error = 0;  // first error code of a bounded wait that gave up

constexpr int TC_M = 128, TC_N = 16, TC_COMPUTE = 512, TC_THREADS = TC_COMPUTE + 32;  // 16 compute warps + the issuing warp
constexpr int TC_A_STEP = TC_M * 32;        // one lane's K step (16 f16) over the 128 rows
constexpr int TC_A_PITCH = TC_A_STEP + 16;  // steps 16 bytes apart beyond their size: the four lane pairs that a
                                            // quarter-warp of the dequantisation stores fall in distinct banks
constexpr int TC_A_PART = 8 * TC_A_PITCH;   // eight lanes: one operand tile (half a super-block of one part)
constexpr int TC_B_STEP = TC_N * 32;
constexpr int TC_B_BUF = 8 * TC_B_STEP;
constexpr int TC_META = 20;  // floats per column and super-block: dx, 3 unused, then q8s[8] (Q4_K/Q5_K) or 2*bsums[16] (Q6_K)
constexpr int TC_STAGES = 4;                       // raw super-blocks in flight (TMA tensor copies)
constexpr int TC_IMG_STAGE = TC_N * Q8K_IMG_BYTES;  // the image blocks of one super-block's 16 columns
constexpr unsigned TC_ERR_WAIT = 0x7c01;

template <int TYPE>
struct TcType {
    static constexpr int PARTS = TYPE == T_Q6_K ? 2 : 1;  // operand parts per half super-block
    static constexpr int STEPS = 2 * PARTS;                // steps per super-block: step st = half * PARTS + part
    static constexpr int TB = TYPE == T_Q4_K ? 1152 : TYPE == T_Q5_K ? 1408 : 1680;  // bytes of one tile block
    static constexpr int ACC_COLS = PARTS * 8 * TC_N;   // TMEM columns of one super-block's lane sums
    static constexpr int TMEM_COLS = 2 * ACC_COLS;      // two super-blocks: the epilogue reads one, the MMAs write the other
    static constexpr int RAW_W = (TC_M / 8) * TB;       // the 16 tile blocks (8 rows each) of one super-block
    static constexpr int RAW = RAW_W + TC_IMG_STAGE;
    static constexpr int OFF_A = TC_STAGES * RAW;       // two operand buffers of each kind
    static constexpr int OFF_B = OFF_A + 2 * TC_A_PART;
    static constexpr int OFF_META = OFF_B + 2 * TC_B_BUF;  // three per-column buffers (super-block % 3)
    static constexpr int OFF_BAR = OFF_META + 3 * TC_N * TC_META * 4;
    static constexpr int SMEM = OFF_BAR + 8 * (1 + TC_STAGES) + 8;
};

struct TcArgs {
    // TMA maps: a matrix as [row group][super-block x tile bytes] (u64 elements, box = 16 row groups x one tile
    // block), the image as [column][super-block x image bytes] (box = 16 columns x one image block)
    CUtensorMap map_w[2];
    CUtensorMap map_img;
    const uint8_t* w[2];  // tile-layout matrices (the second may be null)
    int rows[2];
    float* y[2];          // y[c * rows + r]
    int tiles0;           // 128-row tiles of the first matrix (grid.y beyond it covers the second)
    int nb;               // super-blocks per row
    const uint8_t* img;   // ncols Q8_K image rows of nb blocks, back to back
    int ncols;
};

// instruction descriptor of kind::f16: f16 A and B (K-major), f32 D, M = 128, N = TC_N
constexpr uint32_t TC_IDESC = (1u << 4) | ((uint32_t)(TC_N >> 3) << 17) | ((uint32_t)(TC_M >> 4) << 24);

__device__ __forceinline__ void tc_mma(uint32_t d_tmem, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(da), "l"(db), "r"(TC_IDESC), "r"(accumulate));
}

// four packed bytes b0..b3 (each < 1024) as f16 pairs {1024 + b0, 1024 + b1}, {1024 + b2, 1024 + b3}
__device__ __forceinline__ uint32_t f16_lo(uint32_t v) { return __byte_perm(v, 0x64646464u, 0x5140); }
__device__ __forceinline__ uint32_t f16_hi(uint32_t v) { return __byte_perm(v, 0x64646464u, 0x7362); }

__device__ __forceinline__ uint32_t h2_bits(__half2 h) { return *reinterpret_cast<uint32_t*>(&h); }
__device__ __forceinline__ __half2 bits_h2(uint32_t u) { return *reinterpret_cast<__half2*>(&u); }

// f16 pairs of constants from their bits (a runtime conversion would occupy the XU pipe)
constexpr uint32_t H2_1024 = 0x64006400u, H2_M1024 = 0xE400E400u, H2_1152 = 0x64806480u;

// {s, s} and {-1024 s, -1024 s} in f16 for an unsigned scale byte s < 1024 (exact)
__device__ __forceinline__ void scale_pair(uint32_t s, __half2& sc, __half2& c) {
    const uint32_t b = 0x64006400u | s | (s << 16);
    sc = __hsub2(bits_h2(b), bits_h2(H2_1024));
    c = __hmul2(sc, bits_h2(H2_M1024));
}
// {s, s} in f16 for a signed scale byte (Q6_K): {1024 + (s + 128)} - 1152, exact
__device__ __forceinline__ __half2 signed_scale_pair(uint32_t byte) {
    const uint32_t u = (byte ^ 0x80u) & 0xFFu;
    return __hsub2(bits_h2(0x64006400u | u | (u << 16)), bits_h2(H2_1152));
}

// sc * q for four packed code bytes q (< 1024) with {1024 + q} - 1024 folded into one fma: exact while
// sc * q is (the fma rounds once, and the exact result is representable)
__device__ __forceinline__ uint2 scaled4(uint32_t q, __half2 sc, __half2 c) {
    return make_uint2(h2_bits(__hfma2(bits_h2(f16_lo(q)), sc, c)), h2_bits(__hfma2(bits_h2(f16_hi(q)), sc, c)));
}
// the same for a signed f16 scale (Q6_K): (q + 1024 - 1024) * sc, two exact steps
__device__ __forceinline__ uint2 scaled4_signed(uint32_t q, __half2 sc) {
    const __half2 k = bits_h2(H2_1024);
    return make_uint2(h2_bits(__hmul2(__hsub2(bits_h2(f16_lo(q)), k), sc)),
                      h2_bits(__hmul2(__hsub2(bits_h2(f16_hi(q)), k), sc)));
}

__device__ __forceinline__ void st_shared_v4(uint8_t* p, uint2 a, uint2 b) {
    *reinterpret_cast<uint4*>(p) = make_uint4(a.x, a.y, b.x, b.y);
}

// Dequantise one item of half super-block h: row r of a tile block (in shared memory), lane pair (2tg, 2tg+1),
// into the operand buffer `a` (step l at l * TC_A_PITCH, core column at 2048 per K half, row m at
// (m/8)*128 + (m%8)*16).  Q6_K writes part PART: sc * lo4 (0) or sc * hi2 (1).
template <int TYPE, int PART>
__device__ __forceinline__ void dequant_item(const uint8_t* tile, int r, int tg, int h, uint8_t* a, int m) {
    const int L = r * 4 + tg;
    const uint4 qv = *reinterpret_cast<const uint4*>(tile + h * 512 + L * 16);
    uint8_t* row = a + (m >> 3) * 128 + (m & 7) * 16;
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        // qv: {pair 2h bytes 8tg..+3, pair 2h bytes 8tg+4..+7, pair 2h+1 bytes 8tg..+3, pair 2h+1 bytes 8tg+4..+7};
        // pair p holds sub-block 2p in the low nibbles, 2p+1 in the high nibbles (quant.rs:102-133)
        const uint4 hd = *reinterpret_cast<const uint4*>(tile + (TYPE == T_Q5_K ? 1280 : 1024) + r * 16);
        // the 6-bit scales of sub-blocks 4h..4h+3, one per byte (get_scale_min_k4)
        const uint32_t scb = h == 0 ? (hd.y & 0x3F3F3F3Fu) : ((hd.w & 0x0F0F0F0Fu) | (((hd.y >> 6) & 0x03030303u) << 4));
        __half2 sc[4], cc[4];
#pragma unroll
        for (int i = 0; i < 4; i++) scale_pair((scb >> (8 * i)) & 0xFFu, sc[i], cc[i]);
        uint2 qh = make_uint2(0, 0);
        if constexpr (TYPE == T_Q5_K) qh = *reinterpret_cast<const uint2*>(tile + 1024 + L * 8);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const uint32_t w0 = e ? qv.y : qv.x, w1 = e ? qv.w : qv.z;
            uint32_t q0 = w0 & 0x0F0F0F0Fu, q1 = (w0 >> 4) & 0x0F0F0F0Fu, q2 = w1 & 0x0F0F0F0Fu, q3 = (w1 >> 4) & 0x0F0F0F0Fu;
            if constexpr (TYPE == T_Q5_K) {  // fifth bit: bit s of the qh byte at the same position
                const uint32_t hb = (e ? qh.y : qh.x) >> (4 * h);
                q0 |= (hb & 0x01010101u) << 4;
                q1 |= ((hb >> 1) & 0x01010101u) << 4;
                q2 |= ((hb >> 2) & 0x01010101u) << 4;
                q3 |= ((hb >> 3) & 0x01010101u) << 4;
            }
            uint8_t* step = row + (2 * tg + e) * TC_A_PITCH;
            st_shared_v4(step, scaled4(q0, sc[0], cc[0]), scaled4(q1, sc[1], cc[1]));
            st_shared_v4(step + 2048, scaled4(q2, sc[2], cc[2]), scaled4(q3, sc[3], cc[3]));
        }
    } else {
        // Q6_K (kdot.rs:97-141): qv = {ql chunk 2h bytes 8tg..+3, +4..+7, chunk 2h+1 bytes 8tg..+3, +4..+7}; chunk
        // 2h gives k = 0 (low nibbles) and k = 2 (high), chunk 2h+1 k = 1 and k = 3; the qh bytes of half h hold
        // bits 2k..2k+1; segment 4h + k, scale byte 2 * (4h + k) + lane / 4
        const uint4 scv = *reinterpret_cast<const uint4*>(tile + 1536 + r * 16);
        const uint32_t sw0 = h ? scv.z : scv.x, sw1 = h ? scv.w : scv.y;  // scale bytes 8h .. 8h+7
        uint2 qh = make_uint2(0, 0);
        if constexpr (PART == 1) qh = *reinterpret_cast<const uint2*>(tile + 1024 + L * 16 + h * 8);
#pragma unroll
        for (int e = 0; e < 2; e++) {
            const int lane = 2 * tg + e;
            uint32_t v[4];
            if constexpr (PART == 0) {
                const uint32_t l0 = e ? qv.y : qv.x, l1 = e ? qv.w : qv.z;
                v[0] = l0 & 0x0F0F0F0Fu, v[1] = l1 & 0x0F0F0F0Fu, v[2] = (l0 >> 4) & 0x0F0F0F0Fu, v[3] = (l1 >> 4) & 0x0F0F0F0Fu;
            } else {
                const uint32_t hb = e ? qh.y : qh.x;
#pragma unroll
                for (int k = 0; k < 4; k++) v[k] = (hb >> (2 * k)) & 0x03030303u;
            }
            __half2 sc[4];
#pragma unroll
            for (int k = 0; k < 4; k++) sc[k] = signed_scale_pair((k < 2 ? sw0 : sw1) >> (8 * (2 * (k & 1) + (lane >> 2))));
            uint8_t* step = row + lane * TC_A_PITCH;
            st_shared_v4(step, scaled4_signed(v[0], sc[0]), scaled4_signed(v[1], sc[1]));
            st_shared_v4(step + 2048, scaled4_signed(v[2], sc[2]), scaled4_signed(v[3], sc[3]));
        }
    }
}

// Producer (one thread): super-block sb's 16 tile blocks (one per 8-row group) and 16 image blocks (one per
// column) into raw stage sb % TC_STAGES by two TMA tensor copies, completing on that stage's mbarrier (boxes
// beyond the matrix or the columns land as zeros and count in full).
template <int TYPE>
__device__ __forceinline__ void tc_fetch(const CUtensorMap* map_w, const CUtensorMap* map_img, int g0, int col0, int sb, uint8_t* smem,
                                         uint64_t* full) {
    using C = TcType<TYPE>;
    const int st = sb % TC_STAGES;
    uint8_t* raw = smem + st * C::RAW;
    mbar_expect_tx(full + st, (uint32_t)C::RAW);
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(raw)),
        "l"(map_w), "r"(sb * (C::TB / 8)), "r"(g0), "r"(smem_addr(full + st))
        : "memory");
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
            smem_addr(raw + C::RAW_W)),
        "l"(map_img), "r"(sb * (Q8K_IMG_BYTES / 8)), "r"(col0), "r"(smem_addr(full + st))
        : "memory");
}

// Step gs (super-block gs / STEPS, half and part from gs % STEPS) from its raw stage into operand buffer gs & 1:
// the weights dequantised (A), the activation codes as f16 (B), and with the super-block's first step the
// per-column values of its epilogue.
template <int TYPE>
__device__ __forceinline__ void tc_load(const TcArgs& a, int ngroups, int col0, int gs, uint8_t* smem) {
    using C = TcType<TYPE>;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int sb = gs / C::STEPS, st = gs % C::STEPS, h = st / C::PARTS, part = st % C::PARTS;
    const uint8_t* raw = smem + (sb % TC_STAGES) * C::RAW;
    // weights: warp = row group (8 rows), lane = (row, lane pair)
    {
        const int r = lane >> 2, tg = lane & 3, m = warp * 8 + r;  // lane = the tile block's 16-byte chunk (contiguous reads)
        uint8_t* abuf = smem + C::OFF_A + (gs & 1) * TC_A_PART;
        if (warp < ngroups) {
            if (part == 0) dequant_item<TYPE, 0>(raw + warp * C::TB, r, tg, h, abuf, m);
            else dequant_item<TYPE, 1>(raw + warp * C::TB, r, tg, h, abuf, m);
        } else {  // rows beyond the matrix: zeros (their results are not stored)
            uint8_t* row = abuf + (m >> 3) * 128 + (m & 7) * 16;
#pragma unroll
            for (int e = 0; e < 2; e++) {
                uint8_t* step = row + (2 * tg + e) * TC_A_PITCH;
                *reinterpret_cast<uint4*>(step) = make_uint4(0, 0, 0, 0);
                *reinterpret_cast<uint4*>(step + 2048) = make_uint4(0, 0, 0, 0);
            }
        }
    }
    // activations: thread i < 128 converts 16 codes (lane l, four chunks of half h) of column n
    if (tid < 128) {
        const int n = (tid & 7) + 8 * ((tid >> 3) & 1), l = tid >> 4;
        uint8_t* dst = smem + C::OFF_B + (gs & 1) * TC_B_BUF + l * TC_B_STEP + (n >> 3) * 128 + (n & 7) * 16;
        uint4 v = make_uint4(0x80808080u, 0x80808080u, 0x80808080u, 0x80808080u);  // code 0 after the bias
        if (col0 + n < a.ncols) {
            // image words l*8 + 4h .. +3 = codes (4h + i) * 32 + 4l .. +3 (common.cuh)
            v = *reinterpret_cast<const uint4*>(raw + C::RAW_W + n * Q8K_IMG_BYTES + 32 * l + 16 * h);
            v.x ^= 0x80808080u, v.y ^= 0x80808080u, v.z ^= 0x80808080u, v.w ^= 0x80808080u;
        }
        const __half2 k = bits_h2(H2_1152);  // 1024 + the bias of 128
        auto cv = [&](uint32_t u) {
            return make_uint2(h2_bits(__hsub2(bits_h2(f16_lo(u)), k)), h2_bits(__hsub2(bits_h2(f16_hi(u)), k)));
        };
        st_shared_v4(dst, cv(v.x), cv(v.y));
        st_shared_v4(dst + TC_N * 16, cv(v.z), cv(v.w));
    } else if (st == 0 && tid >= 128 && tid < 128 + TC_N) {
        // per-column values of super-block sb for the epilogue: dx, then the Q4_K/Q5_K q8s or the Q6_K 2 * bsums
        const int n = tid - 128;
        float* meta = reinterpret_cast<float*>(smem + C::OFF_META) + ((sb % 3) * TC_N + n) * TC_META;
        if (col0 + n < a.ncols) {
            const uint8_t* blk = raw + C::RAW_W + n * Q8K_IMG_BYTES;
            meta[0] = *reinterpret_cast<const float*>(blk + Q8K_IMG_D);
            if constexpr (TYPE == T_Q6_K) {
                const uint4 p0 = *reinterpret_cast<const uint4*>(blk + Q8K_IMG_BSP);
                const uint4 p1 = *reinterpret_cast<const uint4*>(blk + Q8K_IMG_BSP + 16);
                const uint32_t pw[8] = {p0.x, p0.y, p0.z, p0.w, p1.x, p1.y, p1.z, p1.w};
#pragma unroll
                for (int g = 0; g < 8; g++) {
                    meta[4 + 2 * g] = __fmul_rn(2.0f, s16f(pw[g] & 0xFFFFu));
                    meta[5 + 2 * g] = __fmul_rn(2.0f, s16f(pw[g] >> 16));
                }
            } else {
                const uint4 p = *reinterpret_cast<const uint4*>(blk + Q8K_IMG_Q8S);
                const uint32_t pw[4] = {p.x, p.y, p.z, p.w};
#pragma unroll
                for (int g = 0; g < 4; g++) {
                    meta[4 + 2 * g] = s16f(pw[g] & 0xFFFFu);
                    meta[5 + 2 * g] = s16f(pw[g] >> 16);
                }
            }
        } else {
            for (int i = 0; i < TC_META; i++) meta[i] = 0.0f;
        }
    }
}

__device__ __forceinline__ void tmem_ld1(uint32_t addr, float& v0) {
    uint32_t r0;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];" : "=r"(r0) : "r"(addr));
    v0 = __uint_as_float(r0);
}
__device__ __forceinline__ void tmem_ld2(uint32_t addr, float& v0, float& v1) {
    uint32_t r0, r1;
    asm volatile("tcgen05.ld.sync.aligned.32x32b.x2.b32 {%0, %1}, [%2];" : "=r"(r0), "=r"(r1) : "r"(addr));
    v0 = __uint_as_float(r0), v1 = __uint_as_float(r1);
}

// The epilogue's per-row values of a super-block (from the row's tile block in the raw stage): the f16 scales
// as f32 and the Q4_K/Q5_K mins or the Q6_K chunk scales.
struct RowVals {
    float dw, dminw;
    float v[16];
};

template <int TYPE>
__device__ __forceinline__ void tc_row_vals(const uint8_t* smem, int sb, int m, RowVals& rv) {
    using C = TcType<TYPE>;
    const uint8_t* tl = smem + (sb % TC_STAGES) * C::RAW + (m >> 3) * C::TB;
    if constexpr (TYPE == T_Q6_K) {
        const uint4 scv = *reinterpret_cast<const uint4*>(tl + 1536 + (m & 7) * 16);
        rv.dw = f16_bits_to_f32(*reinterpret_cast<const uint16_t*>(tl + 1664 + (m & 7) * 2));
        const uint32_t scw[4] = {scv.x, scv.y, scv.z, scv.w};
#pragma unroll
        for (int s = 0; s < 16; s++) rv.v[s] = s8f(scw[s >> 2] >> (8 * (s & 3)));
    } else {
        const uint4 hd = *reinterpret_cast<const uint4*>(tl + (TYPE == T_Q5_K ? 1280 : 1024) + (m & 7) * 16);
        rv.dw = f16_bits_to_f32((uint16_t)(hd.x & 0xFFFFu));
        rv.dminw = f16_bits_to_f32((uint16_t)(hd.x >> 16));
        // the mins of sub-blocks 0..7 (get_scale_min_k4)
        const uint32_t mlo = hd.z & 0x3F3F3F3Fu;
        const uint32_t mhi = ((hd.w >> 4) & 0x0F0F0F0Fu) | (((hd.z >> 6) & 0x03030303u) << 4);
#pragma unroll
        for (int j = 0; j < 4; j++) {
            rv.v[j] = u8f((mlo >> (8 * j)) & 0xFFu);
            rv.v[4 + j] = u8f((mhi >> (8 * j)) & 0xFFu);
        }
    }
}

// Epilogue of super-block sb for this thread's columns I .. I + NCOL - 1 (of its four: row m, columns 4*cb..+3):
// the lane sums from TMEM buffer sb & 1, the reference's f32 steps into the per-lane chains, two lanes (or two
// mins groups) per packed instruction.  acc[i][p] holds lanes 2p, 2p+1; accm[i][p] mins groups 2p, 2p+1.
template <int TYPE, int I, int NCOL>
__device__ __forceinline__ void tc_epilogue_cols(const uint8_t* smem, uint32_t tmem, int sb, int q, int cb, const RowVals& rv,
                                                 float2 (&acc)[4][4], float2 (&accm)[4][2]) {
    using C = TcType<TYPE>;
    const float4* meta = reinterpret_cast<const float4*>(smem + C::OFF_META) + ((sb % 3) * TC_N + 4 * cb + I) * (TC_META / 4);
    const uint32_t trow = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)((sb & 1) * C::ACC_COLS + 4 * cb + I);
    if constexpr (TYPE == T_Q6_K) {
        static_assert(NCOL == 1, "Q6_K takes one column per step");
        float dlo[8], dhi[8];
#pragma unroll
        for (int l = 0; l < 8; l++) {
            tmem_ld1(trow + l * TC_N, dlo[l]);
            tmem_ld1(trow + (8 + l) * TC_N, dhi[l]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        const float d = __fmul_rn(meta[0].x, rv.dw);
        const float4 b0 = meta[1], b1 = meta[2], b2 = meta[3], b3 = meta[4];  // 2 * bsums[0..15]
        const float bs[16] = {b0.x, b0.y, b0.z, b0.w, b1.x, b1.y, b1.z, b1.w, b2.x, b2.y, b2.z, b2.w, b3.x, b3.y, b3.z, b3.w};
#pragma unroll
        for (int p = 0; p < 4; p++) {
            // lanes l = 2p, 2p+1: sumi = (sc*lo) + 16 (sc*hi - 2 (bsum[2l] sc[2l] + bsum[2l+1] sc[2l+1])), one rounding
            const int l = 2 * p;
            const float2 ca = mul2(f2(bs[2 * l], bs[2 * l + 1]), f2(rv.v[2 * l], rv.v[2 * l + 1]));
            const float2 cb2 = mul2(f2(bs[2 * l + 2], bs[2 * l + 3]), f2(rv.v[2 * l + 2], rv.v[2 * l + 3]));
            const float2 c2 = f2(__fadd_rn(ca.x, ca.y), __fadd_rn(cb2.x, cb2.y));
            const float2 t = add2(f2(dhi[l], dhi[l + 1]), f2(-c2.x, -c2.y));
            const float2 sumi = add2(mul2(f2(16.0f, 16.0f), t), f2(dlo[l], dlo[l + 1]));
            acc[I][p] = add2(acc[I][p], mul2(f2(d, d), sumi));
        }
    } else {
        float s[8][NCOL];
#pragma unroll
        for (int l = 0; l < 8; l++) {
            if constexpr (NCOL == 2) tmem_ld2(trow + l * TC_N, s[l][0], s[l][1]);
            else tmem_ld1(trow + l * TC_N, s[l][0]);
        }
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
        for (int j = 0; j < NCOL; j++) {
            const float4* mc = meta + j * (TC_META / 4);
            const float dx = mc[0].x;
            const float4 qa = mc[1], qb = mc[2];  // q8s[0..7]
            const float d = __fmul_rn(dx, rv.dw), dmin = __fmul_rn(-dx, rv.dminw);
            // prod_g = mn[2g] q8s[2g] + mn[2g+1] q8s[2g+1], exact (|prod| < 2^20)
            const float2 p0 = mul2(f2(rv.v[0], rv.v[1]), f2(qa.x, qa.y)), p1 = mul2(f2(rv.v[2], rv.v[3]), f2(qa.z, qa.w));
            const float2 p2 = mul2(f2(rv.v[4], rv.v[5]), f2(qb.x, qb.y)), p3 = mul2(f2(rv.v[6], rv.v[7]), f2(qb.z, qb.w));
            const float2 dm = f2(dmin, dmin), dd = f2(d, d);
            accm[I + j][0] = add2(accm[I + j][0], mul2(dm, f2(__fadd_rn(p0.x, p0.y), __fadd_rn(p1.x, p1.y))));
            accm[I + j][1] = add2(accm[I + j][1], mul2(dm, f2(__fadd_rn(p2.x, p2.y), __fadd_rn(p3.x, p3.y))));
#pragma unroll
            for (int p = 0; p < 4; p++) acc[I + j][p] = add2(acc[I + j][p], mul2(dd, f2(s[2 * p][j], s[2 * p + 1][j])));
        }
    }
}

// The share of super-block sb's epilogue that runs alongside step st of the next super-block: Q4_K/Q5_K two
// columns per step, Q6_K one.
template <int TYPE>
__device__ __forceinline__ void tc_epilogue_step(const uint8_t* smem, uint32_t tmem, int sb, int st, int q, int cb, int m,
                                                 RowVals& rv, float2 (&acc)[4][4], float2 (&accm)[4][2]) {
    if (st == 0) tc_row_vals<TYPE>(smem, sb, m, rv);
    if constexpr (TYPE == T_Q6_K) {
        switch (st) {
        case 0: tc_epilogue_cols<TYPE, 0, 1>(smem, tmem, sb, q, cb, rv, acc, accm); break;
        case 1: tc_epilogue_cols<TYPE, 1, 1>(smem, tmem, sb, q, cb, rv, acc, accm); break;
        case 2: tc_epilogue_cols<TYPE, 2, 1>(smem, tmem, sb, q, cb, rv, acc, accm); break;
        default: tc_epilogue_cols<TYPE, 3, 1>(smem, tmem, sb, q, cb, rv, acc, accm); break;
        }
    } else {
        if (st == 0) tc_epilogue_cols<TYPE, 0, 2>(smem, tmem, sb, q, cb, rv, acc, accm);
        else tc_epilogue_cols<TYPE, 2, 2>(smem, tmem, sb, q, cb, rv, acc, accm);
    }
}

template <int TYPE>
__global__ void __launch_bounds__(TC_THREADS, 1) kq_gemm_tc_kernel(const __grid_constant__ TcArgs a) {
    using C = TcType<TYPE>;
    extern __shared__ __align__(1024) uint8_t smem[];
    uint64_t* mma_bar = reinterpret_cast<uint64_t*>(smem + C::OFF_BAR);
    uint64_t* full = mma_bar + 1;
    uint32_t* tslot = reinterpret_cast<uint32_t*>(full + TC_STAGES);
    __shared__ int s_fail;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

    const int mi = (int)blockIdx.y < a.tiles0 ? 0 : 1;
    const int tile = mi == 0 ? (int)blockIdx.y : (int)blockIdx.y - a.tiles0;
    const CUtensorMap* map_w = mi ? &a.map_w[1] : &a.map_w[0];  // selects, not an indexed parameter array
    const int rows = mi ? a.rows[1] : a.rows[0];
    float* const y = mi ? a.y[1] : a.y[0];
    const int g0 = tile * (TC_M / 8), ngroups = min(TC_M / 8, rows / 8 - g0);
    const int col0 = blockIdx.x * TC_N;
    const int nb = a.nb, nsteps = nb * C::STEPS;
    const bool issuer = warp == TC_COMPUTE / 32;  // the warp that issues the copies and MMAs and waits for the MMAs

    if (warp == 0) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_addr(tslot)),
                     "r"((uint32_t)C::TMEM_COLS));
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
    if (tid == 0) {
        mbar_init1(mma_bar);
        for (int s = 0; s < TC_STAGES; s++) mbar_init1(full + s);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
        s_fail = 0;
    }
    // the activation image is the previous kernel's output
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    __syncthreads();
    int fetched = 0, committed = 0;  // (issuing thread) super-blocks requested, steps committed
    if (issuer && lane == 0)
        for (; fetched < min(TC_STAGES, nb); fetched++) tc_fetch<TYPE>(map_w, &a.map_img, g0, col0, fetched, smem, full);

    // epilogue ownership: row m (TMEM lane), columns 4 * cb .. + 3
    const int q = warp & 3, cb = warp >> 2, m = q * 32 + lane;
    float2 acc[4][4], accm[4][2];
#pragma unroll
    for (int i = 0; i < 4; i++) {
#pragma unroll
        for (int p = 0; p < 4; p++) acc[i][p] = f2(0.0f, 0.0f);
        accm[i][0] = accm[i][1] = f2(0.0f, 0.0f);
    }
    RowVals rv;

    if (!issuer) {
        if (!mbar_wait(full, 0)) s_fail = 1;
        else tc_load<TYPE>(a, ngroups, col0, 0, smem);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // generic-proxy writes -> the tensor core's view
    fence_before_sync();
    __syncthreads();
    fence_after_sync();
    const uint32_t tmem = *tslot;

    for (int gs = 0; gs < nsteps && !s_fail; gs++) {
        const int sb = gs / C::STEPS, st = gs % C::STEPS;
        if (issuer) {
            if (lane == 0) {
                // the stage of super-block sb - 2 is free (dequantised, its epilogue done): super-block sb - 2 + stages
                if (st == 0 && sb >= 2 && sb - 2 + TC_STAGES < nb) tc_fetch<TYPE>(map_w, &a.map_img, g0, col0, fetched++, smem, full);
                const uint32_t abase = smem_addr(smem + C::OFF_A + (gs & 1) * TC_A_PART);
                const uint32_t bbase = smem_addr(smem + C::OFF_B + (gs & 1) * TC_B_BUF);
                const uint32_t dbase = tmem + (uint32_t)((sb & 1) * C::ACC_COLS + (st % C::PARTS) * 8 * TC_N);
                const uint32_t accumulate = st / C::PARTS;  // the second half adds to the first
#pragma unroll
                for (int l = 0; l < 8; l++)
                    tc_mma(dbase + (uint32_t)(l * TC_N), smem_desc(abase + l * TC_A_PITCH, 2048, 128),
                           smem_desc(bbase + l * TC_B_STEP, TC_N * 16, 128), accumulate);
                tc_commit(mma_bar);
                committed = gs + 1;
            }
            __syncwarp();
            // this step's MMAs (their operand buffer is rewritten two steps on, their TMEM read a super-block on)
            if (!__all_sync(0xffffffffu, mbar_wait(mma_bar, (uint32_t)(gs & 1))) && lane == 0) s_fail = 1;
        } else {
            // a share of the previous super-block's epilogue and the next step's operands, alongside this step's MMAs
            if (sb >= 1) tc_epilogue_step<TYPE>(smem, tmem, sb - 1, st, q, cb, m, rv, acc, accm);
            if (gs + 1 < nsteps) {
                const int sbn = (gs + 1) / C::STEPS;
                bool ready = true;
                if ((gs + 1) % C::STEPS == 0) ready = mbar_wait(full + sbn % TC_STAGES, (uint32_t)((sbn / TC_STAGES) & 1));
                if (ready) tc_load<TYPE>(a, ngroups, col0, gs + 1, smem);
                else s_fail = 1;
            }
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        }
        fence_before_sync();
        __syncthreads();
        fence_after_sync();
    }
    if (!s_fail && !issuer) {  // the last super-block's epilogue (its MMAs were waited for in the last step)
#pragma unroll 1
        for (int st = 0; st < C::STEPS; st++) tc_epilogue_step<TYPE>(smem, tmem, nb - 1, st, q, cb, m, rv, acc, accm);
    }

    if (s_fail && issuer && lane == 0) {
        // a wait gave up: record it, then let the copies and MMAs still in flight land (bounded) before the
        // shared memory and TMEM are released
        atomicCAS(&g_tc_error, 0u, TC_ERR_WAIT);
        for (int k = max(0, fetched - TC_STAGES); k < fetched; k++) mbar_wait(full + k % TC_STAGES, (uint32_t)((k / TC_STAGES) & 1));
        if (committed > 0) mbar_wait(mma_bar, (uint32_t)((committed - 1) & 1));
    }
    fence_before_sync();
    __syncthreads();
    if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"((uint32_t)C::TMEM_COLS));
    if (s_fail) return;

    const int row = tile * TC_M + m;
    if (!issuer && row < rows) {
#pragma unroll
        for (int i = 0; i < 4; i++) {
            const int col = col0 + 4 * cb + i;
            if (col < a.ncols) {
                // reduce8 (kdot.rs:20-29): ((l0 + l4) + (l2 + l6)) + ((l1 + l5) + (l3 + l7))
                const float2 r = add2(add2(acc[i][0], acc[i][2]), add2(acc[i][1], acc[i][3]));
                float v = __fadd_rn(r.x, r.y);
                if constexpr (TYPE != T_Q6_K) {  // reduce4: (m0 + m2) + (m1 + m3)
                    const float2 rm = add2(accm[i][0], accm[i][1]);
                    v = __fadd_rn(v, __fadd_rn(rm.x, rm.y));
                }
                y[(size_t)col * rows + row] = v;
            }
        }
    }
}

int g_tc_min_cols = [] {
    // below 16 columns the 4-column GEMV passes are faster (8 columns: 2 passes of a 17408 x 5120 Q4_K pair
    // against one GEMM launch at half the time)
    const char* e = getenv("QDEC_GEMM_TC_MIN_COLS");
    return e ? atoi(e) : 16;
}();

template <int TYPE>
cudaError_t launch_tc(TcArgs& a, int tiles, cudaStream_t s, bool pdl) {
    using C = TcType<TYPE>;
    const size_t wrow = (size_t)a.nb * C::TB;  // bytes of one 8-row group
    for (int i = 0; i < 2; i++)
        if (a.w[i] && !encode_rows(&a.map_w[i], a.w[i], wrow, a.rows[i] / 8, C::TB)) return cudaErrorInvalidValue;
    if (!encode_rows(&a.map_img, a.img, (size_t)a.nb * Q8K_IMG_BYTES, a.ncols, Q8K_IMG_BYTES)) return cudaErrorInvalidValue;
    static bool attr_set[64] = {};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!attr_set[dev]) {
        const cudaError_t e = cudaFuncSetAttribute(kq_gemm_tc_kernel<TYPE>, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
        if (e != cudaSuccess) return e;
        attr_set[dev] = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((a.ncols + TC_N - 1) / TC_N, tiles);
    cfg.blockDim = dim3(TC_THREADS);
    cfg.dynamicSmemBytes = C::SMEM;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kq_gemm_tc_kernel<TYPE>, a);
}

}  // namespace

bool gemm_tc_applies(int type, int ncols) {
    return (type == T_Q4_K_TILE || type == T_Q5_K_TILE || type == T_Q6_K_TILE) && g_tc_min_cols > 0 && ncols >= g_tc_min_cols;
}

void set_gemm_tc_min_cols(int n) { g_tc_min_cols = n; }
int gemm_tc_min_cols() { return g_tc_min_cols; }

cudaError_t launch_gemm_tc(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                           int cols, const void* img, int ncols, cudaStream_t s, bool pdl) {
    if (cols % QK_K || rows_a % 8 || (w_b && rows_b % 8) || ncols <= 0) return cudaErrorInvalidValue;
    if (((uintptr_t)w_a & 15) || (w_b && ((uintptr_t)w_b & 15)) || ((uintptr_t)img & 15)) return cudaErrorInvalidValue;
    TcArgs a{};  // the maps are filled by launch_tc and copied into the launch's parameters
    a.w[0] = w_a, a.rows[0] = rows_a, a.y[0] = y_a;
    a.w[1] = w_b, a.rows[1] = w_b ? rows_b : 0, a.y[1] = y_b;
    a.tiles0 = (rows_a + TC_M - 1) / TC_M;
    const int tiles = a.tiles0 + (w_b ? (rows_b + TC_M - 1) / TC_M : 0);
    a.nb = cols / QK_K;
    a.img = static_cast<const uint8_t*>(img);
    a.ncols = ncols;
    if (tiles == 0) return cudaSuccess;
    const int base = tile_base_type(type);
    if (base == T_Q4_K) return launch_tc<T_Q4_K>(a, tiles, s, pdl);
    if (base == T_Q5_K) return launch_tc<T_Q5_K>(a, tiles, s, pdl);
    if (base == T_Q6_K) return launch_tc<T_Q6_K>(a, tiles, s, pdl);
    return cudaErrorInvalidValue;
}

cudaError_t enqueue_gemm_tc_error_read(unsigned* host_dst, cudaStream_t s) {
    return cudaMemcpyFromSymbolAsync(host_dst, g_tc_error, sizeof(unsigned), 0, cudaMemcpyDeviceToHost, s);
}

unsigned read_gemm_tc_error(bool clear) {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, g_tc_error, sizeof v);
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_tc_error, &z, sizeof z);
    }
    return v;
}

}  // namespace qdec
