// Dequant-GEMV: y[c * rows + r] = W[r] . act_c for up to 4 activation columns, every weight byte read once
// for all columns.  Bit-exact with the reference's scalar kernels:
//
//   K-quants x Q8_K   crates/core/src/kernels/kdot.rs:37-141 (single row) and :176-333 (blocked, same bits)
//   Q8_0/Q4_0 x Q8_0  crates/core/src/kernels/dot.rs:29-64
//   F32 x f32         crates/core/src/kernels/dot.rs:180-198, matvec.rs:270-279
//
// K-quant kernel layout.  Eight consecutive lanes own one weight row; lane l owns the reference's i32 lane l
// (positions 4l..4l+3 of every 32-element sub-block), so its integer lane sum sumi[l] is complete in one
// thread and never crosses lanes.  The lane walks the row's super-blocks in order and keeps the f32
// accumulators acc[l] (and the min lane accm[l], l < 4) in registers, which reproduces the reference's
// "per lane, sequential over super-blocks" f32 chain exactly; the final reduce8 + reduce4 runs on shuffles in
// the reference's order.  Weight bytes stream with ld.global.nc.L1::no_allocate; the activation columns are
// staged once per CTA into shared memory, transposed so lane l reads its 8 code words with two 16-byte loads.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

namespace {

constexpr int GEMV_THREADS = 256;

// Shared-memory image of Q8_K activation columns: per (column, super-block): 64 code words ordered
// [l][s] (word = positions s*32 + 4l .. +3), the f32 scale, and XS int32 sums (q8s for Q4_K/Q5_K, bsums for Q6_K).
template <int XS>
struct Q8KSmem {
    static __host__ __device__ size_t off_xd(int ncols, int nb) { return (size_t)ncols * nb * 256; }
    static __host__ __device__ size_t off_xs(int ncols, int nb) { return (off_xd(ncols, nb) + (size_t)ncols * nb * 4 + 15) & ~(size_t)15; }
    static __host__ __device__ size_t bytes(int ncols, int nb) { return off_xs(ncols, nb) + (size_t)ncols * nb * 4 * XS; }
};

template <int XS>
__device__ void stage_q8k(const uint8_t* __restrict__ act, int ncols, int nb, uint32_t* xq, float* xd, int* xs) {
    const int words = ncols * nb * 73;
    for (int i = threadIdx.x; i < words; i += blockDim.x) {
        const int blk = i / 73, wi = i % 73;
        const uint32_t v = reinterpret_cast<const uint32_t*>(act + (size_t)blk * Q8K_BLOCK_BYTES)[wi];
        if (wi == 0) {
            xd[blk] = __uint_as_float(v);
        } else if (wi <= 64) {
            const int c = wi - 1, l = c & 7, s = c >> 3;
            xq[(size_t)blk * 64 + l * 8 + s] = v;
        } else {
            const int g2 = wi - 65;  // bsums[2*g2] (low half) and bsums[2*g2+1] (high half)
            const int lo = (int)(int16_t)(v & 0xffff), hi = (int)(int16_t)(v >> 16);
            if (XS == 8) {
                xs[blk * 8 + g2] = (int)(int16_t)(lo + hi);  // q8s = bsums[2s] + bsums[2s+1] (q8k.rs:185-193)
            } else {
                xs[blk * 16 + 2 * g2] = lo;
                xs[blk * 16 + 2 * g2 + 1] = hi;
            }
        }
    }
}

__device__ __forceinline__ int byte_of(uint32_t w, int i) { return (int)((w >> (8 * i)) & 0xff); }

__device__ __forceinline__ uint32_t ld_u32_2aligned(const uint8_t* p) {
    // 4 bytes at a 2-byte aligned address: two aligned loads and a funnel shift when misaligned
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    if ((a & 3) == 0) return ld_nc_u32(p);
    const uint32_t lo = ld_nc_u32(reinterpret_cast<const void*>(a - 2));
    const uint32_t hi = ld_nc_u32(reinterpret_cast<const void*>(a + 2));
    return __funnelshift_r(lo, hi, 16);
}

// Reduce the 8 lanes of a row group in the reference's order.  `v` is lane l's f32 lane value; returns the
// reduce8 result on every lane of the group: ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)).
__device__ __forceinline__ float group_reduce8(float v) {
    const float a = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 4, 8));  // l: l + (l+4), valid l<4
    const float b = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 2, 8));  // l: (l,l+4)+(l+2,l+6), valid l<2
    const float c = __fadd_rn(b, __shfl_down_sync(0xffffffffu, b, 1, 8));  // l0 + l1
    return __shfl_sync(0xffffffffu, c, 0, 8);
}
// ((m0+m2)+(m1+m3)) of lanes 0..3 of the group.
__device__ __forceinline__ float group_reduce4(float v) {
    const float a = __fadd_rn(v, __shfl_down_sync(0xffffffffu, v, 2, 8));
    const float b = __fadd_rn(a, __shfl_down_sync(0xffffffffu, a, 1, 8));
    return __shfl_sync(0xffffffffu, b, 0, 8);
}

// Raw bytes of one weight super-block that lane l needs (positions 4l..4l+3 of every 32-element chunk).
template <int TYPE>
struct KBlk;
template <>
struct KBlk<T_Q4_K> {
    uint4 hdr;        // f16 d, f16 dmin, 12 bytes of packed 6-bit scales/mins
    uint32_t cw[4];   // code bytes 16 + 32p + 4l .. +3: sub-block 2p (low nibbles) and 2p+1 (high)
};
template <>
struct KBlk<T_Q5_K> {
    uint4 hdr;
    uint32_t cw[4];   // ql bytes 48 + 32p + 4l .. +3
    uint32_t qh;      // qh bytes 16 + 4l .. +3: bit s = fifth bit of sub-block s
};
template <>
struct KBlk<T_Q6_K> {
    uint32_t ql[4];   // ql bytes 32i + 4l .. +3 (i = 2*half + (k & 1))
    uint32_t qh[2];   // qh bytes 128 + 32*half + 4l .. +3
    uint32_t sc[4];   // the 16 int8 scales
    uint32_t d;       // f16 d (low half)
};

template <int TYPE>
__device__ __forceinline__ void load_blk(const uint8_t* blk, int l, KBlk<TYPE>& b) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        constexpr int QO = TYPE == T_Q4_K ? 16 : 48;
        b.hdr = ld_nc_u128(blk);
#pragma unroll
        for (int p = 0; p < 4; p++) b.cw[p] = ld_nc_u32(blk + QO + 32 * p + 4 * l);
        if constexpr (TYPE == T_Q5_K) b.qh = ld_nc_u32(blk + 16 + 4 * l);
    } else {
#pragma unroll
        for (int i = 0; i < 4; i++) b.ql[i] = ld_u32_2aligned(blk + 32 * i + 4 * l);
#pragma unroll
        for (int h = 0; h < 2; h++) b.qh[h] = ld_u32_2aligned(blk + 128 + 32 * h + 4 * l);
#pragma unroll
        for (int i = 0; i < 4; i++) b.sc[i] = ld_u32_2aligned(blk + 192 + 4 * i);
        b.d = ld_nc_u16(blk + 208);
    }
}

// The f32 terms lane l adds for one (row, super-block): main[n] = (dx * dw) * f32(sumi[l]) and, for
// Q4_K/Q5_K lanes l < 4, mins[n] = (-dx * dminw) * f32(prod[l]) (kdot.rs:37-76, :97-141).
template <int TYPE, int NC>
__device__ __forceinline__ void kblk_terms(const KBlk<TYPE>& b, int l, const uint32_t* __restrict__ xq_sb, int xq_stride,
                                           const float* __restrict__ xd_sb, int xd_stride, const int* __restrict__ xs_sb,
                                           int xs_stride, float (&tmain)[NC], float (&tmin)[NC]) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        // get_scale_min_k4 for the 8 sub-blocks, one byte per sub-block (quant.rs:45-51)
        const uint32_t sc03 = b.hdr.y & 0x3F3F3F3Fu;
        const uint32_t m03 = b.hdr.z & 0x3F3F3F3Fu;
        const uint32_t sc47 = (b.hdr.w & 0x0F0F0F0Fu) | ((b.hdr.y >> 2) & 0x30303030u);
        const uint32_t m47 = ((b.hdr.w >> 4) & 0x0F0F0F0Fu) | ((b.hdr.z >> 2) & 0x30303030u);
        const float dw = f16_bits_to_f32((uint16_t)(b.hdr.x & 0xffff));
        const float dminw = f16_bits_to_f32((uint16_t)(b.hdr.x >> 16));
        int sc[8];
#pragma unroll
        for (int s = 0; s < 4; s++) sc[s] = byte_of(sc03, s), sc[s + 4] = byte_of(sc47, s);
        uint32_t code[8];
#pragma unroll
        for (int p = 0; p < 4; p++) {
            code[2 * p] = b.cw[p] & 0x0F0F0F0Fu;
            code[2 * p + 1] = (b.cw[p] >> 4) & 0x0F0F0F0Fu;
        }
        if constexpr (TYPE == T_Q5_K) {
#pragma unroll
            for (int s = 0; s < 8; s++) code[s] |= ((b.qh >> s) & 0x01010101u) << 4;
        }
        const int lm = l & 3;  // min lane l (l < 4): sub-blocks 2l, 2l+1
        const int mA = (lm < 2) ? byte_of(m03, 2 * lm) : byte_of(m47, 2 * lm - 4);
        const int mB = (lm < 2) ? byte_of(m03, 2 * lm + 1) : byte_of(m47, 2 * lm - 3);
#pragma unroll
        for (int n = 0; n < NC; n++) {
            const uint4* xp = reinterpret_cast<const uint4*>(xq_sb + (size_t)n * xq_stride + l * 8);
            const uint4 x0 = xp[0], x1 = xp[1];
            const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int sumi = 0;
#pragma unroll
            for (int s = 0; s < 8; s++) sumi += sc[s] * __dp4a((int)code[s], (int)xw[s], 0);
            const float dx = xd_sb[n * xd_stride];
            tmain[n] = __fmul_rn(__fmul_rn(dx, dw), (float)sumi);
            const int2 q8 = *reinterpret_cast<const int2*>(xs_sb + (size_t)n * xs_stride + 2 * lm);
            tmin[n] = __fmul_rn(__fmul_rn(-dx, dminw), (float)(mA * q8.x + mB * q8.y));
        }
    } else {
        const float dw = f16_bits_to_f32((uint16_t)(b.d & 0xffff));
        uint32_t code[8];
        int scl[8];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int k = 0; k < 4; k++) {
                const uint32_t lo = (b.ql[2 * h + (k & 1)] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
                const uint32_t hi = ((b.qh[h] >> (2 * k)) & 0x03030303u) << 4;
                code[4 * h + k] = lo | hi;
                const int si = h * 8 + 2 * k + (l >> 2);  // sc[2k + l/16] of half h
                scl[4 * h + k] = (int)(int8_t)byte_of(b.sc[si >> 2], si & 3);
            }
        const int s0 = (int)(int8_t)byte_of(b.sc[(2 * l) >> 2], (2 * l) & 3);
        const int s1 = (int)(int8_t)byte_of(b.sc[(2 * l + 1) >> 2], (2 * l + 1) & 3);
#pragma unroll
        for (int n = 0; n < NC; n++) {
            const uint4* xp = reinterpret_cast<const uint4*>(xq_sb + (size_t)n * xq_stride + l * 8);
            const uint4 x0 = xp[0], x1 = xp[1];
            const uint32_t xw[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
            int sumi = 0;
#pragma unroll
            for (int c = 0; c < 8; c++) sumi += scl[c] * __dp4a((int)code[c], (int)xw[c], 0);
            const int2 bs = *reinterpret_cast<const int2*>(xs_sb + (size_t)n * xs_stride + 2 * l);
            sumi -= 32 * (bs.x * s0 + bs.y * s1);
            tmain[n] = __fmul_rn(__fmul_rn(xd_sb[n * xd_stride], dw), (float)sumi);
            tmin[n] = 0.0f;
        }
    }
}

// K-quant GEMV.  A warp owns R rows; its 32 lanes are 4 super-block slots x 8 lane groups: in round j the
// lane (slot k, group l) takes super-block 4j + k of each of the R rows and computes the f32 terms of the
// reference's lane l.  The per-lane f32 accumulators are then advanced in super-block order by shuffling the
// 4 slots' terms in (the reference's sequential chain, kdot.rs:72-74), so every bit matches while 32 lanes
// keep 4 x R super-blocks in flight; the next round's blocks are loaded before this round is computed.
// Lane l's activation words are read from shared memory once per super-block and reused for the R rows.
template <int TYPE, int NC, int R>
__global__ void __launch_bounds__(GEMV_THREADS)
kq_gemv_kernel(const uint8_t* __restrict__ w, int rows, int nb, const uint8_t* __restrict__ act, float* __restrict__ y) {
    constexpr int BB = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 210;
    constexpr int XS = TYPE == T_Q6_K ? 16 : 8;
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* xq = reinterpret_cast<uint32_t*>(smem);
    float* xd = reinterpret_cast<float*>(smem + Q8KSmem<XS>::off_xd(NC, nb));
    int* xs = reinterpret_cast<int*>(smem + Q8KSmem<XS>::off_xs(NC, nb));
    stage_q8k<XS>(act, NC, nb, xq, xd, xs);
    __syncthreads();

    const int lane = threadIdx.x & 31, l = lane & 7, slot = lane >> 3;
    const size_t row_bytes = (size_t)nb * BB;
    const int warps_total = gridDim.x * (GEMV_THREADS / 32);
    for (int grp = blockIdx.x * (GEMV_THREADS / 32) + (threadIdx.x >> 5); grp * R < rows; grp += warps_total) {
        const int row0 = grp * R;
        const uint8_t* wr[R];
#pragma unroll
        for (int r = 0; r < R; r++) wr[r] = w + (size_t)min(row0 + r, rows - 1) * row_bytes;
        float acc[R][NC], accm[R][NC];
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int n = 0; n < NC; n++) acc[r][n] = 0.0f, accm[r][n] = 0.0f;

        KBlk<TYPE> cur[R], nxt[R];
        if (slot < nb) {
#pragma unroll
            for (int r = 0; r < R; r++) load_blk<TYPE>(wr[r] + (size_t)slot * BB, l, cur[r]);
        }
        for (int base = 0; base < nb; base += 4) {
            const int sb = base + slot;
            if (sb + 4 < nb) {
#pragma unroll
                for (int r = 0; r < R; r++) load_blk<TYPE>(wr[r] + (size_t)(sb + 4) * BB, l, nxt[r]);
            }
            float tmain[R][NC], tmin[R][NC];
            if (sb < nb) {
#pragma unroll
                for (int r = 0; r < R; r++)
                    kblk_terms<TYPE, NC>(cur[r], l, xq + (size_t)sb * 64, nb * 64, xd + sb, nb, xs + (size_t)sb * XS, nb * XS,
                                         tmain[r], tmin[r]);
            } else {
#pragma unroll
                for (int r = 0; r < R; r++)
#pragma unroll
                    for (int n = 0; n < NC; n++) tmain[r][n] = 0.0f, tmin[r][n] = 0.0f;
            }
            const int kmax = min(4, nb - base);
            for (int k = 0; k < kmax; k++) {
#pragma unroll
                for (int r = 0; r < R; r++)
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        acc[r][n] = __fadd_rn(acc[r][n], __shfl_sync(0xffffffffu, tmain[r][n], k * 8 + l));
                        if constexpr (TYPE != T_Q6_K)
                            accm[r][n] = __fadd_rn(accm[r][n], __shfl_sync(0xffffffffu, tmin[r][n], k * 8 + l));
                    }
            }
#pragma unroll
            for (int r = 0; r < R; r++) cur[r] = nxt[r];
        }
        // every slot now holds the same lane accumulators; slot 0 reduces in the reference's order
#pragma unroll
        for (int r = 0; r < R; r++)
#pragma unroll
            for (int n = 0; n < NC; n++) {
                float v = group_reduce8(acc[r][n]);
                if constexpr (TYPE != T_Q6_K) v = __fadd_rn(v, group_reduce4(accm[r][n]));
                if (lane == 0 && row0 + r < rows) y[(size_t)n * rows + row0 + r] = v;
            }
    }
}

// ---------------------------------------------------------------------------- Q8_0 / Q4_0 x Q8_0

// Activation staging: per (column, block): 8 code words (aligned) and the f32 scale.
__device__ void stage_q8_0(const uint8_t* __restrict__ act, int ncols, int nblk, uint32_t* xq, float* xd) {
    const int total = ncols * nblk;
    for (int i = threadIdx.x; i < total * 17; i += blockDim.x) {
        const int blk = i / 17, hw = i % 17;  // 17 half-words per 34-byte block
        const uint8_t* b = act + (size_t)blk * Q8_0_BLOCK_BYTES;
        const uint16_t v = (uint16_t)(b[2 * hw] | (b[2 * hw + 1] << 8));
        if (hw == 0) {
            xd[blk] = f16_bits_to_f32(v);
        } else {
            reinterpret_cast<uint16_t*>(xq)[(size_t)blk * 16 + (hw - 1)] = v;
        }
    }
}

// One warp per row; lane i takes blocks 2i, 2i+1 of every 64-block chunk (one 4-byte aligned pair), and the
// per-block f32 terms are chained left to right over the whole row by lane 0 (dot.rs:29-63 order).
template <int TYPE, int NC>
__global__ void __launch_bounds__(GEMV_THREADS, 1)
q80_gemv_kernel(const uint8_t* __restrict__ w, int rows, int nblk, const uint8_t* __restrict__ act, float* __restrict__ y) {
    constexpr int BB = TYPE == T_Q8_0 ? 34 : 18;
    constexpr int PW = TYPE == T_Q8_0 ? 17 : 9;  // 32-bit words in a pair of blocks
    extern __shared__ __align__(16) uint8_t smem[];
    uint32_t* xq = reinterpret_cast<uint32_t*>(smem);
    float* xd = reinterpret_cast<float*>(smem + (size_t)NC * nblk * 32);
    stage_q8_0(act, NC, nblk, xq, xd);
    __syncthreads();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const size_t row_bytes = (size_t)nblk * BB;
    const int warps = GEMV_THREADS / 32;
    for (int row = blockIdx.x * warps + warp; row < rows; row += gridDim.x * warps) {
        const uint8_t* wrow = w + (size_t)row * row_bytes;
        float acc[NC];
#pragma unroll
        for (int n = 0; n < NC; n++) acc[n] = 0.0f;
        for (int b0 = 0; b0 < nblk; b0 += 64) {
            const int bA = b0 + 2 * lane;
            float tA[NC], tB[NC];
#pragma unroll
            for (int n = 0; n < NC; n++) tA[n] = 0.0f, tB[n] = 0.0f;
            if (bA < nblk) {  // nblk is even for every shape here (cols % 64 == 0 is checked by the host)
                const uint8_t* p = wrow + (size_t)bA * BB;
                uint32_t pw[PW];
#pragma unroll
                for (int i = 0; i < PW; i++) pw[i] = __ldg(reinterpret_cast<const uint32_t*>(p) + i);
                const float dA = f16_bits_to_f32((uint16_t)(pw[0] & 0xffff));
                float dB;
                uint32_t cA[8], cB[8];
                if constexpr (TYPE == T_Q8_0) {
                    dB = f16_bits_to_f32((uint16_t)(pw[8] >> 16));
#pragma unroll
                    for (int i = 0; i < 8; i++) cA[i] = __funnelshift_r(pw[i], pw[i + 1], 16), cB[i] = pw[9 + i];
                } else {
                    dB = f16_bits_to_f32((uint16_t)(pw[4] >> 16));
                    uint32_t qA[4], qB[4];
#pragma unroll
                    for (int i = 0; i < 4; i++) qA[i] = __funnelshift_r(pw[i], pw[i + 1], 16), qB[i] = pw[5 + i];
                    // element j < 16: low nibble of byte j; j >= 16: high nibble of byte j-16; value q - 8
#pragma unroll
                    for (int i = 0; i < 4; i++) {
                        cA[i] = __vsub4(qA[i] & 0x0F0F0F0Fu, 0x08080808u);
                        cA[i + 4] = __vsub4((qA[i] >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                        cB[i] = __vsub4(qB[i] & 0x0F0F0F0Fu, 0x08080808u);
                        cB[i + 4] = __vsub4((qB[i] >> 4) & 0x0F0F0F0Fu, 0x08080808u);
                    }
                }
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint4* xa = reinterpret_cast<const uint4*>(xq + ((size_t)n * nblk + bA) * 8);
                    const uint4 a0 = xa[0], a1 = xa[1], b0v = xa[2], b1v = xa[3];
                    const uint32_t xA[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
                    const uint32_t xB[8] = {b0v.x, b0v.y, b0v.z, b0v.w, b1v.x, b1v.y, b1v.z, b1v.w};
                    int iA = 0, iB = 0;
#pragma unroll
                    for (int i = 0; i < 8; i++) iA = __dp4a((int)cA[i], (int)xA[i], iA), iB = __dp4a((int)cB[i], (int)xB[i], iB);
                    tA[n] = __fmul_rn(__fmul_rn(dA, xd[n * nblk + bA]), (float)iA);
                    tB[n] = __fmul_rn(__fmul_rn(dB, xd[n * nblk + bA + 1]), (float)iB);
                }
            }
            // left-to-right chain over this chunk's blocks (lane order = block order)
            const int nlanes = min(32, (nblk - b0) / 2);
#pragma unroll
            for (int n = 0; n < NC; n++) {
                float a = acc[n];
                for (int i = 0; i < nlanes; i++) {
                    a = __fadd_rn(a, __shfl_sync(0xffffffffu, tA[n], i));
                    a = __fadd_rn(a, __shfl_sync(0xffffffffu, tB[n], i));
                }
                acc[n] = a;
            }
        }
        if (lane == 0)
#pragma unroll
            for (int n = 0; n < NC; n++) y[(size_t)n * rows + row] = acc[n];
    }
}

// ---------------------------------------------------------------------------- F32 x f32

// One CTA per (row, column) of up to two matrices sharing the input columns (rows [0, rows_a) of w_a, then
// [0, rows_b) of w_b): thread j computes the 32-element partial of block j (left to right), then thread 0 chains
// the block partials in order and adds the tail partial (dot.rs:180-198).  All partials of a row are computed at
// once, so the row costs one load latency plus the two dependent chains.
// `early`: x was written at least two kernels before this one (never by the kernel right before it), so the
// whole product runs before griddepcontrol.wait, alongside the preceding kernel.
__global__ void __launch_bounds__(256) f32_gemv_kernel(const float* __restrict__ w_a, int rows_a, float* __restrict__ y_a,
                                                       const float* __restrict__ w_b, int rows_b, float* __restrict__ y_b,
                                                       int cols, const float* __restrict__ x, int early) {
    __shared__ float part[512];
    if (!early) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
    const int n = blockIdx.y;
    const bool first = (int)blockIdx.x < rows_a;
    const int row = first ? blockIdx.x : blockIdx.x - rows_a;
    const float* wr = (first ? w_a : w_b) + (size_t)row * cols;
    const float* xr = x + (size_t)n * cols;
    const int nfull = cols / 32, nparts = nfull + (cols % 32 ? 1 : 0);
    const bool vec = (cols % 4) == 0;
    for (int j = threadIdx.x; j < nparts; j += blockDim.x) {
        const int lo = j * 32, hi = min(cols, lo + 32);
        float p = 0.0f;
        if (vec && hi - lo == 32) {
            float4 wv[8], xv[8];
#pragma unroll
            for (int q = 0; q < 8; q++) wv[q] = __ldg(reinterpret_cast<const float4*>(wr + lo) + q), xv[q] = __ldg(reinterpret_cast<const float4*>(xr + lo) + q);
#pragma unroll
            for (int q = 0; q < 8; q++) {
                p = __fadd_rn(p, __fmul_rn(wv[q].x, xv[q].x));
                p = __fadd_rn(p, __fmul_rn(wv[q].y, xv[q].y));
                p = __fadd_rn(p, __fmul_rn(wv[q].z, xv[q].z));
                p = __fadd_rn(p, __fmul_rn(wv[q].w, xv[q].w));
            }
        } else {
            for (int i = lo; i < hi; i++) p = __fadd_rn(p, __fmul_rn(wr[i], xr[i]));
        }
        part[j] = p;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        float acc = 0.0f;
#pragma unroll 8
        for (int j = 0; j < nfull; j++) acc = __fadd_rn(acc, part[j]);
        acc = __fadd_rn(acc, nparts > nfull ? part[nfull] : 0.0f);  // the tail partial, +0 when empty (dot.rs:194-197)
        (first ? y_a : y_b)[(size_t)n * (first ? rows_a : rows_b) + row] = acc;
    }
    if (early) {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    }
}

int g_num_sms = 0;

template <int TYPE, int NC, int R>
cudaError_t launch_kq_r(const uint8_t* w, int rows, int nb, const void* act, float* y, cudaStream_t s) {
    constexpr int XS = TYPE == T_Q6_K ? 16 : 8;
    const size_t smem = Q8KSmem<XS>::bytes(NC, nb);
    auto kern = kq_gemv_kernel<TYPE, NC, R>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int per_sm = 0;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GEMV_THREADS, smem);
    if (e != cudaSuccess) return e;
    const int warps = GEMV_THREADS / 32;
    const int groups = (rows + R - 1) / R;
    const int grid = std::max(1, std::min((groups + warps - 1) / warps, num_sms() * std::max(1, per_sm)));
    kern<<<grid, GEMV_THREADS, smem, s>>>(w, rows, nb, (const uint8_t*)act, y);
    return cudaGetLastError();
}

// Rows per warp: 4 when there are enough rows to give every SM a few dozen warps (activation reads from shared
// memory then amortise over 4 rows), fewer for short matrices so the grid still covers the GPU.
template <int TYPE, int NC>
cudaError_t launch_kq(const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    const int nb = cols / QK_K;
    const int sms = num_sms();
    static const int forced_r = [] {
        const char* e = getenv("QDEC_GEMV_ROWS_PER_WARP");  // tuning override: 1, 2 or 4
        return e ? atoi(e) : 0;
    }();
    if (forced_r == 4) return launch_kq_r<TYPE, NC, 4>(w, rows, nb, act, y, s);
    if (forced_r == 2) return launch_kq_r<TYPE, NC, 2>(w, rows, nb, act, y, s);
    if (forced_r == 1) return launch_kq_r<TYPE, NC, 1>(w, rows, nb, act, y, s);
    if (rows >= sms * 16 * 4) return launch_kq_r<TYPE, NC, 4>(w, rows, nb, act, y, s);
    if (rows >= sms * 16 * 2) return launch_kq_r<TYPE, NC, 2>(w, rows, nb, act, y, s);
    return launch_kq_r<TYPE, NC, 1>(w, rows, nb, act, y, s);
}

template <int TYPE, int NC>
cudaError_t launch_q80(const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    const int nblk = cols / 32;
    const size_t smem = (size_t)NC * nblk * 36;
    auto kern = q80_gemv_kernel<TYPE, NC>;
    static int per_sm = 0;  // per instantiation, at the largest shared-memory size: set once (graph capture safe)
    if (per_sm == 0) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
        if (e != cudaSuccess) return e;
        e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GEMV_THREADS, 48 * 1024);
        if (e != cudaSuccess) return e;
        per_sm = std::max(1, per_sm);
    }
    if (smem > 200 * 1024) return cudaErrorInvalidValue;
    const int warps = GEMV_THREADS / 32;
    const int grid = std::max(1, std::min((rows + warps - 1) / warps, num_sms() * per_sm));
    kern<<<grid, GEMV_THREADS, smem, s>>>(w, rows, nblk, (const uint8_t*)act, y);
    return cudaGetLastError();
}

template <int NC>
cudaError_t launch_f32(const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    return launch_gemv_f32_pair((const float*)w, rows, y, nullptr, 0, nullptr, cols, (const float*)act, NC, s);
}

int g_gemv_impl = [] {
    const char* e = getenv("QDEC_GEMV_IMPL");  // tuning override: 2 (raw-Q8_K register path)
    return e ? atoi(e) : 0;
}();

// Raw-activation dispatch: block_q8_K / block_q8_0 / f32 columns in the reference's layouts.
template <int NC>
cudaError_t dispatch_type(int type, const uint8_t* w, int rows, int cols, const void* act, float* y, cudaStream_t s) {
    switch (type) {
    case T_Q4_K: return launch_kq<T_Q4_K, NC>(w, rows, cols, act, y, s);
    case T_Q5_K: return launch_kq<T_Q5_K, NC>(w, rows, cols, act, y, s);
    case T_Q6_K: return launch_kq<T_Q6_K, NC>(w, rows, cols, act, y, s);
    case T_Q8_0: return launch_q80<T_Q8_0, NC>(w, rows, cols, act, y, s);
    case T_Q4_0: return launch_q80<T_Q4_0, NC>(w, rows, cols, act, y, s);
    case T_F32: return launch_f32<NC>(w, rows, cols, act, y, s);
    default: return cudaErrorInvalidValue;
    }
}

}  // namespace

bool pdl_enabled() {
    static const bool on = [] {
        const char* e = getenv("QDEC_PDL");
        return !(e && e[0] == '0');
    }();
    return on;
}

int num_sms() {
    if (g_num_sms == 0) {
        int dev = 0;
        cudaGetDevice(&dev);
        cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
        if (g_num_sms <= 0) g_num_sms = 148;
    }
    return g_num_sms;
}

size_t act_row_bytes(int type, int cols) {
    if (is_kquant(type)) return (size_t)(cols / QK_K) * Q8K_BLOCK_BYTES;
    if (type == T_Q8_0 || type == T_Q4_0) return (size_t)(cols / 32) * Q8_0_BLOCK_BYTES;
    return (size_t)cols * 4;
}

void set_gemv_impl(int impl) { g_gemv_impl = impl; }
int gemv_impl() { return g_gemv_impl; }

cudaError_t launch_gemv(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y, cudaStream_t s) {
    if (rows <= 0) return cudaSuccess;
    // columns beyond 4 are processed in groups of at most 4 (each weight byte then read once per group)
    int c0 = 0;
    while (c0 < ncols) {
        const int nc = std::min(4, ncols - c0);
        const void* a = (const uint8_t*)act + act_row_bytes(type, cols) * c0;
        float* yy = y + (size_t)c0 * rows;
        cudaError_t e;
        switch (nc) {
        case 1: e = dispatch_type<1>(type, w, rows, cols, a, yy, s); break;
        case 2: e = dispatch_type<2>(type, w, rows, cols, a, yy, s); break;
        case 3: e = dispatch_type<3>(type, w, rows, cols, a, yy, s); break;
        default: e = dispatch_type<4>(type, w, rows, cols, a, yy, s); break;
        }
        if (e != cudaSuccess) return e;
        c0 += nc;
    }
    return cudaSuccess;
}

cudaError_t launch_gemv_f32_pair(const float* w_a, int rows_a, float* y_a, const float* w_b, int rows_b, float* y_b, int cols,
                                 const float* x, int ncols, cudaStream_t s, bool early) {
    if (cols > 512 * 32) return cudaErrorInvalidValue;  // 512 partials of shared memory: cols <= 16384
    if (rows_a + rows_b == 0 || ncols == 0) return cudaSuccess;
    if (!early) {
        f32_gemv_kernel<<<dim3(rows_a + rows_b, ncols), 256, 0, s>>>(w_a, rows_a, y_a, w_b, rows_b, y_b, cols, x, 0);
        return cudaGetLastError();
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(rows_a + rows_b, ncols);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, f32_gemv_kernel, w_a, rows_a, y_a, w_b, rows_b, y_b, cols, x, 1);
}

cudaError_t launch_quantize_q8k(const float* x, int n, int rows, uint8_t* out, cudaStream_t s) {
    const long long blocks = (long long)rows * (n / QK_K);
    if (blocks == 0) return cudaSuccess;
    const int threads = 256;
    const long long want = (blocks * 32 + threads - 1) / threads;
    const int grid = (int)std::min<long long>(want, (long long)num_sms() * 16);
    q8k_quantize_kernel<<<grid, threads, 0, s>>>(x, n, rows, out);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8k_image(const float* x, int n, int rows, uint8_t* img, cudaStream_t s) {
    const long long blocks = (long long)rows * (n / QK_K);
    if (blocks == 0) return cudaSuccess;
    const int threads = 256;
    const long long want = (blocks * 32 + threads - 1) / threads;
    const int grid = (int)std::min<long long>(want, (long long)num_sms() * 16);
    q8k_image_kernel<<<grid, threads, 0, s>>>(x, n, rows, img);
    return cudaGetLastError();
}

cudaError_t launch_q8k_raw_to_image(const uint8_t* raw, long long nblocks, uint8_t* img, cudaStream_t s) {
    if (nblocks == 0) return cudaSuccess;
    const int threads = 256;
    const int grid = (int)std::min<long long>((nblocks * 32 + threads - 1) / threads, (long long)num_sms() * 16);
    q8k_raw_to_image_kernel<<<grid, threads, 0, s>>>(raw, nblocks, img);
    return cudaGetLastError();
}

cudaError_t launch_quantize_q8_0(const float* x, int n, int rows, uint8_t* out, cudaStream_t s) {
    const long long blocks = (long long)rows * (n / 32);
    if (blocks == 0) return cudaSuccess;
    const int threads = 256;
    const long long want = (blocks * 32 + threads - 1) / threads;
    const int grid = (int)std::min<long long>(want, (long long)num_sms() * 16);
    q8_0_quantize_kernel<<<grid, threads, 0, s>>>(x, n, rows, out);
    return cudaGetLastError();
}

cudaError_t launch_dequant_rows(int type, const uint8_t* w, size_t row_bytes, int n, const int32_t* ids, int nids,
                                float* out, cudaStream_t s) {
    const long long total = (long long)n * nids;
    if (total == 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((total + 255) / 256, (long long)num_sms() * 8);
    dequant_rows_kernel<<<grid, 256, 0, s>>>(type, w, row_bytes, n, ids, nids, out);
    return cudaGetLastError();
}

}  // namespace qdec
