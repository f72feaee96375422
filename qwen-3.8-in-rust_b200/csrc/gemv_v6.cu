// K-quant GEMV over the engine's Q8_K device image (Q4_K, Q5_K, and Q6_K in the split layout), bit-exact with
// crates/core/src/kernels/kdot.rs:37-141 and its blocked form :176-333.
//
// Work split.  GL of the reference's eight i32 lanes (lane g = positions 4g..4g+3 of every 32-element chunk) live
// in one thread, so 8/GL threads share a weight row; each thread owns R consecutive rows with the same lanes,
// which lets one load of the activation words serve R rows.  A CTA is one warp (4*GL*R rows), so the block
// scheduler spreads the rows evenly over the SMs whatever their count.  Each thread walks its rows'
// super-blocks in order and keeps the f32 lane accumulators in registers -- the reference's "per lane,
// sequential over super-blocks" chain -- with one gather + reduce8 + reduce4 per row at the end.
//
// Data movement.  Weight bytes stream from HBM into registers with 8/16-byte non-allocating loads (the threads of
// a row cover whole 32-byte sectors), D super-blocks ahead in a register ring (the loop is unrolled by D so each
// ring slot is a fixed register set).  Activations are read from the Q8_K image (L1-resident: every warp of an SM
// reads the same few KB), 32 contiguous bytes per lane.
//
// Integer work.  For Q4_K/Q5_K the per-sub-block scale multiply either stays on the integer pipe (IMAD into a
// sum biased by 1.5 * 2^23, read back as a float with one FADD) or moves to the FP32 pipe (the dp4a result,
// biased, read as a float; then sc * t accumulated by FFMA) -- every partial sum is an integer below 2^24, so
// both give the reference's exact i32 lane sum.
//
// Programmatic dependent launch: the first D super-blocks of weights are requested before griddepcontrol.wait,
// so the weight stream of this GEMV overlaps the tail of the kernel that produced its activations.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

__device__ unsigned int g_kernel_error = 0;  // first code recorded by a device-side bounded wait that gave up

namespace {

constexpr int MAGIC_I = 0x4B400000;       // bits of 12582912.0f = 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;    // float(bits + k) - MAGIC_F == k exactly for |k| < 2^22

__device__ __forceinline__ uint2 ld_nc_u64(const void* p) {
    uint2 v;
    asm volatile("ld.global.nc.L1::no_allocate.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "l"(p));
    return v;
}

template <int N>
__device__ __forceinline__ void ldg_words(const uint8_t* p, uint32_t (&w)[N]) {
    if constexpr (N == 2) {
        const uint2 a = ld_nc_u64(p);
        w[0] = a.x, w[1] = a.y;
    } else {
        w[0] = ld_nc_u32(p);
    }
}

template <int TYPE, int GL>
struct Frag;
template <int GL>
struct Frag<T_Q4_K, GL> {
    uint4 hdr;              // f16 d, f16 dmin, 12 bytes of 6-bit scales/mins
    uint32_t qs[4][GL];     // bytes 16 + 32p + 4g: sub-block 2p (low nibbles), 2p+1 (high nibbles)
};
template <int GL>
struct Frag<T_Q5_K, GL> {
    uint4 hdr;
    uint32_t qs[4][GL];     // bytes 48 + 32p + 4g
    uint32_t qh[GL];        // bytes 16 + 4g: bit s = fifth bit of sub-block s
};
template <int GL>
struct Frag<T_Q6_K, GL> {   // split layout: 208-byte blocks [ql 128 | qh 64 | scales 16], d array after
    uint4 sc;
    uint32_t ql[4][GL];     // bytes 32i + 4g
    uint32_t qh[2][GL];     // bytes 128 + 32h + 4g
    uint32_t d;             // f16 d (low half)
};

template <int TYPE>
struct BlkB {
    static constexpr int value = TYPE == T_Q4_K ? 144 : TYPE == T_Q5_K ? 176 : 208;
};

template <int TYPE, int GL>
__device__ __forceinline__ void load_frag(const uint8_t* blk, const uint16_t* dptr, int g0, Frag<TYPE, GL>& f) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        constexpr int QO = TYPE == T_Q4_K ? 16 : 48;
        f.hdr = ld_nc_u128(blk);
#pragma unroll
        for (int p = 0; p < 4; p++) ldg_words<GL>(blk + QO + 32 * p + 4 * g0, f.qs[p]);
        if constexpr (TYPE == T_Q5_K) ldg_words<GL>(blk + 16 + 4 * g0, f.qh);
    } else {
        f.sc = ld_nc_u128(blk + 192);
#pragma unroll
        for (int i = 0; i < 4; i++) ldg_words<GL>(blk + 32 * i + 4 * g0, f.ql[i]);
#pragma unroll
        for (int h = 0; h < 2; h++) ldg_words<GL>(blk + 128 + 32 * h + 4 * g0, f.qh[h]);
        f.d = ld_nc_u16(dptr);
    }
}

__device__ __forceinline__ int dp2a_lo(uint32_t a16x2, uint32_t b8x4, int c) {
    int r;
    asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(r) : "r"(a16x2), "r"(b8x4), "r"(c));
    return r;
}
__device__ __forceinline__ float biased_to_f32(int v) { return __fsub_rn(__int_as_float(v), MAGIC_F); }

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Row-dependent decode of one super-block, shared by every column.
template <int TYPE, int GL>
struct Dec;
template <int GL>
struct Dec<T_Q4_K, GL> {
    uint32_t code[8][GL];
    int sc[8];
    float scf[8];
    uint32_t mpair;
    float dw, dminw;
};
template <int GL>
struct Dec<T_Q5_K, GL> : Dec<T_Q4_K, GL> {};
template <int GL>
struct Dec<T_Q6_K, GL> {
    uint32_t code[8][GL];
    int scl[8][GL];
    uint32_t spair[GL];
    float dw;
};

template <int TYPE, int GL, int FPS>
__device__ __forceinline__ void decode(const Frag<TYPE, GL>& f, int tg, Dec<TYPE, GL>& o) {
    const int g0 = tg * GL;
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const uint32_t sc03 = f.hdr.y & 0x3F3F3F3Fu;
        const uint32_t sc47 = (f.hdr.w & 0x0F0F0F0Fu) | ((f.hdr.y >> 2) & 0x30303030u);
        o.dw = f16_bits_to_f32((uint16_t)(f.hdr.x & 0xffff));
        o.dminw = f16_bits_to_f32((uint16_t)(f.hdr.x >> 16));
#pragma unroll
        for (int s = 0; s < 4; s++) {
            o.sc[s] = (int)((sc03 >> (8 * s)) & 0xff);
            o.sc[s + 4] = (int)((sc47 >> (8 * s)) & 0xff);
        }
        if constexpr (FPS != 0) {
#pragma unroll
            for (int s = (FPS == 2 ? 4 : 0); s < 8; s++) o.scf[s] = __fsub_rn(__int_as_float(0x4B000000 | o.sc[s]), 8388608.0f);
        }
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int gi = 0; gi < GL; gi++) {
                o.code[2 * p][gi] = f.qs[p][gi] & 0x0F0F0F0Fu;
                o.code[2 * p + 1][gi] = (f.qs[p][gi] >> 4) & 0x0F0F0F0Fu;
                if constexpr (TYPE == T_Q5_K) {
                    o.code[2 * p][gi] |= ((f.qh[gi] >> (2 * p)) & 0x01010101u) << 4;
                    o.code[2 * p + 1][gi] |= ((f.qh[gi] >> (2 * p + 1)) & 0x01010101u) << 4;
                }
            }
        // min lane i (sub-blocks 2i, 2i+1; kdot.rs:60-66) belongs to thread tg = i of the row
        const int mi = tg & 3;
        const uint32_t mw = mi < 2 ? (f.hdr.z & 0x3F3F3F3Fu) : (((f.hdr.w >> 4) & 0x0F0F0F0Fu) | ((f.hdr.z >> 2) & 0x30303030u));
        o.mpair = mw >> (16 * (mi & 1));  // bytes 0, 1 = the mins of sub-blocks 2i, 2i+1
    } else {
        o.dw = f16_bits_to_f32((uint16_t)(f.d & 0xffff));
        const uint32_t scw[4] = {f.sc.x, f.sc.y, f.sc.z, f.sc.w};
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int gi = 0; gi < GL; gi++) {
                    const uint32_t lo = (f.ql[2 * h + (k & 1)][gi] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
                    const uint32_t hi = ((f.qh[h][gi] >> (2 * k)) & 0x03030303u) << 4;
                    o.code[4 * h + k][gi] = lo | hi;
                    const int si = h * 8 + 2 * k + ((g0 + gi) >> 2);  // sc[2k + l/16] of half h
                    o.scl[4 * h + k][gi] = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xff);
                }
#pragma unroll
        for (int gi = 0; gi < GL; gi++) {
            const int g = g0 + gi;
            o.spair[gi] = scw[g >> 1] >> (16 * (g & 1));  // int8 scales 2g, 2g+1 in bytes 0, 1
        }
    }
}

// The reference's integer lane sum of lane gi (as an exact f32) for one column.
template <int TYPE, int GL, int FPS>
__device__ __forceinline__ float lane_sum(const Dec<TYPE, GL>& o, const uint32_t* xw, int gi, uint32_t bsp) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        if constexpr (FPS == 1) {
            float a = 0.0f;
#pragma unroll
            for (int s = 0; s < 8; s++)
                a = __fmaf_rn(o.scf[s], biased_to_f32(__dp4a((int)o.code[s][gi], (int)xw[gi * 8 + s], MAGIC_I)), a);
            return a;  // every partial sum is an integer of magnitude < 2^23: exact
        } else if constexpr (FPS == 2) {
            // sub-blocks 0..3 on the integer pipe, 4..7 on the FP32 pipe; each half's sum is below 2^22 in
            // magnitude (Q5_K: 4 * 63 * 4 * 31 * 127 < 2^22), so both halves and their sum are exact
            int sumi = MAGIC_I;
#pragma unroll
            for (int s = 0; s < 4; s++) sumi += o.sc[s] * __dp4a((int)o.code[s][gi], (int)xw[gi * 8 + s], 0);
            float a = 0.0f;
#pragma unroll
            for (int s = 4; s < 8; s++)
                a = __fmaf_rn(o.scf[s], biased_to_f32(__dp4a((int)o.code[s][gi], (int)xw[gi * 8 + s], MAGIC_I)), a);
            return __fadd_rn(biased_to_f32(sumi), a);
        } else if constexpr (TYPE == T_Q4_K) {
            int sumi = MAGIC_I;  // |sum| <= 8 * 63 * 4 * 15 * 127 < 2^22
#pragma unroll
            for (int s = 0; s < 8; s++) sumi += o.sc[s] * __dp4a((int)o.code[s][gi], (int)xw[gi * 8 + s], 0);
            return biased_to_f32(sumi);
        } else {
            int sumi = 0;
#pragma unroll
            for (int s = 0; s < 8; s++) sumi += o.sc[s] * __dp4a((int)o.code[s][gi], (int)xw[gi * 8 + s], 0);
            return (float)sumi;
        }
    } else {
        int sumi = 0;
#pragma unroll
        for (int c = 0; c < 8; c++) sumi += o.scl[c][gi] * __dp4a((int)o.code[c][gi], (int)xw[gi * 8 + c], 0);
        sumi -= 32 * dp2a_lo(bsp, o.spair[gi], 0);  // bsums[2g] sc[2g] + bsums[2g+1] sc[2g+1] (kdot.rs:128-133)
        return (float)sumi;
    }
}

template <int TYPE, int NC, int GL, int R, int D, int FPS>
__global__ void __launch_bounds__(32)
kq_gemv_v6_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ dsplit, int rows, int nb,
                  const uint8_t* __restrict__ img, float* __restrict__ y) {
    constexpr int TPR = 8 / GL, RPW = 32 / TPR, BB = BlkB<TYPE>::value;
    constexpr bool Q6 = TYPE == T_Q6_K;
    const int lane = threadIdx.x, rs = lane / TPR, tg = lane % TPR, g0 = tg * GL;
    const int row0 = (blockIdx.x * RPW + rs) * R;
    const size_t row_bytes = (size_t)nb * BB;
    const uint8_t* wr[R];
    const uint16_t* dr[R];
#pragma unroll
    for (int j = 0; j < R; j++) {
        const int r = min(row0 + j, rows - 1);
        wr[j] = w + (size_t)r * row_bytes;
        dr[j] = Q6 ? dsplit + (size_t)r * nb : nullptr;
    }
    Frag<TYPE, GL> ring[D][R];
#pragma unroll
    for (int d = 0; d < D; d++)
        if (d < nb) {
#pragma unroll
            for (int j = 0; j < R; j++) load_frag<TYPE, GL>(wr[j] + (size_t)d * BB, Q6 ? dr[j] + d : nullptr, g0, ring[d][j]);
        }

    griddep_wait();  // the activation image is the previous kernel's output
    griddep_launch();

    float acc[NC][R][GL], accm[NC][R];
#pragma unroll
    for (int n = 0; n < NC; n++)
#pragma unroll
        for (int j = 0; j < R; j++) {
#pragma unroll
            for (int gi = 0; gi < GL; gi++) acc[n][j][gi] = 0.0f;
            accm[n][j] = 0.0f;
        }

    for (int sb0 = 0; sb0 < nb; sb0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int sb = sb0 + d;
            if (sb < nb) {
                Dec<TYPE, GL> dec[R];
#pragma unroll
                for (int j = 0; j < R; j++) decode<TYPE, GL, FPS>(ring[d][j], tg, dec[j]);
                if (sb + D < nb) {
#pragma unroll
                    for (int j = 0; j < R; j++)
                        load_frag<TYPE, GL>(wr[j] + (size_t)(sb + D) * BB, Q6 ? dr[j] + sb + D : nullptr, g0, ring[d][j]);
                }
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint8_t* xb = img + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
                    uint32_t xw[8 * GL];
#pragma unroll
                    for (int c = 0; c < 2 * GL; c++) {
                        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xb + 32 * g0) + c);
                        xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                    }
                    const float dx = __ldg(reinterpret_cast<const float*>(xb + Q8K_IMG_D));
                    uint32_t aux[GL];
                    if constexpr (Q6) {
#pragma unroll
                        for (int gi = 0; gi < GL; gi++) aux[gi] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_BSP) + g0 + gi);
                    } else {
                        aux[0] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S) + (tg & 3));
                    }
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        const float dd = __fmul_rn(dx, dec[j].dw);
#pragma unroll
                        for (int gi = 0; gi < GL; gi++)
                            acc[n][j][gi] = __fadd_rn(acc[n][j][gi], __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dec[j], xw, gi, Q6 ? aux[gi] : 0u)));
                        if constexpr (!Q6) {
                            if (tg < 4) {  // mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1], |.| < 2^22
                                const float prod = biased_to_f32(dp2a_lo(aux[0], dec[j].mpair, MAGIC_I));
                                accm[n][j] = __fadd_rn(accm[n][j], __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod));
                            }
                        }
                    }
                }
            }
        }
    }
    // gather the row's 8 main and 4 min lanes; reduce in the reference's order
    // ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) + ((m0+m2)+(m1+m3))
    const int base = rs * TPR;
#pragma unroll
    for (int n = 0; n < NC; n++)
#pragma unroll
        for (int j = 0; j < R; j++) {
            float l8[8], m4[4];
#pragma unroll
            for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[n][j][g % GL], base + g / GL);
#pragma unroll
            for (int m = 0; m < 4; m++) m4[m] = __shfl_sync(0xffffffffu, accm[n][j], base + m);
            const int row = row0 + j;
            if (tg == 0 && row < rows) {
                float v = reduce8(l8);
                if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
                y[(size_t)n * rows + row] = v;
            }
        }
}

// ------------------------------------------------------------------------------------------------ tiles
// Tile layout: 8 rows x one super-block of a K-quant matrix stored as one "tile block" of 8 * (block bytes), in
// the order the GEMV's 32 threads read it (thread L = 4 * row + tg holds reference lanes 2tg, 2tg+1), so every
// warp-wide load of the weight stream is 512 contiguous bytes and a warp's whole stream is one contiguous range:
//   Q4_K (1152 B): [2 x 32 x 16 B] code chunks  -- chunk j of thread L = qs bytes 16+32*2j+8tg..+8 | 16+32*(2j+1)+8tg..+8
//                  [8 x 16 B]      headers (d, dmin, scales) of rows 0..7
//   Q5_K (1408 B): [2 x 32 x 16 B] code chunks from offset 48, [32 x 8 B] qh bytes 16+8tg..+8, [8 x 16 B] headers
//   Q6_K (1680 B): [3 x 32 x 16 B] chunk 0: ql 8tg | ql 32+8tg; chunk 1: ql 64+8tg | ql 96+8tg; chunk 2: qh 128+8tg |
//                  qh 160+8tg; [8 x 16 B] scales; [8 x 2 B] f16 d
// Tiles follow each other, a tile's super-blocks in order: tile t, super-block sb at (t * nb + sb) * TILE_BYTES.
template <int TYPE>
struct TileB {
    static constexpr int value = TYPE == T_Q4_K ? 1152 : TYPE == T_Q5_K ? 1408 : 1680;
};

template <int TYPE>
__device__ __forceinline__ void load_frag_tile(const uint8_t* ts, int L, int rs, Frag<TYPE, 2>& f) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const uint4 c0 = ld_nc_u128(ts + L * 16), c1 = ld_nc_u128(ts + 512 + L * 16);
        f.qs[0][0] = c0.x, f.qs[0][1] = c0.y, f.qs[1][0] = c0.z, f.qs[1][1] = c0.w;
        f.qs[2][0] = c1.x, f.qs[2][1] = c1.y, f.qs[3][0] = c1.z, f.qs[3][1] = c1.w;
        if constexpr (TYPE == T_Q5_K) {
            const uint2 h = ld_nc_u64(ts + 1024 + L * 8);
            f.qh[0] = h.x, f.qh[1] = h.y;
            f.hdr = ld_nc_u128(ts + 1280 + rs * 16);
        } else {
            f.hdr = ld_nc_u128(ts + 1024 + rs * 16);
        }
    } else {
        const uint4 c0 = ld_nc_u128(ts + L * 16), c1 = ld_nc_u128(ts + 512 + L * 16), c2 = ld_nc_u128(ts + 1024 + L * 16);
        f.ql[0][0] = c0.x, f.ql[0][1] = c0.y, f.ql[1][0] = c0.z, f.ql[1][1] = c0.w;
        f.ql[2][0] = c1.x, f.ql[2][1] = c1.y, f.ql[3][0] = c1.z, f.ql[3][1] = c1.w;
        f.qh[0][0] = c2.x, f.qh[0][1] = c2.y, f.qh[1][0] = c2.z, f.qh[1][1] = c2.w;
        f.sc = ld_nc_u128(ts + 1536 + rs * 16);
        f.d = ld_nc_u16(ts + 1664 + rs * 2);
    }
}

// One warp = R tiles (8R rows); thread L = 4 * rs + tg owns row rs of each tile and lanes 2tg, 2tg+1.
template <int TYPE, int NC, int R, int D, int FPS>
__global__ void __launch_bounds__(32)
kq_gemv_tile_kernel(const uint8_t* __restrict__ w, int rows, int nb, const uint8_t* __restrict__ img, float* __restrict__ y) {
    constexpr int GL = 2, TB = TileB<TYPE>::value;
    constexpr bool Q6 = TYPE == T_Q6_K;
    const int lane = threadIdx.x, rs = lane >> 2, tg = lane & 3, g0 = tg * GL;
    const int tiles = rows / 8;
    const uint8_t* wt[R];
#pragma unroll
    for (int j = 0; j < R; j++) wt[j] = w + (size_t)min(blockIdx.x * R + j, tiles - 1) * nb * TB;
    Frag<TYPE, GL> ring[D][R];
#pragma unroll
    for (int d = 0; d < D; d++)
        if (d < nb) {
#pragma unroll
            for (int j = 0; j < R; j++) load_frag_tile<TYPE>(wt[j] + (size_t)d * TB, lane, rs, ring[d][j]);
        }

    griddep_wait();  // the activation image is the previous kernel's output
    griddep_launch();

    float acc[NC][R][GL], accm[NC][R];
#pragma unroll
    for (int n = 0; n < NC; n++)
#pragma unroll
        for (int j = 0; j < R; j++) {
#pragma unroll
            for (int gi = 0; gi < GL; gi++) acc[n][j][gi] = 0.0f;
            accm[n][j] = 0.0f;
        }

    for (int sb0 = 0; sb0 < nb; sb0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int sb = sb0 + d;
            if (sb < nb) {
                Dec<TYPE, GL> dec[R];
#pragma unroll
                for (int j = 0; j < R; j++) decode<TYPE, GL, FPS>(ring[d][j], tg, dec[j]);
                if (sb + D < nb) {
#pragma unroll
                    for (int j = 0; j < R; j++) load_frag_tile<TYPE>(wt[j] + (size_t)(sb + D) * TB, lane, rs, ring[d][j]);
                }
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint8_t* xb = img + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
                    uint32_t xw[8 * GL];
#pragma unroll
                    for (int c = 0; c < 2 * GL; c++) {
                        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xb + 32 * g0) + c);
                        xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                    }
                    const float dx = __ldg(reinterpret_cast<const float*>(xb + Q8K_IMG_D));
                    uint32_t aux[GL];
                    if constexpr (Q6) {
                        const uint2 a2 = __ldg(reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP) + tg);
                        aux[0] = a2.x, aux[1] = a2.y;
                    } else {
                        aux[0] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S) + tg);
                    }
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        const float dd = __fmul_rn(dx, dec[j].dw);
#pragma unroll
                        for (int gi = 0; gi < GL; gi++)
                            acc[n][j][gi] = __fadd_rn(acc[n][j][gi], __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dec[j], xw, gi, Q6 ? aux[gi] : 0u)));
                        if constexpr (!Q6) {  // mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1], |.| < 2^22
                            const float prod = biased_to_f32(dp2a_lo(aux[0], dec[j].mpair, MAGIC_I));
                            accm[n][j] = __fadd_rn(accm[n][j], __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod));
                        }
                    }
                }
            }
        }
    }
    const int base = rs * 4;
#pragma unroll
    for (int n = 0; n < NC; n++)
#pragma unroll
        for (int j = 0; j < R; j++) {
            float l8[8], m4[4];
#pragma unroll
            for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[n][j][g % GL], base + g / GL);
#pragma unroll
            for (int m = 0; m < 4; m++) m4[m] = __shfl_sync(0xffffffffu, accm[n][j], base + m);
            const int tile = blockIdx.x * R + j;
            if (tg == 0 && tile < tiles) {
                float v = reduce8(l8);
                if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
                y[(size_t)n * rows + tile * 8 + rs] = v;
            }
        }
}

template <int TYPE, int NC, int R, int D, int FPS>
cudaError_t launch_tile(const uint8_t* w, int rows, int nb, const void* img, float* y, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows / 8 + R - 1) / R);
    cfg.blockDim = dim3(32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kq_gemv_tile_kernel<TYPE, NC, R, D, FPS>, w, rows, nb, (const uint8_t*)img, y);
}

// Split super-block range: a CTA of S warps shares R tiles; warp s computes super-blocks s, s+S, s+2S, ... and
// writes each super-block's f32 lane terms -- d * f32(sumi) per reference lane and (-d_x * dmin) * f32(prod) per
// min lane, every column -- to shared memory; after each window of S super-blocks, the chain owners (one
// thread per (tile, column, row, lane)) add the window's terms in super-block order.  The additions are the
// reference's own sequence acc = ((0 + t_0) + t_1) + ... per lane, so the bits do not change; S times as many
// warps stream the same rows, which short matrices (5120 rows) need to keep enough bytes in flight.
template <int NC, int R>
struct SplitTerms {  // one window buffer: [S][R][NC][8 rows][12] (8 main lanes, then 4 min lanes)
    static constexpr int PER_SB = R * NC * 8 * 12;
};

template <int TYPE, int NC, int R, int D, int S, int FPS, int MINB = 1, bool XP = false, bool XR = false>
__global__ void __launch_bounds__(32 * S, MINB)
kq_gemv_split_kernel(const uint8_t* __restrict__ w_a, int rows_a, float* __restrict__ y_a, const uint8_t* __restrict__ w_b,
                     int rows_b, float* __restrict__ y_b, int nb, const uint8_t* __restrict__ img) {
    constexpr int GL = 2, TB = TileB<TYPE>::value, PER_SB = SplitTerms<NC, R>::PER_SB;
    constexpr bool Q6 = TYPE == T_Q6_K;
    constexpr int CHAINS = R * NC * 8 * (Q6 ? 8 : 12);
    constexpr int CPT = (CHAINS + 32 * S - 1) / (32 * S);  // chains per thread
    __shared__ float terms[2][S * PER_SB];
    __shared__ float fin[R * NC * 8 * 12];
    const int lane = threadIdx.x & 31, ws = threadIdx.x >> 5, rs = lane >> 2, tg = lane & 3, g0 = tg * GL;
    // two matrices sharing the input columns: CTAs of the first, then of the second (w_b may be null)
    const int ctas_a = (rows_a / 8 + R - 1) / R;
    const bool second = (int)blockIdx.x >= ctas_a;
    const uint8_t* w = second ? w_b : w_a;
    const int rows = second ? rows_b : rows_a;
    float* y = second ? y_b : y_a;
    const int bid = second ? (int)blockIdx.x - ctas_a : (int)blockIdx.x;
    const int tiles = rows / 8;
    const uint8_t* wt[R];
#pragma unroll
    for (int j = 0; j < R; j++) wt[j] = w + (size_t)min(bid * R + j, tiles - 1) * nb * TB;
    Frag<TYPE, GL> ring[D][R];
#pragma unroll
    for (int d = 0; d < D; d++) {
        const int sb = ws + d * S;
        if (sb < nb) {
#pragma unroll
            for (int j = 0; j < R; j++) load_frag_tile<TYPE>(wt[j] + (size_t)sb * TB, lane, rs, ring[d][j]);
        }
    }

    griddep_wait();
    griddep_launch();

    float cacc[CPT];
#pragma unroll
    for (int c = 0; c < CPT; c++) cacc[c] = 0.0f;

    const int nwin = (nb + S - 1) / S;
    for (int w0 = 0; w0 < nwin; w0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int win = w0 + d;
            if (win < nwin) {  // uniform over the CTA
                const int sb = win * S + ws;
                float* tb = terms[win & 1] + ws * PER_SB;
                if (sb < nb) {
                  if constexpr (XR) {
                    // every column's activation words for this super-block stay in registers while the R tiles
                    // are decoded one at a time against them (one load of each word serves R rows)
                    uint32_t xw[NC][8 * GL];
                    float xdv[NC];
                    uint32_t xav[NC][GL];
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const uint8_t* xb = img + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
#pragma unroll
                        for (int c = 0; c < 2 * GL; c++) {
                            const uint4 v = __ldg(reinterpret_cast<const uint4*>(xb + 32 * g0) + c);
                            xw[n][4 * c] = v.x, xw[n][4 * c + 1] = v.y, xw[n][4 * c + 2] = v.z, xw[n][4 * c + 3] = v.w;
                        }
                        xdv[n] = __ldg(reinterpret_cast<const float*>(xb + Q8K_IMG_D));
                        if constexpr (Q6) {
                            const uint2 a2 = __ldg(reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP) + tg);
                            xav[n][0] = a2.x, xav[n][1] = a2.y;
                        } else {
                            xav[n][0] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S) + tg);
                        }
                    }
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        Dec<TYPE, GL> dj;
                        decode<TYPE, GL, FPS>(ring[d][j], tg, dj);
                        if (sb + D * S < nb) load_frag_tile<TYPE>(wt[j] + (size_t)(sb + D * S) * TB, lane, rs, ring[d][j]);
#pragma unroll
                        for (int n = 0; n < NC; n++) {
                            const float dd = __fmul_rn(xdv[n], dj.dw);
                            float* t = tb + ((j * NC + n) * 8 + rs) * 12;
                            float2 mt;
                            mt.x = __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dj, xw[n], 0, Q6 ? xav[n][0] : 0u));
                            mt.y = __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dj, xw[n], 1, Q6 ? xav[n][1] : 0u));
                            *reinterpret_cast<float2*>(t + 2 * tg) = mt;
                            if constexpr (!Q6) {
                                const float prod = biased_to_f32(dp2a_lo(xav[n][0], dj.mpair, MAGIC_I));
                                t[8 + tg] = __fmul_rn(__fmul_rn(-xdv[n], dj.dminw), prod);
                            }
                        }
                    }
                  } else {
                    Dec<TYPE, GL> dec[R];
#pragma unroll
                    for (int j = 0; j < R; j++) decode<TYPE, GL, FPS>(ring[d][j], tg, dec[j]);
                    if (sb + D * S < nb) {
#pragma unroll
                        for (int j = 0; j < R; j++) load_frag_tile<TYPE>(wt[j] + (size_t)(sb + D * S) * TB, lane, rs, ring[d][j]);
                    }
                    // activation words of column n + 1 are requested while column n computes (XP)
                    uint4 xv[2][2 * GL];
                    float xd[2];
                    uint32_t xa[2][GL];
                    auto load_x = [&](int n, int b) {
                        const uint8_t* xb = img + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
#pragma unroll
                        for (int c = 0; c < 2 * GL; c++) xv[b][c] = __ldg(reinterpret_cast<const uint4*>(xb + 32 * g0) + c);
                        xd[b] = __ldg(reinterpret_cast<const float*>(xb + Q8K_IMG_D));
                        if constexpr (Q6) {
                            const uint2 a2 = __ldg(reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP) + tg);
                            xa[b][0] = a2.x, xa[b][1] = a2.y;
                        } else {
                            xa[b][0] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S) + tg);
                        }
                    };
                    if constexpr (XP) load_x(0, 0);
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const int b = XP ? (n & 1) : 0;
                        if constexpr (XP) {
                            if (n + 1 < NC) load_x(n + 1, b ^ 1);
                        } else {
                            load_x(n, 0);
                        }
                        uint32_t xw[8 * GL];
#pragma unroll
                        for (int c = 0; c < 2 * GL; c++) {
                            const uint4 v = xv[b][c];
                            xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                        }
                        const float dx = xd[b];
                        uint32_t aux[GL];
#pragma unroll
                        for (int gi = 0; gi < GL; gi++) aux[gi] = xa[b][gi];
#pragma unroll
                        for (int j = 0; j < R; j++) {
                            const float dd = __fmul_rn(dx, dec[j].dw);
                            float* t = tb + ((j * NC + n) * 8 + rs) * 12;
                            float2 mt;
                            mt.x = __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dec[j], xw, 0, Q6 ? aux[0] : 0u));
                            mt.y = __fmul_rn(dd, lane_sum<TYPE, GL, FPS>(dec[j], xw, 1, Q6 ? aux[1] : 0u));
                            *reinterpret_cast<float2*>(t + 2 * tg) = mt;
                            if constexpr (!Q6) {
                                const float prod = biased_to_f32(dp2a_lo(aux[0], dec[j].mpair, MAGIC_I));
                                t[8 + tg] = __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod);
                            }
                        }
                    }
                  }
                }
                __syncthreads();
                // chain owners: add this window's terms in super-block order
                const float* tw = terms[win & 1];
                const int nsb = min(S, nb - win * S);
#pragma unroll
                for (int c = 0; c < CPT; c++) {
                    const int ci = threadIdx.x + c * 32 * S;
                    if (ci < CHAINS) {
                        // chain ci = ((j * NC + n) * 8 + r) * LPC + lane, LPC = 12 (Q4_K/Q5_K) or 8 (Q6_K)
                        constexpr int LPC = Q6 ? 8 : 12;
                        const int slot = (ci / LPC) * 12 + ci % LPC;
                        float a = cacc[c];
#pragma unroll
                        for (int k = 0; k < S; k++)
                            if (k < nsb) a = __fadd_rn(a, tw[k * PER_SB + slot]);
                        cacc[c] = a;
                    }
                }
            }
        }
    }
    // final reduce per (tile, column, row): reduce8 of the main lanes + reduce4 of the min lanes
#pragma unroll
    for (int c = 0; c < CPT; c++) {
        const int ci = threadIdx.x + c * 32 * S;
        constexpr int LPC = Q6 ? 8 : 12;
        if (ci < CHAINS) fin[(ci / LPC) * 12 + ci % LPC] = cacc[c];
    }
    __syncthreads();
    for (int o = threadIdx.x; o < R * NC * 8; o += 32 * S) {
        const int r = o % 8, n = (o / 8) % NC, j = o / (8 * NC);
        const float* f = fin + o * 12;
        float v = reduce8(f);
        if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(f[8], f[10]), __fadd_rn(f[9], f[11])));
        const int tile = bid * R + j;
        if (tile < tiles) y[(size_t)n * rows + tile * 8 + r] = v;
    }
}

template <int TYPE, int NC, int R, int D, int S, int FPS, int MINB = 1, bool XP = false, bool XR = false>
cudaError_t launch_split(const uint8_t* w, int rows, int nb, const void* img, float* y, cudaStream_t s, bool pdl,
                         const uint8_t* w_b = nullptr, int rows_b = 0, float* y_b = nullptr) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows / 8 + R - 1) / R + (w_b ? (rows_b / 8 + R - 1) / R : 0));
    cfg.blockDim = dim3(32 * S);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kq_gemv_split_kernel<TYPE, NC, R, D, S, FPS, MINB, XP, XR>, w, rows, y, w_b, rows_b, y_b, nb,
                              (const uint8_t*)img);
}

// ---------------------------------------------------------------------------------- bulk-copy split kernel
// The split kernel with the weights staged through shared memory: each warp keeps D tile blocks of its own
// super-blocks in flight with cp.async.bulk copies (no multicast; completion on one mbarrier per stage) instead of
// in registers, so the bytes in flight no longer cost registers and more warps fit on an SM.  Waits are bounded:
// a wait that gives up records a code in the device error word, the warp stops computing (its outputs are not
// written) and, before leaving, waits -- again bounded -- for the copies it still has in flight.
constexpr uint32_t BULK_WAIT_LIMIT = 1u << 26;

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
    for (uint32_t it = 0; it < BULK_WAIT_LIMIT; it++)
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

template <int TYPE>
__device__ __forceinline__ void load_frag_smem(const uint8_t* ts, int L, int rs, Frag<TYPE, 2>& f) {
    auto ld16 = [](const uint8_t* p) { return *reinterpret_cast<const uint4*>(p); };
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const uint4 c0 = ld16(ts + L * 16), c1 = ld16(ts + 512 + L * 16);
        f.qs[0][0] = c0.x, f.qs[0][1] = c0.y, f.qs[1][0] = c0.z, f.qs[1][1] = c0.w;
        f.qs[2][0] = c1.x, f.qs[2][1] = c1.y, f.qs[3][0] = c1.z, f.qs[3][1] = c1.w;
        if constexpr (TYPE == T_Q5_K) {
            const uint2 h = *reinterpret_cast<const uint2*>(ts + 1024 + L * 8);
            f.qh[0] = h.x, f.qh[1] = h.y;
            f.hdr = ld16(ts + 1280 + rs * 16);
        } else {
            f.hdr = ld16(ts + 1024 + rs * 16);
        }
    } else {
        const uint4 c0 = ld16(ts + L * 16), c1 = ld16(ts + 512 + L * 16), c2 = ld16(ts + 1024 + L * 16);
        f.ql[0][0] = c0.x, f.ql[0][1] = c0.y, f.ql[1][0] = c0.z, f.ql[1][1] = c0.w;
        f.ql[2][0] = c1.x, f.ql[2][1] = c1.y, f.ql[3][0] = c1.z, f.ql[3][1] = c1.w;
        f.qh[0][0] = c2.x, f.qh[0][1] = c2.y, f.qh[1][0] = c2.z, f.qh[1][1] = c2.w;
        f.sc = ld16(ts + 1536 + rs * 16);
        f.d = *reinterpret_cast<const uint16_t*>(ts + 1664 + rs * 2);
    }
}

template <int TYPE, int NC, int R, int D, int S>
struct BulkGeo {
    static constexpr int TB = TileB<TYPE>::value;
    static constexpr int STAGE = R * TB;                          // bytes of one stage of one warp
    static constexpr int PER_SB = SplitTerms<NC, R>::PER_SB;
    static constexpr size_t BAR = 128;                            // S * D mbarriers (<= 16)
    static constexpr size_t W = BAR;                              // weights [S][D][STAGE]
    static constexpr size_t T = W + (size_t)S * D * STAGE;        // terms [2][S][PER_SB] floats
    static constexpr size_t F = T + (size_t)2 * S * PER_SB * 4;   // fin [R*NC*8*12] floats
    static constexpr size_t BYTES = F + (size_t)R * NC * 8 * 12 * 4;
};

template <int TYPE, int NC, int R, int D, int S>
__global__ void __launch_bounds__(32 * S)
kq_gemv_bulk_kernel(const uint8_t* __restrict__ w, int rows, int nb, const uint8_t* __restrict__ img, float* __restrict__ y) {
    using G = BulkGeo<TYPE, NC, R, D, S>;
    constexpr int GL = 2, TB = G::TB, PER_SB = G::PER_SB;
    constexpr bool Q6 = TYPE == T_Q6_K, XP = false;
    constexpr int CHAINS = R * NC * 8 * (Q6 ? 8 : 12);
    constexpr int CPT = (CHAINS + 32 * S - 1) / (32 * S);
    static_assert(S * D <= 16, "mbarrier region");
    extern __shared__ __align__(128) uint8_t smem[];
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem);
    float* terms = reinterpret_cast<float*>(smem + G::T);
    float* fin = reinterpret_cast<float*>(smem + G::F);
    const int lane = threadIdx.x & 31, ws = threadIdx.x >> 5, rs = lane >> 2, tg = lane & 3, g0 = tg * GL;
    const int tiles = rows / 8;
    uint64_t* wbar = bars + ws * D;
    uint8_t* wst = smem + G::W + (size_t)ws * D * G::STAGE;
    const uint8_t* wt[R];
#pragma unroll
    for (int j = 0; j < R; j++) wt[j] = w + (size_t)min(blockIdx.x * R + j, tiles - 1) * nb * TB;
    if (lane < D) mbar_init(&wbar[lane], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    __syncwarp();
    auto issue = [&](int d, int sb) {  // lane 0: stage d <- super-block sb of the warp's R tiles
        if (lane == 0) {
            mbar_expect_tx(&wbar[d], (uint32_t)G::STAGE);
#pragma unroll
            for (int j = 0; j < R; j++) bulk_g2s(wst + (size_t)d * G::STAGE + j * TB, wt[j] + (size_t)sb * TB, TB, &wbar[d]);
        }
    };
#pragma unroll
    for (int d = 0; d < D; d++)
        if (ws + d * S < nb) issue(d, ws + d * S);

    griddep_wait();
    griddep_launch();

    float cacc[CPT];
#pragma unroll
    for (int c = 0; c < CPT; c++) cacc[c] = 0.0f;
    bool alive = true;
    const int nwin = (nb + S - 1) / S;
    for (int w0 = 0; w0 < nwin; w0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int win = w0 + d;
            if (win < nwin) {
                const int sb = win * S + ws;
                float* tb = terms + (size_t)((win & 1) * S + ws) * PER_SB;
                if (sb < nb && alive) {
                    const uint32_t parity = (uint32_t)((win / D) & 1);
                    if (!mbar_wait_bounded(&wbar[d], parity, 0x300u | (unsigned)TYPE)) alive = false;
                }
                if (sb < nb && alive) {
                    Dec<TYPE, GL> dec[R];
#pragma unroll
                    for (int j = 0; j < R; j++) {
                        Frag<TYPE, GL> f;
                        load_frag_smem<TYPE>(wst + (size_t)d * G::STAGE + j * TB, lane, rs, f);
                        decode<TYPE, GL, 0>(f, tg, dec[j]);
                    }
                    __syncwarp();
                    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                    if (sb + D * S < nb) issue(d, sb + D * S);
                    // activation words of column n + 1 are requested while column n computes (XP)
                    uint4 xv[2][2 * GL];
                    float xd[2];
                    uint32_t xa[2][GL];
                    auto load_x = [&](int n, int b) {
                        const uint8_t* xb = img + ((size_t)n * nb + sb) * Q8K_IMG_BYTES;
#pragma unroll
                        for (int c = 0; c < 2 * GL; c++) xv[b][c] = __ldg(reinterpret_cast<const uint4*>(xb + 32 * g0) + c);
                        xd[b] = __ldg(reinterpret_cast<const float*>(xb + Q8K_IMG_D));
                        if constexpr (Q6) {
                            const uint2 a2 = __ldg(reinterpret_cast<const uint2*>(xb + Q8K_IMG_BSP) + tg);
                            xa[b][0] = a2.x, xa[b][1] = a2.y;
                        } else {
                            xa[b][0] = __ldg(reinterpret_cast<const uint32_t*>(xb + Q8K_IMG_Q8S) + tg);
                        }
                    };
                    if constexpr (XP) load_x(0, 0);
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        const int b = XP ? (n & 1) : 0;
                        if constexpr (XP) {
                            if (n + 1 < NC) load_x(n + 1, b ^ 1);
                        } else {
                            load_x(n, 0);
                        }
                        uint32_t xw[8 * GL];
#pragma unroll
                        for (int c = 0; c < 2 * GL; c++) {
                            const uint4 v = xv[b][c];
                            xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
                        }
                        const float dx = xd[b];
                        uint32_t aux[GL];
#pragma unroll
                        for (int gi = 0; gi < GL; gi++) aux[gi] = xa[b][gi];
#pragma unroll
                        for (int j = 0; j < R; j++) {
                            const float dd = __fmul_rn(dx, dec[j].dw);
                            float* t = tb + ((j * NC + n) * 8 + rs) * 12;
                            float2 mt;
                            mt.x = __fmul_rn(dd, lane_sum<TYPE, GL, 0>(dec[j], xw, 0, Q6 ? aux[0] : 0u));
                            mt.y = __fmul_rn(dd, lane_sum<TYPE, GL, 0>(dec[j], xw, 1, Q6 ? aux[1] : 0u));
                            *reinterpret_cast<float2*>(t + 2 * tg) = mt;
                            if constexpr (!Q6) {
                                const float prod = biased_to_f32(dp2a_lo(aux[0], dec[j].mpair, MAGIC_I));
                                t[8 + tg] = __fmul_rn(__fmul_rn(-dx, dec[j].dminw), prod);
                            }
                        }
                    }
                }
                __syncthreads();
                const float* tw = terms + (size_t)((win & 1) * S) * PER_SB;
                const int nsb = min(S, nb - win * S);
#pragma unroll
                for (int c = 0; c < CPT; c++) {
                    const int ci = threadIdx.x + c * 32 * S;
                    if (ci < CHAINS) {
                        constexpr int LPC = Q6 ? 8 : 12;
                        const int slot = (ci / LPC) * 12 + ci % LPC;
                        float a = cacc[c];
                        for (int k = 0; k < nsb; k++) a = __fadd_rn(a, tw[k * PER_SB + slot]);
                        cacc[c] = a;
                    }
                }
            }
        }
    }
    if (!alive) {
        // a wait gave up: drain this warp's copies still in flight (bounded) so none lands after the CTA exits
        for (int d = 0; d < D; d++) {
            int last = -1;  // the last window that used stage d
            for (int win = d; win < nwin; win += D)
                if (win * S + ws < nb) last = win;
            if (last >= 0) mbar_wait_bounded(&wbar[d], (uint32_t)((last / D) & 1), 0x300u | (unsigned)TYPE);
        }
    }
    const int bad = __syncthreads_or(!alive);
#pragma unroll
    for (int c = 0; c < CPT; c++) {
        const int ci = threadIdx.x + c * 32 * S;
        constexpr int LPC = Q6 ? 8 : 12;
        if (ci < CHAINS) fin[(ci / LPC) * 12 + ci % LPC] = cacc[c];
    }
    __syncthreads();
    if (bad) return;
    for (int o = threadIdx.x; o < R * NC * 8; o += 32 * S) {
        const int r = o % 8, n = (o / 8) % NC, j = o / (8 * NC);
        const float* f = fin + o * 12;
        float v = reduce8(f);
        if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(f[8], f[10]), __fadd_rn(f[9], f[11])));
        const int tile = blockIdx.x * R + j;
        if (tile < tiles) y[(size_t)n * rows + tile * 8 + r] = v;
    }
}

template <int TYPE, int NC, int R, int D, int S>
cudaError_t launch_bulk(const uint8_t* w, int rows, int nb, const void* img, float* y, cudaStream_t s, bool pdl) {
    using G = BulkGeo<TYPE, NC, R, D, S>;
    auto kern = kq_gemv_bulk_kernel<TYPE, NC, R, D, S>;
    static bool attr_done = false;
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)G::BYTES);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows / 8 + R - 1) / R);
    cfg.blockDim = dim3(32 * S);
    cfg.dynamicSmemBytes = G::BYTES;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, kern, w, rows, nb, (const uint8_t*)img, y);
}

int g_tile_cfg = [] {
    const char* e = getenv("QDEC_GEMV_TILE_CFG");
    return e ? atoi(e) : 0;
}();

// The default configuration for `rows` rows (all of them split kernels with one super-block in flight per warp
// and the next column's activation words requested while a column computes), measured on B200 over the shapes of
// one GPU and of the tensor-parallel slices (640 .. 248320 rows, 5120 .. 17408 columns): the fewer the rows, the
// fewer CTAs, so short matrices take one tile per warp and split the super-blocks over 8 warps, long ones two
// tiles per warp over 4 warps at <= 128 registers (4 CTAs per SM).
// For Q4_K / Q5_K at several columns the R tiles of a warp are decoded one after another against every column's
// activation words held in registers (one load of a word serves R rows), which relieves the L1 pipe; Q6_K
// (twice the decode registers) keeps the column-by-column order.
template <int TYPE>
inline int default_split_cfg(int nc, int rows) {
    if (nc == 1) return rows <= 6144 ? 30 : 28;
    if (rows <= 2048) return 31;  // R1, S8, 2 CTAs per SM
    if (rows <= 3072) return 30;  // R1, S4
    if (TYPE != T_Q6_K) return rows <= 12288 ? 32 : 34;  // resident activations: R2 S4 3 CTAs / R4 S2 2 CTAs per SM
    if (rows <= 6144) return 29;  // R2, S4, 168 registers
    return 28;                    // R2, S4, 128 registers
}

// Configurations (R tiles per warp, D super-blocks in flight, FP32 scale multiply for Q4_K/Q5_K).
template <int TYPE, int NC>
cudaError_t launch_tile_cfg(const uint8_t* w, int rows, int nb, const void* img, float* y, cudaStream_t s, bool pdl) {
    constexpr bool KQ = TYPE != T_Q6_K;
    int cfg = g_tile_cfg;
    if (cfg == 0) cfg = default_split_cfg<TYPE>(NC, rows);
    switch (cfg) {
    case 1: return launch_tile<TYPE, NC, 1, 4, false>(w, rows, nb, img, y, s, pdl);
    case 2: return launch_tile<TYPE, NC, 1, 8, false>(w, rows, nb, img, y, s, pdl);
    case 3: return launch_tile<TYPE, NC, 2, 4, false>(w, rows, nb, img, y, s, pdl);
    case 4: return launch_tile<TYPE, NC, 2, 2, false>(w, rows, nb, img, y, s, pdl);
    case 5: return launch_tile<TYPE, NC, 1, 4, KQ>(w, rows, nb, img, y, s, pdl);
    case 6: return launch_tile<TYPE, NC, 1, 8, KQ>(w, rows, nb, img, y, s, pdl);
    case 7: return launch_tile<TYPE, NC, 2, 4, KQ>(w, rows, nb, img, y, s, pdl);
    case 8: return launch_tile<TYPE, NC, 2, 2, KQ>(w, rows, nb, img, y, s, pdl);
    case 9: return launch_split<TYPE, NC, 1, 2, 4, false>(w, rows, nb, img, y, s, pdl);
    case 10: return launch_split<TYPE, NC, 2, 2, 4, false>(w, rows, nb, img, y, s, pdl);
    case 11: return launch_split<TYPE, NC, 1, 2, 4, KQ>(w, rows, nb, img, y, s, pdl);
    case 12: return launch_split<TYPE, NC, 2, 2, 4, KQ>(w, rows, nb, img, y, s, pdl);
    case 13: return launch_split<TYPE, NC, 2, 2, 2, KQ>(w, rows, nb, img, y, s, pdl);
    case 14: return launch_split<TYPE, NC, 1, 4, 2, KQ>(w, rows, nb, img, y, s, pdl);
    case 15: return launch_split<TYPE, NC, 2, 2, 4, KQ ? 2 : 0>(w, rows, nb, img, y, s, pdl);
    case 16: return launch_split<TYPE, NC, 1, 2, 4, KQ ? 2 : 0>(w, rows, nb, img, y, s, pdl);
    case 17: return launch_tile<TYPE, NC, 2, 2, KQ ? 2 : 0>(w, rows, nb, img, y, s, pdl);
    case 18: return launch_split<TYPE, NC, 2, 2, 4, 0, 4>(w, rows, nb, img, y, s, pdl);
    case 19: return launch_split<TYPE, NC, 2, 2, 4, 0, 5>(w, rows, nb, img, y, s, pdl);
    case 20: return launch_split<TYPE, NC, 2, 1, 4, 0, 4>(w, rows, nb, img, y, s, pdl);
    case 21: return launch_split<TYPE, NC, 2, 2, 2, 0, 8>(w, rows, nb, img, y, s, pdl);
    case 22: return launch_bulk<TYPE, NC, 2, 3, 4>(w, rows, nb, img, y, s, pdl);
    case 23: return launch_bulk<TYPE, NC, 2, 4, 4>(w, rows, nb, img, y, s, pdl);
    case 24: return launch_bulk<TYPE, NC, 1, 4, 4>(w, rows, nb, img, y, s, pdl);
    case 25: return launch_bulk<TYPE, NC, 2, 2, 4>(w, rows, nb, img, y, s, pdl);
    case 26: return launch_split<TYPE, NC, 1, 1, 8, 0, 2>(w, rows, nb, img, y, s, pdl);
    case 27: return launch_split<TYPE, NC, 1, 2, 8, 0, 2>(w, rows, nb, img, y, s, pdl);
    case 28: return launch_split<TYPE, NC, 2, 1, 4, 0, 4, true>(w, rows, nb, img, y, s, pdl);
    case 29: return launch_split<TYPE, NC, 2, 1, 4, 0, 3, true>(w, rows, nb, img, y, s, pdl);
    case 30: return launch_split<TYPE, NC, 1, 1, 4, 0, 4, true>(w, rows, nb, img, y, s, pdl);
    case 31: return launch_split<TYPE, NC, 1, 1, 8, 0, 2, true>(w, rows, nb, img, y, s, pdl);
    case 32: return launch_split<TYPE, NC, 2, 1, 4, 0, 3, false, true>(w, rows, nb, img, y, s, pdl);
    case 33: return launch_split<TYPE, NC, 2, 1, 4, 0, 4, false, true>(w, rows, nb, img, y, s, pdl);
    case 34: return launch_split<TYPE, NC, 4, 1, 2, 0, 2, false, true>(w, rows, nb, img, y, s, pdl);
    default: return launch_split<TYPE, NC, 1, 1, 8, 0, 2, false, true>(w, rows, nb, img, y, s, pdl);
    }
}

template <int TYPE>
cudaError_t launch_tile_type(const uint8_t* w, int rows, int nb, const void* img, int ncols, float* y, cudaStream_t s, bool pdl) {
    switch (ncols) {
    case 1: return launch_tile_cfg<TYPE, 1>(w, rows, nb, img, y, s, pdl);
    case 2: return launch_tile_cfg<TYPE, 2>(w, rows, nb, img, y, s, pdl);
    case 3: return launch_tile_cfg<TYPE, 3>(w, rows, nb, img, y, s, pdl);
    default: return launch_tile_cfg<TYPE, 4>(w, rows, nb, img, y, s, pdl);
    }
}

// ggml blocks -> tile layout: one CTA per (super-block, tile), byte by byte through the source offset formula.
template <int TYPE>
__device__ __forceinline__ void tile_src(int o, int& r, int& off) {
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        constexpr int QO = TYPE == T_Q4_K ? 16 : 48;
        if (o < 1024) {
            const int j = o / 512, L = (o % 512) / 16, b = o % 16, tg = L % 4, p = 2 * j + b / 8;
            r = L / 4, off = QO + 32 * p + 8 * tg + b % 8;
        } else if (TYPE == T_Q5_K && o < 1280) {
            const int L = (o - 1024) / 8, b = (o - 1024) % 8;
            r = L / 4, off = 16 + 8 * (L % 4) + b;
        } else {
            const int h0 = TYPE == T_Q5_K ? 1280 : 1024;
            r = (o - h0) / 16, off = (o - h0) % 16;
        }
    } else {
        if (o < 1536) {
            const int j = o / 512, L = (o % 512) / 16, b = o % 16, tg = L % 4, q = 2 * j + b / 8;
            r = L / 4, off = (q < 4 ? 32 * q : 128 + 32 * (q - 4)) + 8 * tg + b % 8;
        } else if (o < 1664) {
            r = (o - 1536) / 16, off = 192 + (o - 1536) % 16;
        } else {
            r = (o - 1664) / 2, off = 208 + (o - 1664) % 2;
        }
    }
}

template <int TYPE>
__global__ void repack_tiles_kernel(const uint8_t* __restrict__ src, int nb, uint8_t* __restrict__ dst) {
    constexpr int TB = TileB<TYPE>::value, BB = TB / 8;
    const int sb = blockIdx.x, t = blockIdx.y;
    uint8_t* o = dst + ((size_t)t * nb + sb) * TB;
    for (int i = threadIdx.x; i < TB; i += blockDim.x) {
        int r, off;
        tile_src<TYPE>(i, r, off);
        o[i] = src[((size_t)(t * 8 + r) * nb + sb) * BB + off];
    }
}

template <int TYPE, int NC, int GL, int R, int D, int FPS>
cudaError_t launch_v6(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* img, float* y, cudaStream_t s, bool pdl) {
    constexpr int RPC = 4 * GL * R;  // rows per CTA (one warp)
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows + RPC - 1) / RPC);
    cfg.blockDim = dim3(32);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;  // without the attribute griddepcontrol.wait returns at once
    return cudaLaunchKernelEx(&cfg, kq_gemv_v6_kernel<TYPE, NC, GL, R, D, FPS>, w, dsplit, rows, nb, (const uint8_t*)img, y);
}

// Tuning (tests, sweeps): 0 = automatic; otherwise the configuration index of kConfigs.
int g_v6_cfg = [] {
    const char* e = getenv("QDEC_GEMV_V6_CFG");
    return e ? atoi(e) : 0;
}();

// Configurations: (GL, R, D, FPS).  FPS applies to Q4_K/Q5_K only.
template <int TYPE, int NC>
cudaError_t launch_v6_cfg(int cfg, const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* img, float* y,
                          cudaStream_t s, bool pdl) {
    constexpr bool KQ = TYPE != T_Q6_K;
    switch (cfg) {
    case 1: return launch_v6<TYPE, NC, 1, 1, 8, false>(w, dsplit, rows, nb, img, y, s, pdl);
    case 2: return launch_v6<TYPE, NC, 2, 1, 4, false>(w, dsplit, rows, nb, img, y, s, pdl);
    case 3: return launch_v6<TYPE, NC, 1, 2, 4, false>(w, dsplit, rows, nb, img, y, s, pdl);
    case 4: return launch_v6<TYPE, NC, 2, 2, 2, false>(w, dsplit, rows, nb, img, y, s, pdl);
    case 5: return launch_v6<TYPE, NC, 1, 1, 8, KQ>(w, dsplit, rows, nb, img, y, s, pdl);
    case 6: return launch_v6<TYPE, NC, 2, 1, 4, KQ>(w, dsplit, rows, nb, img, y, s, pdl);
    case 7: return launch_v6<TYPE, NC, 1, 2, 4, KQ>(w, dsplit, rows, nb, img, y, s, pdl);
    default: return launch_v6<TYPE, NC, 2, 2, 2, KQ>(w, dsplit, rows, nb, img, y, s, pdl);
    }
}

template <int TYPE, int NC>
cudaError_t launch_v6_auto(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* img, float* y, cudaStream_t s,
                           bool pdl) {
    int cfg = g_v6_cfg;
    if (cfg == 0) cfg = NC == 1 ? 2 : 3;
    return launch_v6_cfg<TYPE, NC>(cfg, w, dsplit, rows, nb, img, y, s, pdl);
}

template <int TYPE>
cudaError_t launch_v6_type(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* img, int ncols, float* y,
                           cudaStream_t s, bool pdl) {
    switch (ncols) {
    case 1: return launch_v6_auto<TYPE, 1>(w, dsplit, rows, nb, img, y, s, pdl);
    case 2: return launch_v6_auto<TYPE, 2>(w, dsplit, rows, nb, img, y, s, pdl);
    case 3: return launch_v6_auto<TYPE, 3>(w, dsplit, rows, nb, img, y, s, pdl);
    default: return launch_v6_auto<TYPE, 4>(w, dsplit, rows, nb, img, y, s, pdl);
    }
}

}  // namespace

bool v6_gemv_supported(int type) {
    return type == T_Q4_K || type == T_Q5_K || type == T_Q6_K_SPLIT || type == T_Q4_K_TILE || type == T_Q5_K_TILE ||
           type == T_Q6_K_TILE;
}

cudaError_t launch_gemv_img(int type, const uint8_t* w, int rows, int cols, const void* img, int ncols, float* y, cudaStream_t s,
                            bool pdl) {
    const int nb = cols / QK_K;
    if (rows <= 0 || ncols <= 0) return cudaSuccess;
    if (gemm_tc_applies(type, ncols)) return launch_gemm_tc(type, w, rows, y, nullptr, 0, nullptr, cols, img, ncols, s, pdl);
    if (gemv7_supported(type) && gemv_impl() != 6) return launch_gemv7(type, w, rows, y, nullptr, 0, nullptr, cols, img, ncols, s, pdl);
    for (int c0 = 0; c0 < ncols; c0 += 4) {  // columns beyond 4 in groups of at most 4
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * nb * Q8K_IMG_BYTES;
        float* yy = y + (size_t)c0 * rows;
        cudaError_t e;
        if (type == T_Q4_K_TILE) e = launch_tile_type<T_Q4_K>(w, rows, nb, im, nc, yy, s, pdl);
        else if (type == T_Q5_K_TILE) e = launch_tile_type<T_Q5_K>(w, rows, nb, im, nc, yy, s, pdl);
        else if (type == T_Q6_K_TILE) e = launch_tile_type<T_Q6_K>(w, rows, nb, im, nc, yy, s, pdl);
        else if (type == T_Q4_K) e = launch_v6_type<T_Q4_K>(w, nullptr, rows, nb, im, nc, yy, s, pdl);
        else if (type == T_Q5_K) e = launch_v6_type<T_Q5_K>(w, nullptr, rows, nb, im, nc, yy, s, pdl);
        else if (type == T_Q6_K_SPLIT) {
            const uint16_t* dsplit = reinterpret_cast<const uint16_t*>(w + (size_t)rows * nb * 208);
            e = launch_v6_type<T_Q6_K>(w, dsplit, rows, nb, im, nc, yy, s, pdl);
        } else {
            return cudaErrorInvalidValue;
        }
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

namespace {
template <int TYPE, int NC>
cudaError_t launch_pair_nc(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                           const void* img, cudaStream_t s, bool pdl) {
    // the configuration of one matrix with the rows of both (the launch has the CTAs of both)
    switch (default_split_cfg<TYPE>(NC, rows_a + rows_b)) {
    case 31: return launch_split<TYPE, NC, 1, 1, 8, 0, 2, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    case 30: return launch_split<TYPE, NC, 1, 1, 4, 0, 4, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    case 29: return launch_split<TYPE, NC, 2, 1, 4, 0, 3, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    case 32: return launch_split<TYPE, NC, 2, 1, 4, 0, 3, false, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    case 34: return launch_split<TYPE, NC, 4, 1, 2, 0, 2, false, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    default: return launch_split<TYPE, NC, 2, 1, 4, 0, 4, true>(w_a, rows_a, nb, img, y_a, s, pdl, w_b, rows_b, y_b);
    }
}

template <int TYPE>
cudaError_t launch_pair_type(const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b, int nb,
                             const void* img, int nc, cudaStream_t s, bool pdl) {
    switch (nc) {
    case 1: return launch_pair_nc<TYPE, 1>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 2: return launch_pair_nc<TYPE, 2>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    case 3: return launch_pair_nc<TYPE, 3>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    default: return launch_pair_nc<TYPE, 4>(w_a, rows_a, y_a, w_b, rows_b, y_b, nb, img, s, pdl);
    }
}
}  // namespace

cudaError_t launch_gemv_img_pair(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                                 int cols, const void* img, int ncols, cudaStream_t s, bool pdl) {
    if (rows_a % 8 || rows_b % 8) return cudaErrorInvalidValue;
    if (gemm_tc_applies(type, ncols)) return launch_gemm_tc(type, w_a, rows_a, y_a, w_b, rows_b, y_b, cols, img, ncols, s, pdl);
    if (gemv7_supported(type) && gemv_impl() != 6) return launch_gemv7(type, w_a, rows_a, y_a, w_b, rows_b, y_b, cols, img, ncols, s, pdl);
    const int nb = cols / QK_K;
    for (int c0 = 0; c0 < ncols; c0 += 4) {
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * nb * Q8K_IMG_BYTES;
        float* ya = y_a + (size_t)c0 * rows_a;
        float* yb = y_b + (size_t)c0 * rows_b;
        cudaError_t e;
        if (type == T_Q4_K_TILE) e = launch_pair_type<T_Q4_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else if (type == T_Q5_K_TILE) e = launch_pair_type<T_Q5_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else if (type == T_Q6_K_TILE) e = launch_pair_type<T_Q6_K>(w_a, rows_a, ya, w_b, rows_b, yb, nb, im, nc, s, pdl);
        else return cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

void set_gemv_v6_config(int cfg) {
    g_v6_cfg = cfg;
    g_tile_cfg = cfg;
}

cudaError_t launch_repack_tiles(int ggml_type, const uint8_t* src, int rows, int cols, uint8_t* dst, cudaStream_t s) {
    if (rows % 8 || cols % QK_K) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    const dim3 grid(cols / QK_K, rows / 8);
    if (ggml_type == T_Q4_K) repack_tiles_kernel<T_Q4_K><<<grid, 256, 0, s>>>(src, cols / QK_K, dst);
    else if (ggml_type == T_Q5_K) repack_tiles_kernel<T_Q5_K><<<grid, 256, 0, s>>>(src, cols / QK_K, dst);
    else if (ggml_type == T_Q6_K) repack_tiles_kernel<T_Q6_K><<<grid, 256, 0, s>>>(src, cols / QK_K, dst);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

namespace {
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
}  // namespace

cudaError_t launch_repack_q6k(const uint8_t* src, size_t nblocks, uint8_t* dst, cudaStream_t s) {
    if (nblocks == 0) return cudaSuccess;
    const int grid = (int)std::min<size_t>(nblocks, (size_t)num_sms() * 32);
    repack_q6k_kernel<<<grid, 128, 0, s>>>(src, nblocks, dst);
    return cudaGetLastError();
}

unsigned read_kernel_error(bool clear) {
    unsigned v = 0;
    cudaMemcpyFromSymbol(&v, g_kernel_error, sizeof v);
    if (clear && v) {
        const unsigned z = 0;
        cudaMemcpyToSymbol(g_kernel_error, &z, sizeof z);
    }
    const unsigned t = read_gemm_tc_error(clear);
    const unsigned g7 = read_gemv7_error(clear);
    return v ? v : t ? t : g7;
}

}  // namespace qdec
