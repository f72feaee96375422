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
    if (gemv7_supported(type)) return launch_gemv7(type, w, rows, y, nullptr, 0, nullptr, cols, img, ncols, s, pdl);
    for (int c0 = 0; c0 < ncols; c0 += 4) {  // columns beyond 4 in groups of at most 4
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * nb * Q8K_IMG_BYTES;
        float* yy = y + (size_t)c0 * rows;
        cudaError_t e;
        if (type == T_Q4_K) e = launch_v6_type<T_Q4_K>(w, nullptr, rows, nb, im, nc, yy, s, pdl);
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

cudaError_t launch_gemv_img_pair(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                                 int cols, const void* img, int ncols, cudaStream_t s, bool pdl) {
    if (rows_a % 8 || rows_b % 8) return cudaErrorInvalidValue;
    if (gemm_tc_applies(type, ncols)) return launch_gemm_tc(type, w_a, rows_a, y_a, w_b, rows_b, y_b, cols, img, ncols, s, pdl);
    if (!gemv7_supported(type)) return cudaErrorInvalidValue;
    return launch_gemv7(type, w_a, rows_a, y_a, w_b, rows_b, y_b, cols, img, ncols, s, pdl);
}

void set_gemv_v6_config(int cfg) { g_v6_cfg = cfg; }

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

cudaError_t enqueue_kernel_error_read(unsigned* host2, cudaStream_t s) {
    const cudaError_t e = enqueue_gemm_tc_error_read(host2, s);
    return e != cudaSuccess ? e : enqueue_gemv7_error_read(host2 + 1, s);
}

unsigned read_kernel_error(bool clear) {  // the error words of the kernels with bounded waits (0 = none)
    const unsigned t = read_gemm_tc_error(clear);
    const unsigned g7 = read_gemv7_error(clear);
    return t ? t : g7;
}

}  // namespace qdec
