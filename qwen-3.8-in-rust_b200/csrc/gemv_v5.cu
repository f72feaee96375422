// K-quant GEMV, register-streamed (Q4_K, Q5_K, and Q6_K in the split layout) x Q8_K activations, bit-exact with
// crates/core/src/kernels/kdot.rs:37-141 and its blocked form :176-333.
//
// Work split.  GL of the reference's eight i32 lanes (lane g = positions 4g..4g+3 of every 32-element chunk) live
// in one thread, so 8/GL threads share a weight row and a warp holds 32*GL/8 rows.  Each thread walks its rows'
// super-blocks in order and keeps the f32 lane accumulators in registers -- the reference's "per lane,
// sequential over super-blocks" chain -- with one gather + reduce8 + reduce4 per row at the end.
//
// Data movement.  Weight bytes go straight from HBM into registers with 8/16-byte non-allocating loads: the
// threads of a row read whole 32-byte sectors together, and each thread keeps D super-blocks of loads in flight
// in a register ring (the loop is unrolled by D so every ring slot is a fixed register set).  A warp's work is
// the linear sequence of (row group, super-block) pairs it owns, so the ring runs on across row groups without
// draining.  The activation columns are staged once per CTA into shared memory in the order each thread reads
// them (8*GL code words contiguous per thread, 16-byte chunks XOR-swizzled against bank conflicts).
//
// Programmatic dependent launch: the first D super-blocks of weights are requested before griddepcontrol.wait,
// so the weight stream of this GEMV overlaps the tail of the kernel that produced its activations.
#include <algorithm>
#include <cstdlib>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

namespace {

constexpr int V5_WARPS = 8;

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

// Per-thread fragment of one super-block: the bytes of its GL lanes.
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
    uint4 sc;               // the 16 int8 scales
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

// Shared-memory image of the activation columns, per (column, super-block): 64 code words (thread group tg's
// 8*GL words contiguous, 16-byte chunks XOR-swizzled), an f32 scale, and 8 packed 16-bit pairs (Q4_K/Q5_K: the
// min-lane pairs (q8s[2i], q8s[2i+1]) in entries 0..3; Q6_K: the bsums pairs (2g, 2g+1) in entries 0..7).
struct XGeo {
    static __host__ __device__ size_t off_d(int nc, int nb) { return (size_t)nc * nb * 256; }
    static __host__ __device__ size_t off_a(int nc, int nb) { return off_d(nc, nb) + (size_t)nc * nb * 4; }
    static __host__ __device__ size_t bytes(int nc, int nb) { return off_a(nc, nb) + (size_t)nc * nb * 32; }
};

template <int GL>
__device__ __forceinline__ int code_word_index(int s, int g) {
    const int tg = g / GL, gi = g % GL;
    const int k = s * GL + gi;                    // word within the thread's 8*GL
    const int chunk = (k >> 2) ^ ((tg * GL / 4) & 1);
    return tg * 8 * GL + chunk * 4 + (k & 3);
}

template <int GL, bool Q6>
__device__ void stage_x(const uint8_t* __restrict__ act, int nc, int nb, uint8_t* sm) {
    uint32_t* xq = reinterpret_cast<uint32_t*>(sm);
    float* xd = reinterpret_cast<float*>(sm + XGeo::off_d(nc, nb));
    uint32_t* xa = reinterpret_cast<uint32_t*>(sm + XGeo::off_a(nc, nb));
    uint16_t* xa16 = reinterpret_cast<uint16_t*>(xa);
    for (int i = threadIdx.x; i < nc * nb * 73; i += blockDim.x) {
        const int blk = i / 73, wi = i % 73;
        const uint32_t v = reinterpret_cast<const uint32_t*>(act + (size_t)blk * Q8K_BLOCK_BYTES)[wi];
        if (wi == 0) {
            xd[blk] = __uint_as_float(v);
        } else if (wi <= 64) {
            const int c = wi - 1, s = c >> 3, g = c & 7;
            xq[(size_t)blk * 64 + code_word_index<GL>(s, g)] = v;
        } else {
            const int j = wi - 65;  // bsums 2j (low half), 2j+1 (high half)
            if (Q6) {
                xa[(size_t)blk * 8 + j] = v;
            } else {  // q8s[j] = bsums[2j] + bsums[2j+1] (q8k.rs:185-193), paired for min lane j/2
                const int16_t q = (int16_t)((int16_t)(v & 0xffff) + (int16_t)(v >> 16));
                xa16[(size_t)blk * 16 + j] = (uint16_t)q;
            }
        }
    }
}

__device__ __forceinline__ int dp2a_lo(uint32_t a16x2, uint32_t b8x4) {
    int r;
    asm("dp2a.lo.s32.s32 %0, %1, %2, 0;" : "=r"(r) : "r"(a16x2), "r"(b8x4));
    return r;
}

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// Accumulate one super-block of this thread's GL lanes (and its min lane) into acc/accm, every column.
template <int TYPE, int NC, int GL>
__device__ __forceinline__ void sb_terms(const Frag<TYPE, GL>& f, int tg, const uint32_t* __restrict__ xq, const float* __restrict__ xd,
                                         const uint32_t* __restrict__ xa, int nb, int sb, float (&acc)[NC][GL], float (&accm)[NC]) {
    static_assert(GL == 1 || GL == 2, "one or two reference lanes per thread");
    const int g0 = tg * GL;
    const int swz = (tg * GL / 4) & 1;
    if constexpr (TYPE == T_Q4_K || TYPE == T_Q5_K) {
        const uint32_t sc03 = f.hdr.y & 0x3F3F3F3Fu;
        const uint32_t sc47 = (f.hdr.w & 0x0F0F0F0Fu) | ((f.hdr.y >> 2) & 0x30303030u);
        const float dw = f16_bits_to_f32((uint16_t)(f.hdr.x & 0xffff));
        const float dminw = f16_bits_to_f32((uint16_t)(f.hdr.x >> 16));
        int sc[8];
#pragma unroll
        for (int s = 0; s < 4; s++) sc[s] = (int)((sc03 >> (8 * s)) & 0xff), sc[s + 4] = (int)((sc47 >> (8 * s)) & 0xff);
        uint32_t code[8][GL];
#pragma unroll
        for (int p = 0; p < 4; p++)
#pragma unroll
            for (int gi = 0; gi < GL; gi++) {
                code[2 * p][gi] = f.qs[p][gi] & 0x0F0F0F0Fu;
                code[2 * p + 1][gi] = (f.qs[p][gi] >> 4) & 0x0F0F0F0Fu;
                if constexpr (TYPE == T_Q5_K) {
                    code[2 * p][gi] |= ((f.qh[gi] >> (2 * p)) & 0x01010101u) << 4;
                    code[2 * p + 1][gi] |= ((f.qh[gi] >> (2 * p + 1)) & 0x01010101u) << 4;
                }
            }
        // min lane i (sub-blocks 2i, 2i+1; kdot.rs:60-66) belongs to thread tg = i of the row
        const bool has_min = tg < 4;
        const int mi = tg & 3;
        const uint32_t mw = mi < 2 ? (f.hdr.z & 0x3F3F3F3Fu) : (((f.hdr.w >> 4) & 0x0F0F0F0Fu) | ((f.hdr.z >> 2) & 0x30303030u));
        const uint32_t mpair = mw >> (16 * (mi & 1));  // bytes 0, 1 = the mins of sub-blocks 2i, 2i+1
#pragma unroll
        for (int n = 0; n < NC; n++) {
            const uint32_t* xb = xq + ((size_t)n * nb + sb) * 64 + tg * 8 * GL;
            uint32_t xw[8 * GL];
#pragma unroll
            for (int c = 0; c < 2 * GL; c++) {
                const uint4 v = *reinterpret_cast<const uint4*>(xb + 4 * (c ^ swz));
                xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
            }
            const float dx = xd[n * nb + sb];
            const float d = __fmul_rn(dx, dw);
#pragma unroll
            for (int gi = 0; gi < GL; gi++) {
                int sumi = 0;
#pragma unroll
                for (int s = 0; s < 8; s++) sumi += sc[s] * __dp4a((int)code[s][gi], (int)xw[s * GL + gi], 0);
                acc[n][gi] = __fadd_rn(acc[n][gi], __fmul_rn(d, (float)sumi));
            }
            if (has_min) {
                const float dmin = __fmul_rn(-dx, dminw);
                const int prod = dp2a_lo(xa[((size_t)n * nb + sb) * 8 + mi], mpair);  // mn[2i] q8s[2i] + mn[2i+1] q8s[2i+1]
                accm[n] = __fadd_rn(accm[n], __fmul_rn(dmin, (float)prod));
            }
        }
    } else {
        const float dw = f16_bits_to_f32((uint16_t)(f.d & 0xffff));
        const uint32_t scw[4] = {f.sc.x, f.sc.y, f.sc.z, f.sc.w};
        uint32_t code[8][GL];
        int scl[8][GL];
#pragma unroll
        for (int h = 0; h < 2; h++)
#pragma unroll
            for (int k = 0; k < 4; k++)
#pragma unroll
                for (int gi = 0; gi < GL; gi++) {
                    const uint32_t lo = (f.ql[2 * h + (k & 1)][gi] >> (4 * (k >> 1))) & 0x0F0F0F0Fu;
                    const uint32_t hi = ((f.qh[h][gi] >> (2 * k)) & 0x03030303u) << 4;
                    code[4 * h + k][gi] = lo | hi;
                    const int si = h * 8 + 2 * k + ((g0 + gi) >> 2);  // sc[2k + l/16] of half h
                    scl[4 * h + k][gi] = (int)(int8_t)((scw[si >> 2] >> (8 * (si & 3))) & 0xff);
                }
        uint32_t spair[GL];
#pragma unroll
        for (int gi = 0; gi < GL; gi++) {
            const int g = g0 + gi;
            spair[gi] = scw[g >> 1] >> (16 * (g & 1));  // int8 scales 2g, 2g+1 in bytes 0, 1
        }
#pragma unroll
        for (int n = 0; n < NC; n++) {
            const uint32_t* xb = xq + ((size_t)n * nb + sb) * 64 + tg * 8 * GL;
            uint32_t xw[8 * GL];
#pragma unroll
            for (int c = 0; c < 2 * GL; c++) {
                const uint4 v = *reinterpret_cast<const uint4*>(xb + 4 * (c ^ swz));
                xw[4 * c] = v.x, xw[4 * c + 1] = v.y, xw[4 * c + 2] = v.z, xw[4 * c + 3] = v.w;
            }
            const float d = __fmul_rn(xd[n * nb + sb], dw);
#pragma unroll
            for (int gi = 0; gi < GL; gi++) {
                int sumi = 0;
#pragma unroll
                for (int c = 0; c < 8; c++) sumi += scl[c][gi] * __dp4a((int)code[c][gi], (int)xw[c * GL + gi], 0);
                sumi -= 32 * dp2a_lo(xa[((size_t)n * nb + sb) * 8 + g0 + gi], spair[gi]);
                acc[n][gi] = __fadd_rn(acc[n][gi], __fmul_rn(d, (float)sumi));
            }
        }
    }
}

template <int TYPE, int NC, int GL, int D>
__global__ void __launch_bounds__(V5_WARPS * 32)
kq_gemv_v5_kernel(const uint8_t* __restrict__ w, const uint16_t* __restrict__ dsplit, int rows, int nb,
                  const uint8_t* __restrict__ act, float* __restrict__ y) {
    constexpr int TPR = 8 / GL, RPW = 32 / TPR, BB = BlkB<TYPE>::value;
    constexpr bool Q6 = TYPE == T_Q6_K;
    extern __shared__ __align__(16) uint8_t smem[];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rsub = lane / TPR, tg = lane % TPR;
    const size_t row_bytes = (size_t)nb * BB;
    const int groups = (rows + RPW - 1) / RPW;
    const int wstride = gridDim.x * V5_WARPS;
    const int first = blockIdx.x * V5_WARPS + warp;
    const int my_groups = first < groups ? (groups - first + wstride - 1) / wstride : 0;
    const int total = my_groups * nb;

    // load cursor: (row pointer, super-block) of linear item `ld`
    int ld_sb = 0, ld_grp = first;
    const uint8_t* ld_row = w + (size_t)min(first * RPW + rsub, rows - 1) * row_bytes;
    const uint16_t* ld_d = Q6 ? dsplit + (size_t)min(first * RPW + rsub, rows - 1) * nb : nullptr;
    auto advance_load = [&]() {
        if (++ld_sb == nb) {
            ld_sb = 0;
            ld_grp += wstride;
            const int r = min(ld_grp * RPW + rsub, rows - 1);
            ld_row = w + (size_t)r * row_bytes;
            if constexpr (Q6) ld_d = dsplit + (size_t)r * nb;
        }
    };
    Frag<TYPE, GL> ring[D];
#pragma unroll
    for (int j = 0; j < D; j++) {
        if (j < total) {
            load_frag<TYPE, GL>(ld_row + (size_t)ld_sb * BB, Q6 ? ld_d + ld_sb : nullptr, tg * GL, ring[j]);
            advance_load();
        }
    }

    griddep_wait();  // the activations are the previous kernel's output
    stage_x<GL, Q6>(act, NC, nb, smem);
    __syncthreads();
    griddep_launch();
    const uint32_t* xq = reinterpret_cast<const uint32_t*>(smem);
    const float* xd = reinterpret_cast<const float*>(smem + XGeo::off_d(NC, nb));
    const uint32_t* xa = reinterpret_cast<const uint32_t*>(smem + XGeo::off_a(NC, nb));

    float acc[NC][GL], accm[NC];
#pragma unroll
    for (int n = 0; n < NC; n++) {
#pragma unroll
        for (int gi = 0; gi < GL; gi++) acc[n][gi] = 0.0f;
        accm[n] = 0.0f;
    }
    int c_sb = 0, c_grp = first;
    for (int i0 = 0; i0 < total; i0 += D) {
#pragma unroll
        for (int j = 0; j < D; j++) {
            if (i0 + j < total) {
                sb_terms<TYPE, NC, GL>(ring[j], tg, xq, xd, xa, nb, c_sb, acc, accm);
                if (i0 + j + D < total) {
                    load_frag<TYPE, GL>(ld_row + (size_t)ld_sb * BB, Q6 ? ld_d + ld_sb : nullptr, tg * GL, ring[j]);
                    advance_load();
                }
                if (++c_sb == nb) {
                    // the row group is complete: gather the row's 8 main and 4 min lanes, reduce in the
                    // reference's order ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7)) + ((m0+m2)+(m1+m3))
                    const int row = c_grp * RPW + rsub;
                    const int base = rsub * TPR;
#pragma unroll
                    for (int n = 0; n < NC; n++) {
                        float l8[8], m4[4];
#pragma unroll
                        for (int g = 0; g < 8; g++) l8[g] = __shfl_sync(0xffffffffu, acc[n][g % GL], base + g / GL);
#pragma unroll
                        for (int m = 0; m < 4; m++) m4[m] = __shfl_sync(0xffffffffu, accm[n], base + m);
                        if (tg == 0 && row < rows) {
                            float v = reduce8(l8);
                            if constexpr (!Q6) v = __fadd_rn(v, __fadd_rn(__fadd_rn(m4[0], m4[2]), __fadd_rn(m4[1], m4[3])));
                            y[(size_t)n * rows + row] = v;
                        }
#pragma unroll
                        for (int gi = 0; gi < GL; gi++) acc[n][gi] = 0.0f;
                        accm[n] = 0.0f;
                    }
                    c_sb = 0;
                    c_grp += wstride;
                }
            }
        }
    }
}

constexpr size_t V5_SMEM_LIMIT = 227 * 1024;

template <int TYPE, int NC, int GL, int D>
cudaError_t launch_v5(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, float* y, cudaStream_t s,
                      bool pdl) {
    const size_t smem = XGeo::bytes(NC, nb);
    if (smem > V5_SMEM_LIMIT) return cudaErrorInvalidConfiguration;
    auto kern = kq_gemv_v5_kernel<TYPE, NC, GL, D>;
    static bool attr_done = false;  // per instantiation: raise the dynamic shared-memory cap once
    if (!attr_done) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)V5_SMEM_LIMIT);
        if (e != cudaSuccess) return e;
        attr_done = true;
    }
    int per_sm = 0;
    cudaError_t e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, V5_WARPS * 32, smem);
    if (e != cudaSuccess) return e;
    if (per_sm < 1) return cudaErrorInvalidConfiguration;
    constexpr int RPW = 32 * GL / 8;
    const int groups = (rows + RPW - 1) / RPW;
    const int grid = std::max(1, std::min((groups + V5_WARPS - 1) / V5_WARPS, num_sms() * per_sm));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(V5_WARPS * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;  // without the attribute griddepcontrol.wait returns at once
    return cudaLaunchKernelEx(&cfg, kern, w, dsplit, rows, nb, (const uint8_t*)act, y);
}

int g_v5_gl = [] {
    const char* e = getenv("QDEC_GEMV_GL");  // tuning override: 1 or 2 lanes per thread
    return e ? atoi(e) : 0;
}();
int g_v5_depth = [] {
    const char* e = getenv("QDEC_GEMV_DEPTH");  // tuning override: 4 or 8 super-blocks in flight per thread
    return e ? atoi(e) : 0;
}();

template <int TYPE, int NC, int GL>
cudaError_t launch_v5_d(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, float* y, cudaStream_t s,
                        bool pdl) {
    const int d = g_v5_depth ? g_v5_depth : (GL == 1 ? 8 : 4);
    if (d == 8) return launch_v5<TYPE, NC, GL, 8>(w, dsplit, rows, nb, act, y, s, pdl);
    return launch_v5<TYPE, NC, GL, 4>(w, dsplit, rows, nb, act, y, s, pdl);
}

template <int TYPE, int NC>
cudaError_t launch_v5_gl(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, float* y, cudaStream_t s,
                         bool pdl) {
    // two lanes per thread where the matrix is tall enough to give every SM ~12 warps; one otherwise
    const int gl = g_v5_gl ? g_v5_gl : ((long)rows * 4 >= (long)num_sms() * 12 * 32 ? 2 : 1);
    if (gl == 2) return launch_v5_d<TYPE, NC, 2>(w, dsplit, rows, nb, act, y, s, pdl);
    return launch_v5_d<TYPE, NC, 1>(w, dsplit, rows, nb, act, y, s, pdl);
}

template <int TYPE>
cudaError_t launch_v5_type(const uint8_t* w, const uint16_t* dsplit, int rows, int nb, const void* act, int ncols, float* y,
                           cudaStream_t s, bool pdl) {
    switch (ncols) {
    case 1: return launch_v5_gl<TYPE, 1>(w, dsplit, rows, nb, act, y, s, pdl);
    case 2: return launch_v5_gl<TYPE, 2>(w, dsplit, rows, nb, act, y, s, pdl);
    case 3: return launch_v5_gl<TYPE, 3>(w, dsplit, rows, nb, act, y, s, pdl);
    default: return launch_v5_gl<TYPE, 4>(w, dsplit, rows, nb, act, y, s, pdl);
    }
}

}  // namespace

bool v5_gemv_supported(int type, int cols, int ncols) {
    if (type != T_Q4_K && type != T_Q5_K && type != T_Q6_K_SPLIT) return false;
    if (ncols < 1 || ncols > 4 || cols % QK_K) return false;
    return XGeo::bytes(ncols, cols / QK_K) <= V5_SMEM_LIMIT;
}

cudaError_t launch_gemv_v5(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y, cudaStream_t s,
                           bool pdl) {
    const int nb = cols / QK_K;
    if (rows == 0 || ncols == 0) return cudaSuccess;
    if (type == T_Q4_K) return launch_v5_type<T_Q4_K>(w, nullptr, rows, nb, act, ncols, y, s, pdl);
    if (type == T_Q5_K) return launch_v5_type<T_Q5_K>(w, nullptr, rows, nb, act, ncols, y, s, pdl);
    const uint16_t* dsplit = reinterpret_cast<const uint16_t*>(w + (size_t)rows * nb * 208);
    return launch_v5_type<T_Q6_K>(w, dsplit, rows, nb, act, ncols, y, s, pdl);
}

void set_gemv_v5_tuning(int gl, int depth) {
    g_v5_gl = gl;
    g_v5_depth = depth;
}

}  // namespace qdec
