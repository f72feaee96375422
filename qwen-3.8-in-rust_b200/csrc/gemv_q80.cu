// Q8_0 / Q4_0 GEMV over the engine's Q8_0 activation image, weights in the tile layout, bit-exact with
// crates/core/src/kernels/dot.rs:29-64 (per 32-block i32 sum, then acc += (d_w * d_x) * f32(isum), left to right
// over the row's blocks).
//
// Tile layout: 8 rows x 8 blocks (256 columns) per tile block, arranged in the order the GEMV's 32 threads read
// it (thread L = 4 * row + tg takes blocks 2tg, 2tg+1 of its row), so every warp-wide load is 512 contiguous
// bytes and a warp streams one contiguous range:
//   Q8_0 (2176 B): [4 x 32 x 16 B] codes -- chunk c of thread L = bytes (c % 2) * 16 .. +16 of block 2tg + c / 2
//                  [8 rows x 8 blocks x f16] scales
//   Q4_0 (1152 B): [2 x 32 x 16 B] nibbles -- chunk c of thread L = the 16 bytes of block 2tg + c
//                  [8 rows x 8 blocks x f16] scales
// Tile t, group g (columns 256g .. 256g + 255) at (t * groups + g) * TILE_BYTES.
//
// The block terms of a group are computed by 4 threads of the row (two blocks each, all columns); each thread
// writes them to shared memory and thread tg = n then adds column n's 8 terms in block order -- the reference's
// own chain, so every bit matches.
#include <algorithm>

#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

namespace {

constexpr int MAGIC_I = 0x4B400000;     // bits of 1.5 * 2^23
constexpr float MAGIC_F = 12582912.0f;  // float(bits + k) - MAGIC_F == k for |k| < 2^22
constexpr int Q80_WARPS = 4;

template <int TYPE>
struct Q80Tile {
    static constexpr int TB = TYPE == T_Q8_0 ? 2176 : 1152;   // tile block bytes
    static constexpr int CODE = TYPE == T_Q8_0 ? 2048 : 1024; // code bytes (scales follow)
    static constexpr int CH = TYPE == T_Q8_0 ? 4 : 2;         // 16-byte code chunks per thread
    static constexpr int BB = TYPE == T_Q8_0 ? 34 : 18;       // ggml block bytes
};

__device__ __forceinline__ void griddep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void griddep_launch() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

template <int TYPE>
struct QFrag {
    uint4 c[Q80Tile<TYPE>::CH];
    uint32_t sc;  // f16 scales of blocks 2tg (low half) and 2tg+1 (high half)
};

template <int TYPE>
__device__ __forceinline__ void load_qfrag(const uint8_t* tb, int lane, int rs, int tg, QFrag<TYPE>& f) {
#pragma unroll
    for (int c = 0; c < Q80Tile<TYPE>::CH; c++) f.c[c] = ld_nc_u128(tb + c * 512 + lane * 16);
    f.sc = ld_nc_u32(tb + Q80Tile<TYPE>::CODE + rs * 16 + tg * 4);
}

template <int TYPE, int NC, int D>
__global__ void __launch_bounds__(32 * Q80_WARPS)
q80_tile_kernel(const uint8_t* __restrict__ w, int rows, int groups, const uint8_t* __restrict__ img, float* __restrict__ y) {
    constexpr int TB = Q80Tile<TYPE>::TB;
    __shared__ __align__(16) float terms[Q80_WARPS][8][NC][8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rs = lane >> 2, tg = lane & 3;
    const int tiles = rows / 8;
    const int tile = blockIdx.x * Q80_WARPS + warp;
    const bool active = tile < tiles;
    const uint8_t* wt = w + (size_t)min(tile, tiles - 1) * groups * TB;
    const int nb = groups * 8;  // 32-blocks per row
    QFrag<TYPE> ring[D];
#pragma unroll
    for (int d = 0; d < D; d++)
        if (d < groups) load_qfrag<TYPE>(wt + (size_t)d * TB, lane, rs, tg, ring[d]);

    griddep_wait();  // the activation image is the previous kernel's output
    griddep_launch();

    float acc = 0.0f;  // column tg of row rs (threads tg < NC)
    for (int g0 = 0; g0 < groups; g0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int g = g0 + d;
            if (g < groups) {
                const QFrag<TYPE> f = ring[d];
                if (g + D < groups) load_qfrag<TYPE>(wt + (size_t)(g + D) * TB, lane, rs, tg, ring[d]);
                const float dw0 = f16_bits_to_f32((uint16_t)(f.sc & 0xffff)), dw1 = f16_bits_to_f32((uint16_t)(f.sc >> 16));
                const int blk = g * 8 + 2 * tg;
#pragma unroll
                for (int n = 0; n < NC; n++) {
                    const uint8_t* xr = img + (size_t)n * nb * Q80_IMG_BYTES;
                    const uint4* xc = reinterpret_cast<const uint4*>(xr + (size_t)blk * 32);
                    const uint4 meta = __ldg(reinterpret_cast<const uint4*>(xr + (size_t)nb * 32 + (size_t)blk * 8));
                    float t2[2];
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        const uint4 xa = __ldg(xc + 2 * k), xb = __ldg(xc + 2 * k + 1);
                        const uint32_t xw[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
                        int s;
                        if constexpr (TYPE == T_Q8_0) {
                            const uint4 wa = f.c[2 * k], wb = f.c[2 * k + 1];
                            const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                            s = MAGIC_I;
#pragma unroll
                            for (int i = 0; i < 8; i++) s = __dp4a((int)ww[i], (int)xw[i], s);
                        } else {
                            // element j < 16: low nibble of byte j, j >= 16: high nibble of byte j - 16; value q - 8:
                            // isum = sum q x - 8 * sum x (dot.rs:46-63)
                            const uint4 wa = f.c[k];
                            const uint32_t ww[4] = {wa.x, wa.y, wa.z, wa.w};
                            const int xsum = (int)(k ? meta.w : meta.y);
                            s = MAGIC_I - 8 * xsum;
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                s = __dp4a((int)(ww[i] & 0x0F0F0F0Fu), (int)xw[i], s);
                                s = __dp4a((int)((ww[i] >> 4) & 0x0F0F0F0Fu), (int)xw[4 + i], s);
                            }
                        }
                        const float dx = __uint_as_float(k ? meta.z : meta.x);
                        const float isum = __fsub_rn(__int_as_float(s), MAGIC_F);  // |isum| < 2^22: exact
                        t2[k] = __fmul_rn(__fmul_rn(k ? dw1 : dw0, dx), isum);
                    }
                    *reinterpret_cast<float2*>(&terms[warp][rs][n][2 * tg]) = make_float2(t2[0], t2[1]);
                }
                __syncwarp();
                if (tg < NC) {
                    const float4 a = *reinterpret_cast<const float4*>(&terms[warp][rs][tg][0]);
                    const float4 b = *reinterpret_cast<const float4*>(&terms[warp][rs][tg][4]);
                    acc = __fadd_rn(acc, a.x), acc = __fadd_rn(acc, a.y), acc = __fadd_rn(acc, a.z), acc = __fadd_rn(acc, a.w);
                    acc = __fadd_rn(acc, b.x), acc = __fadd_rn(acc, b.y), acc = __fadd_rn(acc, b.z), acc = __fadd_rn(acc, b.w);
                }
                __syncwarp();
            }
        }
    }
    if (active && tg < NC) y[(size_t)tg * rows + tile * 8 + rs] = acc;
}

// Split group range: one CTA of S warps per R tiles; warp w computes groups w, w+S, ... of every tile and writes
// their block terms to shared memory; after each window of S groups, the chain owners (thread (tile j, row rs,
// column tg < NC) of the first R warps) add the window's terms in block order (the reference's chain).  S times
// the warps stream each tile, which 5120-row matrices need; with R = 2 one load of a column's activation words
// serves both tiles.
template <int TYPE, int NC, int S, int R = 1>
__global__ void __launch_bounds__(32 * S)
q80_split_kernel(const uint8_t* __restrict__ w, int rows, int groups, const uint8_t* __restrict__ img, float* __restrict__ y) {
    constexpr int TB = Q80Tile<TYPE>::TB;
    static_assert(R <= S, "chain owners: one warp per tile");
    __shared__ __align__(16) float terms[2][S][R][8][NC][8];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, rs = lane >> 2, tg = lane & 3;
    const int tiles = rows / 8;
    const uint8_t* wt[R];
#pragma unroll
    for (int j = 0; j < R; j++) wt[j] = w + (size_t)min((int)blockIdx.x * R + j, tiles - 1) * groups * TB;
    const int nb = groups * 8;
    QFrag<TYPE> nxt[R];
    if (warp < groups) {
#pragma unroll
        for (int j = 0; j < R; j++) load_qfrag<TYPE>(wt[j] + (size_t)warp * TB, lane, rs, tg, nxt[j]);
    }

    griddep_wait();  // the activation image is the previous kernel's output
    griddep_launch();

    float acc = 0.0f;  // warp j < R: column tg of row rs of tile j (tg < NC)
    const int nwin = (groups + S - 1) / S;
    for (int win = 0; win < nwin; win++) {
        const int g = win * S + warp;
        if (g < groups) {
            QFrag<TYPE> f[R];
            float dw0[R], dw1[R];
#pragma unroll
            for (int j = 0; j < R; j++) {
                f[j] = nxt[j];
                if (g + S < groups) load_qfrag<TYPE>(wt[j] + (size_t)(g + S) * TB, lane, rs, tg, nxt[j]);
                dw0[j] = f16_bits_to_f32((uint16_t)(f[j].sc & 0xffff));
                dw1[j] = f16_bits_to_f32((uint16_t)(f[j].sc >> 16));
            }
            const int blk = g * 8 + 2 * tg;
#pragma unroll
            for (int n = 0; n < NC; n++) {
                const uint8_t* xr = img + (size_t)n * nb * Q80_IMG_BYTES;
                const uint4* xc = reinterpret_cast<const uint4*>(xr + (size_t)blk * 32);
                const uint4 meta = __ldg(reinterpret_cast<const uint4*>(xr + (size_t)nb * 32 + (size_t)blk * 8));
                uint32_t xw[2][8];
#pragma unroll
                for (int k = 0; k < 2; k++) {
                    const uint4 xa = __ldg(xc + 2 * k), xb = __ldg(xc + 2 * k + 1);
                    xw[k][0] = xa.x, xw[k][1] = xa.y, xw[k][2] = xa.z, xw[k][3] = xa.w;
                    xw[k][4] = xb.x, xw[k][5] = xb.y, xw[k][6] = xb.z, xw[k][7] = xb.w;
                }
#pragma unroll
                for (int j = 0; j < R; j++) {
                    float t2[2];
#pragma unroll
                    for (int k = 0; k < 2; k++) {
                        int sacc;
                        if constexpr (TYPE == T_Q8_0) {
                            const uint4 wa = f[j].c[2 * k], wb = f[j].c[2 * k + 1];
                            const uint32_t ww[8] = {wa.x, wa.y, wa.z, wa.w, wb.x, wb.y, wb.z, wb.w};
                            sacc = MAGIC_I;
#pragma unroll
                            for (int i = 0; i < 8; i++) sacc = __dp4a((int)ww[i], (int)xw[k][i], sacc);
                        } else {  // q - 8 per nibble: sum q x - 8 sum x (dot.rs:46-63)
                            const uint4 wa = f[j].c[k];
                            const uint32_t ww[4] = {wa.x, wa.y, wa.z, wa.w};
                            sacc = MAGIC_I - 8 * (int)(k ? meta.w : meta.y);
#pragma unroll
                            for (int i = 0; i < 4; i++) {
                                sacc = __dp4a((int)(ww[i] & 0x0F0F0F0Fu), (int)xw[k][i], sacc);
                                sacc = __dp4a((int)((ww[i] >> 4) & 0x0F0F0F0Fu), (int)xw[k][4 + i], sacc);
                            }
                        }
                        const float dx = __uint_as_float(k ? meta.z : meta.x);
                        t2[k] = __fmul_rn(__fmul_rn(k ? dw1[j] : dw0[j], dx), __fsub_rn(__int_as_float(sacc), MAGIC_F));
                    }
                    *reinterpret_cast<float2*>(&terms[win & 1][warp][j][rs][n][2 * tg]) = make_float2(t2[0], t2[1]);
                }
            }
        }
        __syncthreads();
        if (warp < R && tg < NC) {
            const int ng = min(S, groups - win * S);
#pragma unroll
            for (int k = 0; k < S; k++)
                if (k < ng) {
                    const float4 a = *reinterpret_cast<const float4*>(&terms[win & 1][k][warp][rs][tg][0]);
                    const float4 b = *reinterpret_cast<const float4*>(&terms[win & 1][k][warp][rs][tg][4]);
                    acc = __fadd_rn(acc, a.x), acc = __fadd_rn(acc, a.y), acc = __fadd_rn(acc, a.z), acc = __fadd_rn(acc, a.w);
                    acc = __fadd_rn(acc, b.x), acc = __fadd_rn(acc, b.y), acc = __fadd_rn(acc, b.z), acc = __fadd_rn(acc, b.w);
                }
        }
    }
    const int tile = (int)blockIdx.x * R + warp;
    if (warp < R && tg < NC && tile < tiles) y[(size_t)tg * rows + tile * 8 + rs] = acc;
}

template <int TYPE, int NC, int R = 1>
cudaError_t launch_q80_split_nc(const uint8_t* w, int rows, int groups, const void* img, float* y, cudaStream_t s, bool pdl) {
    constexpr int S = 4;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows / 8 + R - 1) / R);
    cfg.blockDim = dim3(32 * S);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q80_split_kernel<TYPE, NC, S, R>, w, rows, groups, (const uint8_t*)img, y);
}

template <int TYPE, int NC>
cudaError_t launch_q80_tile_nc(const uint8_t* w, int rows, int groups, const void* img, float* y, cudaStream_t s, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((rows / 8 + Q80_WARPS - 1) / Q80_WARPS);
    cfg.blockDim = dim3(32 * Q80_WARPS);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl && pdl_enabled() ? 1 : 0;
    return cudaLaunchKernelEx(&cfg, q80_tile_kernel<TYPE, NC, 4>, w, rows, groups, (const uint8_t*)img, y);
}

int g_q80_split = [] {
    const char* e = getenv("QDEC_Q80_SPLIT");  // tuning override: 0 = one warp per tile, 1 = split groups
    return e ? atoi(e) : -1;
}();

template <int TYPE>
cudaError_t launch_q80_tile_type(const uint8_t* w, int rows, int groups, const void* img, int ncols, float* y, cudaStream_t s,
                                 bool pdl) {
    // split the group range over 4 warps unless the matrix alone gives every SM ~16 warps; two tiles per CTA
    // (one load of the activation words for both) on matrices with >= 4096 rows, for several columns, and for Q4_0
    // also for one (measured: 10 % faster on the MTP block's shapes)
    const bool split = g_q80_split >= 0 ? g_q80_split != 0 : rows / 8 < num_sms() * 16;
    const bool two = g_q80_split >= 0 ? g_q80_split == 2 : ((ncols > 1 || TYPE == T_Q4_0) && rows >= 4096);
    if (split && two) {
        switch (ncols) {
        case 1: return launch_q80_split_nc<TYPE, 1, 2>(w, rows, groups, img, y, s, pdl);
        case 2: return launch_q80_split_nc<TYPE, 2, 2>(w, rows, groups, img, y, s, pdl);
        case 3: return launch_q80_split_nc<TYPE, 3, 2>(w, rows, groups, img, y, s, pdl);
        default: return launch_q80_split_nc<TYPE, 4, 2>(w, rows, groups, img, y, s, pdl);
        }
    }
    if (split) {
        switch (ncols) {
        case 1: return launch_q80_split_nc<TYPE, 1>(w, rows, groups, img, y, s, pdl);
        case 2: return launch_q80_split_nc<TYPE, 2>(w, rows, groups, img, y, s, pdl);
        case 3: return launch_q80_split_nc<TYPE, 3>(w, rows, groups, img, y, s, pdl);
        default: return launch_q80_split_nc<TYPE, 4>(w, rows, groups, img, y, s, pdl);
        }
    }
    switch (ncols) {
    case 1: return launch_q80_tile_nc<TYPE, 1>(w, rows, groups, img, y, s, pdl);
    case 2: return launch_q80_tile_nc<TYPE, 2>(w, rows, groups, img, y, s, pdl);
    case 3: return launch_q80_tile_nc<TYPE, 3>(w, rows, groups, img, y, s, pdl);
    default: return launch_q80_tile_nc<TYPE, 4>(w, rows, groups, img, y, s, pdl);
    }
}

// ggml blocks -> tile layout, one CTA per (group, tile), byte by byte through the source offset formula.
template <int TYPE>
__global__ void repack_q80_tiles_kernel(const uint8_t* __restrict__ src, int nb, uint8_t* __restrict__ dst) {
    constexpr int TB = Q80Tile<TYPE>::TB, CODE = Q80Tile<TYPE>::CODE, BB = Q80Tile<TYPE>::BB;
    const int g = blockIdx.x, t = blockIdx.y, groups = nb / 8;
    uint8_t* o = dst + ((size_t)t * groups + g) * TB;
    for (int i = threadIdx.x; i < TB; i += blockDim.x) {
        int r, blk, off;
        if (i < CODE) {
            const int c = i / 512, L = (i % 512) / 16, b = i % 16, tg = L % 4;
            r = L / 4;
            if (TYPE == T_Q8_0) blk = 2 * tg + c / 2, off = 2 + (c % 2) * 16 + b;
            else blk = 2 * tg + c, off = 2 + b;
        } else {
            const int q = i - CODE;
            r = q / 16, blk = (q % 16) / 2, off = q % 2;
        }
        o[i] = src[((size_t)(t * 8 + r) * nb + g * 8 + blk) * BB + off];
    }
}

}  // namespace

void set_q80_split(int mode) { g_q80_split = mode; }

cudaError_t launch_gemv_q80_img(int type, const uint8_t* w, int rows, int cols, const void* img, int ncols, float* y,
                                cudaStream_t s, bool pdl) {
    if (rows <= 0 || ncols <= 0) return cudaSuccess;
    if (rows % 8 || cols % 256) return cudaErrorInvalidValue;
    const int groups = cols / 256;
    for (int c0 = 0; c0 < ncols; c0 += 4) {
        const int nc = std::min(4, ncols - c0);
        const uint8_t* im = (const uint8_t*)img + (size_t)c0 * (cols / 32) * Q80_IMG_BYTES;
        float* yy = y + (size_t)c0 * rows;
        cudaError_t e;
        if (type == T_Q8_0_TILE) e = launch_q80_tile_type<T_Q8_0>(w, rows, groups, im, nc, yy, s, pdl);
        else if (type == T_Q4_0_TILE) e = launch_q80_tile_type<T_Q4_0>(w, rows, groups, im, nc, yy, s, pdl);
        else return cudaErrorInvalidValue;
        if (e != cudaSuccess) return e;
    }
    return cudaSuccess;
}

cudaError_t launch_repack_q80_tiles(int ggml_type, const uint8_t* src, int rows, int cols, uint8_t* dst, cudaStream_t s) {
    if (rows % 8 || cols % 256) return cudaErrorInvalidValue;
    if (rows == 0) return cudaSuccess;
    const dim3 grid(cols / 256, rows / 8);
    if (ggml_type == T_Q8_0) repack_q80_tiles_kernel<T_Q8_0><<<grid, 256, 0, s>>>(src, cols / 32, dst);
    else if (ggml_type == T_Q4_0) repack_q80_tiles_kernel<T_Q4_0><<<grid, 256, 0, s>>>(src, cols / 32, dst);
    else return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_quantize_q80_image(const float* x, int n, int rows, uint8_t* img, cudaStream_t s) {
    const long long blocks = (long long)rows * (n / 32);
    if (blocks == 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((blocks * 32 + 255) / 256, (long long)num_sms() * 16);
    q80_image_kernel<<<grid, 256, 0, s>>>(x, n, rows, img);
    return cudaGetLastError();
}

cudaError_t launch_q80_raw_to_image(const uint8_t* raw, int n, int rows, uint8_t* img, cudaStream_t s) {
    const long long blocks = (long long)rows * (n / 32);
    if (blocks == 0) return cudaSuccess;
    const int grid = (int)std::min<long long>((blocks * 32 + 255) / 256, (long long)num_sms() * 16);
    q80_raw_to_image_kernel<<<grid, 256, 0, s>>>(raw, n / 32, rows, img);
    return cudaGetLastError();
}

}  // namespace qdec
