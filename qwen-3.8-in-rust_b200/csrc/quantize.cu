// Activation quantisers and row dequantisation.
//
//  * q8k_quantize_kernel  -- ggml block_q8_K rows, bit-exact with crates/core/src/kernels/q8k.rs:76-114
//  * q8_0_quantize_kernel -- ggml block_q8_0 rows, bit-exact with crates/core/src/kernels/q8.rs:81-103
//  * dequant_rows_kernel  -- f32 rows from ggml blocks, bit-exact with crates/core/src/quant.rs:67-229
//    (the embedding gather of crates/core/src/model.rs:364-368)
#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

// One warp per 256-value block; lane i holds values 8i..8i+7.
__global__ void q8k_quantize_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ out) {
    const int nb = n / QK_K;
    const long long total = (long long)rows * nb;
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < total; b += nwarps) {
        const long long r = b / nb, sb = b % nb;
        const float* blk = x + r * (long long)n + sb * QK_K;
        float v[8];
        const float4 a0 = reinterpret_cast<const float4*>(blk)[2 * lane];
        const float4 a1 = reinterpret_cast<const float4*>(blk)[2 * lane + 1];
        v[0] = a0.x; v[1] = a0.y; v[2] = a0.z; v[3] = a0.w;
        v[4] = a1.x; v[5] = a1.y; v[6] = a1.z; v[7] = a1.w;
        // the first element with the largest |x| (strict > scan of q8k.rs:88-95)
        float amax = 0.0f, mx = 0.0f;
        int idx = 0x7fffffff;
        for (int i = 0; i < 8; i++) {
            float a = fabsf(v[i]);
            if (a > amax) { amax = a; mx = v[i]; idx = lane * 8 + i; }
        }
        for (int off = 16; off > 0; off >>= 1) {
            float oa = __shfl_xor_sync(0xffffffffu, amax, off);
            float om = __shfl_xor_sync(0xffffffffu, mx, off);
            int oi = __shfl_xor_sync(0xffffffffu, idx, off);
            if (oa > amax || (oa == amax && oi < idx)) { amax = oa; mx = om; idx = oi; }
        }
        uint8_t* o = out + b * Q8K_BLOCK_BYTES;
        if (amax == 0.0f) {
            // d = 0, codes 0, bsums 0 (q8k.rs:96-101); 292 bytes = 73 words
            for (int w = lane; w < 73; w += 32) reinterpret_cast<uint32_t*>(o)[w] = 0u;
            continue;
        }
        const float iscale = __fdiv_rn(-127.0f, mx);
        int q[8];
        for (int i = 0; i < 8; i++) {
            int qi = __float2int_rn(__fmul_rn(iscale, v[i]));  // round_ties_even, then min(127)
            q[i] = qi > 127 ? 127 : qi;
        }
        uint32_t w0 = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
        uint32_t w1 = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
        reinterpret_cast<uint32_t*>(o + 4)[2 * lane] = w0;
        reinterpret_cast<uint32_t*>(o + 4)[2 * lane + 1] = w1;
        int s = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
        s += __shfl_xor_sync(0xffffffffu, s, 1);  // group g = lanes 2g, 2g+1
        if ((lane & 1) == 0) reinterpret_cast<int16_t*>(o + 260)[lane >> 1] = (int16_t)s;
        if (lane == 0) {
            const float d = __fdiv_rn(1.0f, iscale);
            *reinterpret_cast<float*>(o) = d;
        }
    }
}

// f32 rows -> the engine's Q8_K device image (common.cuh), one warp per 256-value block.
__global__ void q8k_image_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ img) {
    const int nb = n / QK_K;
    const long long total = (long long)rows * nb;
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < total; b += nwarps) {
        const long long r = b / nb, sb = b % nb;
        const float4* blk = reinterpret_cast<const float4*>(x + r * (long long)n + sb * QK_K);
        const float4 a0 = blk[2 * lane], a1 = blk[2 * lane + 1];
        const float v[8] = {a0.x, a0.y, a0.z, a0.w, a1.x, a1.y, a1.z, a1.w};
        q8k_quantize_to_image(v, img + b * Q8K_IMG_BYTES);
    }
}

// ggml block_q8_K rows -> the device image: the same values, rearranged (one warp per block).
__global__ void q8k_raw_to_image_kernel(const uint8_t* __restrict__ raw, long long nblocks, uint8_t* __restrict__ img) {
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < nblocks; b += nwarps) {
        const uint32_t* r = reinterpret_cast<const uint32_t*>(raw + b * Q8K_BLOCK_BYTES);
        uint32_t* o = reinterpret_cast<uint32_t*>(img + b * Q8K_IMG_BYTES);
        for (int c = lane; c < 64; c += 32) o[(c & 7) * 8 + (c >> 3)] = r[1 + c];  // codes word c: s = c/8, g = c%8
        if (lane < 8) {
            const uint32_t pr = r[65 + lane];  // bsums[2g], bsums[2g+1]
            o[Q8K_IMG_BSP / 4 + lane] = pr;
            const int q8s = (int)(int16_t)((int16_t)(pr & 0xffff) + (int16_t)(pr >> 16));  // q8s[lane]
            const int q8s_hi = __shfl_down_sync(0xffu, q8s, 1, 8);
            if ((lane & 1) == 0) o[Q8K_IMG_Q8S / 4 + lane / 2] = (uint32_t)(q8s & 0xffff) | ((uint32_t)(q8s_hi & 0xffff) << 16);
        }
        if (lane == 8) o[Q8K_IMG_D / 4] = r[0];
        if (lane >= 9 && lane < 12) o[Q8K_IMG_D / 4 + lane - 8] = 0u;
    }
}

// f32 rows -> the engine's Q8_0 row image (common.cuh), one warp per 32-value block.
__global__ void q80_image_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ img) {
    const int nb = n / 32;
    const long long total = (long long)rows * nb;
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < total; b += nwarps) {
        const long long r = b / nb, blk = b % nb;
        uint8_t* row = img + r * nb * Q80_IMG_BYTES;
        q80_quantize_to_image(x[r * (long long)n + blk * 32 + lane], row + blk * 32, row + (size_t)nb * 32 + blk * 8);
    }
}

// block_q8_0 rows -> the Q8_0 row image: the same values, rearranged (one warp per block).
__global__ void q80_raw_to_image_kernel(const uint8_t* __restrict__ raw, int nb, int rows, uint8_t* __restrict__ img) {
    const long long total = (long long)rows * nb;
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < total; b += nwarps) {
        const long long r = b / nb, blk = b % nb;
        const uint8_t* src = raw + b * Q8_0_BLOCK_BYTES;
        uint8_t* row = img + r * nb * Q80_IMG_BYTES;
        const int q = (int)(int8_t)src[2 + lane];
        const uint32_t bb = (uint32_t)(q & 0xff) << (8 * (lane & 3));
        uint32_t wv = bb | __shfl_xor_sync(0xffffffffu, bb, 1);
        wv |= __shfl_xor_sync(0xffffffffu, wv, 2);
        const int sum = __reduce_add_sync(0xffffffffu, q);
        if ((lane & 3) == 0) reinterpret_cast<uint32_t*>(row + blk * 32)[lane >> 2] = wv;
        if (lane == 0) {
            uint8_t* meta = row + (size_t)nb * 32 + blk * 8;
            reinterpret_cast<float*>(meta)[0] = f16_bits_to_f32((uint16_t)(src[0] | (src[1] << 8)));
            reinterpret_cast<int*>(meta)[1] = sum;
        }
    }
}

// One warp per 32-value block; lane i holds value i.
__global__ void q8_0_quantize_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ out) {
    const int nb = n / 32;
    const long long total = (long long)rows * nb;
    const int lane = threadIdx.x & 31;
    const long long warp0 = ((long long)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
    const long long nwarps = ((long long)gridDim.x * blockDim.x) >> 5;
    for (long long b = warp0; b < total; b += nwarps) {
        const long long r = b / nb, blk = b % nb;
        const float v = x[r * (long long)n + blk * 32 + lane];
        float amax = fabsf(v);
        for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
        const float dd = __fdiv_rn(amax, 127.0f);
        const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
        float qf = roundf(__fmul_rn(v, id));  // round half away from zero, then `as i8` (saturating)
        const int qi = qf > 127.0f ? 127 : (qf < -128.0f ? -128 : (int)qf);
        // the 34-byte block as 17 half-words: lane 0 the f16 scale, lane j (1..16) codes 2j-2 and 2j-1
        const int lo = __shfl_sync(0xffffffffu, qi, (2 * lane - 2) & 31);
        const int hi = __shfl_sync(0xffffffffu, qi, (2 * lane - 1) & 31);
        uint16_t* o = reinterpret_cast<uint16_t*>(out + b * Q8_0_BLOCK_BYTES);
        if (lane == 0) {
            o[0] = __half_as_ushort(__float2half_rn(dd));
        } else if (lane <= 16) {
            o[lane] = (uint16_t)((lo & 0xff) | ((hi & 0xff) << 8));
        }
    }
}

__device__ __forceinline__ float f16_at(const uint8_t* b, int off) {
    return f16_bits_to_f32((uint16_t)(b[off] | (b[off + 1] << 8)));
}

__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, int& sc, int& m) {
    if (j < 4) {
        sc = q[j] & 63;
        m = q[j + 4] & 63;
    } else {
        sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

// Value e of a block, exactly as crates/core/src/quant.rs computes it.
__device__ float dequant_value(int type, const uint8_t* b, int e) {
    switch (type) {
    case T_F32: return *reinterpret_cast<const float*>(b);  // F32: one element per 4-byte "block"
    case T_Q4_0: {
        const float d = f16_at(b, 0);
        const int j = e & 15;
        const int q = (e < 16) ? (b[2 + j] & 0x0F) : (b[2 + j] >> 4);
        return __fmul_rn((float)(q - 8), d);
    }
    case T_Q8_0: return __fmul_rn((float)(int8_t)b[2 + e], f16_at(b, 0));
    case T_Q4_K:
    case T_Q5_K: {
        const float d = f16_at(b, 0), mn = f16_at(b, 2);
        const int g = e / 64, hi = (e / 32) & 1, l = e & 31;
        int sc, m;
        scale_min_k4(2 * g + hi, b + 4, sc, m);
        const float d1 = __fmul_rn(d, (float)sc), m1 = __fmul_rn(mn, (float)m);
        int q;
        if (type == T_Q4_K) {
            const uint8_t byte = b[16 + g * 32 + l];
            q = hi ? (byte >> 4) : (byte & 0xF);
        } else {
            const uint8_t byte = b[48 + g * 32 + l];
            q = (hi ? (byte >> 4) : (byte & 0xF)) + ((b[16 + l] & (1u << (2 * g + hi))) ? 16 : 0);
        }
        return __fsub_rn(__fmul_rn(d1, (float)q), m1);
    }
    case T_Q6_K: {
        const float d = f16_at(b, 208);
        const int half = e / 128, r = e & 127, k = r / 32, l = r & 31;
        const uint8_t* ql = b + half * 64;
        const uint8_t* qh = b + 128 + half * 32;
        const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192 + half * 8);
        const int lo = (k == 0) ? (ql[l] & 0xF) : (k == 1) ? (ql[l + 32] & 0xF) : (k == 2) ? (ql[l] >> 4) : (ql[l + 32] >> 4);
        const int q = (lo | (((qh[l] >> (2 * k)) & 3) << 4)) - 32;
        const int is = l / 16;
        return __fmul_rn(__fmul_rn(d, (float)sc[is + 2 * k]), (float)q);
    }
    default: return 0.0f;
    }
}

// out[i * n + e] = dequant(row ids[i])[e]; ids and the row count are on the device so a CUDA graph can gather
// the token ids the previous kernel wrote.
__global__ void dequant_rows_kernel(int type, const uint8_t* __restrict__ w, size_t row_bytes, int n,
                                    const int32_t* __restrict__ ids, int nids, float* __restrict__ out) {
    const int be = block_elems(type), bb = block_bytes(type);
    for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < (long long)nids * n;
         i += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(i / n), e = (int)(i % n);
        const uint8_t* rb = w + (size_t)ids[row] * row_bytes;
        out[i] = dequant_value(type, rb + (size_t)(e / be) * bb, e % be);
    }
}

}  // namespace qdec
