// Shared device helpers for the qdec kernels (sm_100a).
//
// Arithmetic contract: every float operation that the reference engine performs in a fixed order is
// performed here in the same order with IEEE round-to-nearest and no contraction (the library is built
// with --fmad=false; the explicit __f*_rn intrinsics below make the intent visible where it matters).
#pragma once
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace qdec {

// Programmatic dependent launch on (default) or off (QDEC_PDL=0: every kernel waits for its predecessor to finish
// before it starts, which is what per-kernel timings need).
bool pdl_enabled();

// ggml tensor type ids (GGUF), the same numbering as crates/core/src/gguf.rs GgmlType.
enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };
// Q6_K in the split layout: 208-byte blocks [ql | qh | scales], then every block's f16 d (gemv_v6.cu).
constexpr int T_Q6_K_SPLIT = 114;
// K-quants in the tile layout of gemv_v6.cu (8 rows x one super-block per tile block; rows % 8 == 0).
constexpr int T_Q4_K_TILE = 112, T_Q5_K_TILE = 113, T_Q6_K_TILE = 116;
// Q8_0 / Q4_0 in the tile layout (8 rows x 8 blocks per tile block; rows % 8 == 0, cols % 256 == 0).
constexpr int T_Q8_0_TILE = 108, T_Q4_0_TILE = 102;
__host__ __device__ inline int tile_base_type(int t) {
    return t == T_Q4_K_TILE ? T_Q4_K : t == T_Q5_K_TILE ? T_Q5_K : t == T_Q6_K_TILE ? T_Q6_K
         : t == T_Q8_0_TILE ? T_Q8_0 : t == T_Q4_0_TILE ? T_Q4_0 : t;
}

constexpr int QK_K = 256;
constexpr int Q8K_BLOCK_BYTES = 292;  // f32 d, 256 x i8, 16 x i16 (ggml block_q8_K)

// The engine's device image of one Q8_K block (the GEMV reads it; same values as block_q8_K, rearranged):
//   [0, 256)   the 256 codes, lane-major: word g*8 + s = codes s*32 + 4g .. +3 (the reference's i32 lane g of
//              sub-block s), so the reader of lane g loads 32 contiguous bytes
//   [256, 260) f32 d
//   [272, 304) 8 x (bsums[2g] | bsums[2g+1] << 16)           -- the Q6_K bsum pairs
//   [304, 320) 4 x (q8s[2i] | q8s[2i+1] << 16), q8s[j] = bsums[2j] + bsums[2j+1]  -- the Q4_K/Q5_K min pairs
constexpr int Q8K_IMG_BYTES = 320;
constexpr int Q8K_IMG_D = 256, Q8K_IMG_BSP = 272, Q8K_IMG_Q8S = 304;

// The engine's device image of a row of Q8_0 blocks (the same values as block_q8_0, rearranged): the 32 codes
// of every block back to back (32 bytes per block, 16-byte aligned), then per block {f32 d (the f16 scale,
// converted exactly), i32 sum of the 32 codes} -- 40 bytes per block in all.
constexpr int Q80_IMG_BYTES = 40;
constexpr int Q8_0_BLOCK_BYTES = 34;  // f16 d, 32 x i8 (ggml block_q8_0)

__host__ __device__ inline int block_elems(int t) {
    t = tile_base_type(t);
    return (t == T_F32) ? 1 : (t == T_Q4_0 || t == T_Q8_0) ? 32 : 256;
}
__host__ __device__ inline int block_bytes(int t) {
    t = tile_base_type(t);
    switch (t) {
    case T_F32: return 4;
    case T_Q4_0: return 18;
    case T_Q8_0: return 34;
    case T_Q4_K: return 144;
    case T_Q5_K: return 176;
    case T_Q6_K: return 210;
    case T_Q6_K_SPLIT: return 210;  // 208 in the block array + 2 in the scale array
    default: return 0;
    }
}
__host__ __device__ inline bool is_q80(int t) {
    t = tile_base_type(t);
    return t == T_Q8_0 || t == T_Q4_0;
}
__host__ __device__ inline bool is_kquant(int t) {
    t = tile_base_type(t);
    return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_Q6_K_SPLIT;
}

// Exact f16 -> f32 (the `half` crate's to_f32; hardware conversion is exact).
__device__ __forceinline__ float f16_bits_to_f32(uint16_t h) { return __half2float(__ushort_as_half(h)); }

// exp and log1p in f32, correctly rounded for practical purposes: evaluated in double and rounded once.
// The reference calls the platform libm (f32::exp, f32::ln_1p); this is the correctly-rounded member of
// that family, and the CPU oracle's default mode uses the same formula.
__device__ __forceinline__ float exp_f32(float x) { return (float)exp((double)x); }
__device__ __forceinline__ float log1p_f32(float x) { return (float)log1p((double)x); }

// crates/core/src/kernels/act.rs:7-40
__device__ __forceinline__ float silu_f32(float x) { return __fdiv_rn(x, __fadd_rn(1.0f, exp_f32(-x))); }
__device__ __forceinline__ float sigmoid_f32(float x) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_f32(-x))); }
__device__ __forceinline__ float softplus_f32(float x) { return x > 20.0f ? x : log1p_f32(exp_f32(x)); }

// ((l0+l4)+(l2+l6)) + ((l1+l5)+(l3+l7))  (crates/core/src/kernels/rmsnorm.rs:74)
__device__ __forceinline__ float reduce8(const float* l) {
    return __fadd_rn(__fadd_rn(__fadd_rn(l[0], l[4]), __fadd_rn(l[2], l[6])),
                     __fadd_rn(__fadd_rn(l[1], l[5]), __fadd_rn(l[3], l[7])));
}

__device__ __forceinline__ uint32_t ld_nc_u32(const void* p) {
    uint32_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u32 %0, [%1];" : "=r"(v) : "l"(p));
    return v;
}
__device__ __forceinline__ uint4 ld_nc_u128(const void* p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}
// One Q8_K block quantised by a warp and written as the device image (layout above); lane i holds values
// 8i..8i+7.  Bit-exact with crates/core/src/kernels/q8k.rs:76-114 (the first element of largest |x| sets the
// scale; iscale = -127 / max; q = min(127, round_ties_even(iscale * x)); d = 1 / iscale; bsums per 16).
__device__ __forceinline__ void q8k_quantize_to_image(const float (&v)[8], uint8_t* __restrict__ img) {
    const int lane = threadIdx.x & 31;
    float amax = 0.0f, mx = 0.0f;
    int idx = 0x7fffffff;
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const float a = fabsf(v[i]);
        if (a > amax) amax = a, mx = v[i], idx = lane * 8 + i;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) {
        const float oa = __shfl_xor_sync(0xffffffffu, amax, off);
        const float om = __shfl_xor_sync(0xffffffffu, mx, off);
        const int oi = __shfl_xor_sync(0xffffffffu, idx, off);
        if (oa > amax || (oa == amax && oi < idx)) amax = oa, mx = om, idx = oi;
    }
    uint32_t* ow = reinterpret_cast<uint32_t*>(img);
    if (amax == 0.0f) {  // d = 0, codes 0, sums 0 (q8k.rs:96-101)
        for (int w = lane; w < Q8K_IMG_BYTES / 4; w += 32) ow[w] = 0u;
        return;
    }
    const float iscale = __fdiv_rn(-127.0f, mx);
    int q[8];
#pragma unroll
    for (int i = 0; i < 8; i++) {
        const int qi = __float2int_rn(__fmul_rn(iscale, v[i]));
        q[i] = qi > 127 ? 127 : qi;
    }
    // lane i holds sub-block s = i / 4, positions (i % 4) * 8 .. +7 = reference lanes g = 2(i%4), 2(i%4)+1
    const int s = lane >> 2, g = 2 * (lane & 3);
    ow[g * 8 + s] = (q[0] & 0xff) | ((q[1] & 0xff) << 8) | ((q[2] & 0xff) << 16) | ((uint32_t)(q[3] & 0xff) << 24);
    ow[(g + 1) * 8 + s] = (q[4] & 0xff) | ((q[5] & 0xff) << 8) | ((q[6] & 0xff) << 16) | ((uint32_t)(q[7] & 0xff) << 24);
    int sum8 = q[0] + q[1] + q[2] + q[3] + q[4] + q[5] + q[6] + q[7];
    const int bsum = sum8 + __shfl_xor_sync(0xffffffffu, sum8, 1);   // bsums[lane / 2]
    const int bsum_hi = __shfl_down_sync(0xffffffffu, bsum, 2);      // at lane 4g': bsums[2g'+1]
    const int q8s = (int)(int16_t)(bsum + bsum_hi);                    // at lane 4j: q8s[j]
    const int q8s_hi = __shfl_down_sync(0xffffffffu, q8s, 4);         // at lane 8i: q8s[2i+1]
    if ((lane & 3) == 0) ow[Q8K_IMG_BSP / 4 + (lane >> 2)] = (uint32_t)(bsum & 0xffff) | ((uint32_t)(bsum_hi & 0xffff) << 16);
    if ((lane & 7) == 0) ow[Q8K_IMG_Q8S / 4 + (lane >> 3)] = (uint32_t)(q8s & 0xffff) | ((uint32_t)(q8s_hi & 0xffff) << 16);
    if (lane == 0) {
        ow[Q8K_IMG_D / 4] = __float_as_uint(__fdiv_rn(1.0f, iscale));
        ow[Q8K_IMG_D / 4 + 1] = ow[Q8K_IMG_D / 4 + 2] = ow[Q8K_IMG_D / 4 + 3] = 0u;
    }
}

// One Q8_0 block quantised by a warp (lane i holds value i) into the row image: codes at `codes`, {d, sum} at
// `meta`.  Bit-exact with crates/core/src/kernels/q8.rs:81-103: d = amax / 127 stored as f16, id = 1/d (0 for a
// zero block), q = round-half-away(x * id) saturated to i8.
__device__ __forceinline__ void q80_quantize_to_image(float v, uint8_t* __restrict__ codes, uint8_t* __restrict__ meta) {
    const int lane = threadIdx.x & 31;
    float amax = fabsf(v);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float dd = __fdiv_rn(amax, 127.0f);
    const float id = dd != 0.0f ? __fdiv_rn(1.0f, dd) : 0.0f;
    const float qf = roundf(__fmul_rn(v, id));
    const int qi = qf > 127.0f ? 127 : (qf < -128.0f ? -128 : (int)qf);
    const uint32_t b = (uint32_t)(qi & 0xff) << (8 * (lane & 3));
    uint32_t wv = b | __shfl_xor_sync(0xffffffffu, b, 1);
    wv |= __shfl_xor_sync(0xffffffffu, wv, 2);
    const int sum = __reduce_add_sync(0xffffffffu, qi);
    if ((lane & 3) == 0) reinterpret_cast<uint32_t*>(codes)[lane >> 2] = wv;
    if (lane == 0) {
        reinterpret_cast<float*>(meta)[0] = __half2float(__float2half_rn(dd));
        reinterpret_cast<int*>(meta)[1] = sum;
    }
}

__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

}  // namespace qdec
