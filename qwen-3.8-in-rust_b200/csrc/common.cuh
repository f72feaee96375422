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

// ggml tensor type ids (GGUF), the same numbering as crates/core/src/gguf.rs GgmlType.
enum GgmlType : int { T_F32 = 0, T_F16 = 1, T_Q4_0 = 2, T_Q8_0 = 8, T_Q4_K = 12, T_Q5_K = 13, T_Q6_K = 14 };
// Q6_K in the engine's split layout: 208-byte blocks [ql | qh | scales], then every block's f16 d (gemv_tma.cu).
constexpr int T_Q6_K_SPLIT = 114;

constexpr int QK_K = 256;
constexpr int Q8K_BLOCK_BYTES = 292;  // f32 d, 256 x i8, 16 x i16 (ggml block_q8_K)
constexpr int Q8_0_BLOCK_BYTES = 34;  // f16 d, 32 x i8 (ggml block_q8_0)

__host__ __device__ inline int block_elems(int t) {
    return (t == T_F32) ? 1 : (t == T_Q4_0 || t == T_Q8_0) ? 32 : 256;
}
__host__ __device__ inline int block_bytes(int t) {
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
__host__ __device__ inline bool is_kquant(int t) { return t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_Q6_K_SPLIT; }

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
__device__ __forceinline__ uint16_t ld_nc_u16(const void* p) {
    uint16_t v;
    asm volatile("ld.global.nc.L1::no_allocate.u16 %0, [%1];" : "=h"(v) : "l"(p));
    return v;
}

}  // namespace qdec
