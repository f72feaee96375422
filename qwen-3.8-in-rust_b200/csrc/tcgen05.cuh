// Helpers of the tensor-core kernel (gemm_tc.cu, the prompt prefill GEMM): shared-memory addressing, the
// shared-memory matrix descriptor, mbarriers with bounded waits, the tcgen05 fences and commit, exact
// small-integer conversions, IEEE f32 pairs and the 2-D TMA tensor maps over tile-layout rows.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <stdint.h>

namespace qdec {

constexpr unsigned long long TC_WAIT_NS = 1000000000ull;  // every mbarrier wait gives up after about a second

__device__ __forceinline__ uint32_t smem_addr(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ unsigned long long tc_clock_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

// shared-memory matrix descriptor: canonical K-major layout without swizzle (8-row x 16-byte core matrices;
// lbo = byte distance of the two core matrices along K, sbo = of consecutive 8-row groups), sm100 version bit
__device__ __forceinline__ uint64_t smem_desc(uint32_t addr, uint32_t lbo, uint32_t sbo) {
    return (uint64_t)((addr >> 4) & 0x3FFF) | ((uint64_t)((lbo >> 4) & 0x3FFF) << 16) |
           ((uint64_t)((sbo >> 4) & 0x3FFF) << 32) | (1ull << 46);
}

__device__ __forceinline__ void fence_before_sync() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after_sync() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mbar_init1(uint64_t* bar) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(1u));
}
__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes) : "memory");
}
// bounded wait for the completion of the phase with `parity`; false after about a second
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    const unsigned long long t0 = tc_clock_ns();
    for (uint32_t it = 0;; it++) {
        uint32_t done;
        asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
                     : "=r"(done)
                     : "r"(smem_addr(bar)), "r"(parity)
                     : "memory");
        if (done) return true;
        if ((it & 255) == 255 && tc_clock_ns() - t0 > TC_WAIT_NS) return false;
    }
}
// the completion of every tcgen05 operation this thread issued before, as one arrival on `bar`
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_addr(bar)) : "memory");
}

// f32 of an unsigned byte / signed byte / signed 16-bit value held in the low bits (exact, no conversion unit)
__device__ __forceinline__ float u8f(uint32_t b) { return __fsub_rn(__uint_as_float(0x4B000000u | b), 8388608.0f); }
__device__ __forceinline__ float s8f(uint32_t b) { return __fsub_rn(__uint_as_float(0x4B000000u | ((b ^ 0x80u) & 0xFFu)), 8388736.0f); }
__device__ __forceinline__ float s16f(uint32_t h) {
    return __fsub_rn(__uint_as_float(0x4B000000u | ((h ^ 0x8000u) & 0xFFFFu)), 8421376.0f);
}

// f32 pairs: two of the reference's independent chains side by side, each step the scalar IEEE
// round-to-nearest operation.
__device__ __forceinline__ float2 f2(float a, float b) { return make_float2(a, b); }
__device__ __forceinline__ float2 add2(float2 a, float2 b) { return make_float2(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y)); }
__device__ __forceinline__ float2 mul2(float2 a, float2 b) { return make_float2(__fmul_rn(a.x, b.x), __fmul_rn(a.y, b.y)); }

inline PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static PFN_cuTensorMapEncodeTiled_v12000 fn = [] {
        void* f = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &f, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return (PFN_cuTensorMapEncodeTiled_v12000) nullptr;
        return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(f);
    }();
    return fn;
}

// 2-D map of `outer` rows of `row_bytes` (u64 elements), box = 16 rows x `box_bytes`
inline bool encode_rows(CUtensorMap* m, const void* base, size_t row_bytes, int outer, int box_bytes) {
    auto enc = tensor_map_encoder();
    if (!enc) return false;
    const cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 8), (cuuint64_t)outer};
    const cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    const cuuint32_t box[2] = {(cuuint32_t)(box_bytes / 8), 16u};
    const cuuint32_t estr[2] = {1u, 1u};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_UINT64, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
               CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace qdec
