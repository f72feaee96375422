// Tensor-parallel exchange kernels.  The ranks are processes on the GPUs of one node; each maps the others'
// exchange blocks (CUDA IPC, plain peer loads and stores over NVLink -- no multicast) and the all-gather of a
// sharded activation is one kernel per rank: copy the slice to every rank, fence, flag, wait for every flag.
// Stream order then makes the gathered rows visible to the kernels that read them.
#include <cuda_runtime.h>

#include <algorithm>

#include "tp.cuh"

namespace qdec {

namespace {

constexpr unsigned long long EXCHANGE_WAIT_NS = 5000000000ull;  // 5 s: a peer this late is treated as gone

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned* p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ void st_release_sys(unsigned* p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__global__ void __launch_bounds__(256) exchange_kernel(const XArgs a) {
    int rb = 0;
    for (int s = 0; s < a.nseg; s++) rb += a.seg_len[s];
    const int vpr = rb / 16;
    const long long total = (long long)vpr * a.rows;
    for (long long v = blockIdx.x * (long long)blockDim.x + threadIdx.x; v < total; v += (long long)gridDim.x * blockDim.x) {
        const int row = (int)(v / vpr);
        int o = (int)(v % vpr) * 16, s = 0;
        while (s + 1 < a.nseg && o >= a.seg_len[s]) o -= a.seg_len[s++];
        const uint4 val = *reinterpret_cast<const uint4*>(a.src + row * a.src_ld + a.seg_src[s] + o);
        for (int k = 0; k < a.world; k++) *reinterpret_cast<uint4*>(a.dst[k] + row * a.dst_ld + a.seg_dst[s] + o) = val;
    }
    __shared__ bool last;
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();  // this CTA's stores (ordered by the barrier) before its count
        last = atomicAdd(&a.cnt[a.slot], 1u) == gridDim.x - 1;
    }
    __syncthreads();
    if (!last || threadIdx.x != 0) return;
    a.cnt[a.slot] = 0u;
    __threadfence_system();  // every CTA's stores before the flags
    const unsigned e = *reinterpret_cast<const volatile unsigned*>(a.epoch);
    for (int k = 0; k < a.world; k++) st_release_sys(a.pflags[k] + a.slot * 8 + a.rank, e);
    const unsigned long long t0 = globaltimer_ns();
    for (int k = 0; k < a.world; k++) {
        // flags only grow (one session's value per use); a peer cannot run a whole session ahead of this rank
        while ((int)(ld_acquire_sys(a.lflags + a.slot * 8 + k) - e) < 0) {
            if (globaltimer_ns() - t0 > EXCHANGE_WAIT_NS) {
                atomicCAS(a.err, 0u, 0x10000u | (unsigned)a.slot);
                return;
            }
            __nanosleep(64);
        }
    }
    __threadfence_system();
}

__global__ void epoch_kernel(unsigned* e) { *e += 1u; }

__global__ void argmax_combine_kernel(const uint8_t* __restrict__ pairs, int world, int rows, int32_t* __restrict__ out) {
    const int row = blockIdx.x * blockDim.x + threadIdx.x;
    if (row >= rows) return;
    const uint8_t* p = pairs + (size_t)row * world * 16;
    float g = *reinterpret_cast<const float*>(p);
    int gi = *reinterpret_cast<const int*>(p + 4);
    for (int k = 1; k < world; k++) {
        const float v = *reinterpret_cast<const float*>(p + 16 * k);
        const int i = *reinterpret_cast<const int*>(p + 16 * k + 4);
        if (i >= 0 && (gi < 0 || v > g)) g = v, gi = i;
    }
    out[row] = gi;
}

}  // namespace

cudaError_t launch_exchange(const XArgs& a, cudaStream_t s) {
    if (a.world < 1 || a.world > 8 || a.nseg < 1 || a.nseg > 4 || a.rows <= 0) return cudaErrorInvalidValue;
    int rb = 0;
    for (int i = 0; i < a.nseg; i++) {
        if (a.seg_len[i] <= 0 || (a.seg_len[i] | a.seg_src[i] | a.seg_dst[i]) % 16) return cudaErrorInvalidValue;
        rb += a.seg_len[i];
    }
    if (a.src_ld % 16 || a.dst_ld % 16) return cudaErrorInvalidValue;
    const long long vec = (long long)rb / 16 * a.rows;
    const int grid = (int)std::min<long long>((vec + 255) / 256, 64);
    exchange_kernel<<<grid, 256, 0, s>>>(a);
    return cudaGetLastError();
}

cudaError_t launch_tp_epoch(unsigned* epoch, cudaStream_t s) {
    epoch_kernel<<<1, 1, 0, s>>>(epoch);
    return cudaGetLastError();
}

cudaError_t launch_argmax_combine(const uint8_t* pairs, int world, int rows, int32_t* out, cudaStream_t s) {
    argmax_combine_kernel<<<(rows + 127) / 128, 128, 0, s>>>(pairs, world, rows, out);
    return cudaGetLastError();
}

}  // namespace qdec
