// Tensor-parallel exchange kernels.  The ranks are processes on the GPUs of one node; each maps the others'
// exchange blocks (CUDA IPC, plain peer stores over NVLink -- no multicast) and the all-gather of a sharded
// activation is one kernel per rank: write its slice to every rank as tagged 16-byte lines, poll its own line
// buffer until every line of the full rows carries the step's tag, unpack.  Stream order then makes the
// gathered rows visible to the kernels that read them.
#include <cuda_runtime.h>

#include <algorithm>

#include "tp.cuh"

namespace qdec {

namespace {

constexpr unsigned long long EXCHANGE_WAIT_NS = 5000000000ull;  // 5 s: a peer this late is treated as gone
constexpr unsigned XSLOT_TAGS = 1024;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void st_line(uint8_t* p, uint32_t d0, uint32_t d1, uint32_t tag) {
    asm volatile("st.volatile.global.v4.u32 [%0], {%1, %2, %3, %4};" ::"l"(p), "r"(d0), "r"(tag), "r"(d1), "r"(tag) : "memory");
}
__device__ __forceinline__ uint4 ld_line(const uint8_t* p) {
    uint4 v;
    asm volatile("ld.volatile.global.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "l"(p) : "memory");
    return v;
}

// which segment (and offset in it) a byte offset of a slice row falls in
__device__ __forceinline__ int seg_of(const XArgs& a, int& o) {
    int s = 0;
    while (s + 1 < a.nseg && o >= a.seg_len[s]) o -= a.seg_len[s++];
    return s;
}

__global__ void __launch_bounds__(256) exchange_kernel(const XArgs a) {
    // launched as a programmatic dependent: wait for the producer of `src`, then let the consumer be scheduled
    // (its own griddepcontrol.wait holds it until this kernel has completed, polls included)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
    const unsigned long long t0 = globaltimer_ns();
    const unsigned tag = *reinterpret_cast<const volatile unsigned*>(a.epoch) * XSLOT_TAGS + (unsigned)a.slot + 1u;
    const long long nthr = (long long)gridDim.x * blockDim.x, tid = blockIdx.x * (long long)blockDim.x + threadIdx.x;
    int rb = 0;
    for (int s = 0; s < a.nseg; s++) rb += a.seg_len[s];
    // push: this rank's slice, 8 bytes per line, to every other rank; and into its own receive buffer
    const int upr = rb / 8;
    for (long long u = tid; u < (long long)upr * a.rows; u += nthr) {
        const int row = (int)(u / upr);
        int o = (int)(u % upr) * 8;
        const int s = seg_of(a, o);
        const uint2 d = *reinterpret_cast<const uint2*>(a.src + row * a.src_ld + a.seg_src[s] + o);
        const long long pos = row * a.dst_ld + a.seg_dst[s] + o;  // byte offset in the full rows
        *reinterpret_cast<uint2*>(a.out + pos) = d;
        for (int k = 0; k < a.world; k++)
            if (k != a.rank) st_line(a.ll[k] + pos * 2, d.x, d.y, tag);
    }
    const unsigned long long t1 = globaltimer_ns();
    // poll: every line of the full rows outside this rank's own slice
    const int lpr = (int)(a.dst_ld / 8);
    bool ok = true;
    for (long long u = tid; u < (long long)lpr * a.rows && ok; u += nthr) {
        const int row = (int)(u / lpr);
        const int b = (int)(u % lpr) * 8;
        bool mine = false;
        for (int s = 0; s < a.nseg; s++) mine |= b >= a.seg_dst[s] && b < a.seg_dst[s] + a.seg_len[s];
        if (mine) continue;
        const long long pos = row * a.dst_ld + b;
        uint4 v = ld_line(a.ll_local + pos * 2);
        if (v.y != tag || v.w != tag) {
            const unsigned long long w0 = globaltimer_ns();
            do {
                __nanosleep(32);
                v = ld_line(a.ll_local + pos * 2);
                if (globaltimer_ns() - w0 > EXCHANGE_WAIT_NS) {
                    atomicCAS(a.err, 0u, 0x10000u | (unsigned)a.slot);
                    ok = false;
                    break;
                }
            } while (v.y != tag || v.w != tag);
        }
        *reinterpret_cast<uint2*>(a.out + pos) = make_uint2(v.x, v.z);
    }
    if (a.stats && threadIdx.x == 0 && blockIdx.x == 0) {
        const unsigned long long t2 = globaltimer_ns();
        atomicAdd(a.stats, 1ull);
        atomicAdd(a.stats + 1, t1 - t0);
        atomicAdd(a.stats + 2, t2 - t1);
    }
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
    for (int i = 0; i < a.nseg; i++)
        if (a.seg_len[i] <= 0 || (a.seg_len[i] | a.seg_src[i] | a.seg_dst[i]) % 16 || a.seg_dst[i] + a.seg_len[i] > a.dst_ld)
            return cudaErrorInvalidValue;
    if (a.src_ld % 16 || a.dst_ld % 16) return cudaErrorInvalidValue;
    const long long lines = a.dst_ld / 8 * a.rows;
    const int grid = (int)std::max<long long>(1, std::min<long long>((lines + 255) / 256, 32));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(256);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, exchange_kernel, a);
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
