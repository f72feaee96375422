// Tensor-parallel exchange kernels.  The ranks are processes on the GPUs of one node; each maps the others'
// exchange blocks (CUDA IPC, plain peer stores over NVLink -- no multicast) and the all-gather of a sharded
// activation is one kernel per rank: write its slice to every rank as tagged 8-byte lines, poll its own line
// buffer until every line of the full rows carries the step's tag, unpack.  Stream order then makes the
// gathered rows visible to the kernels that read them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>

#include "tp.cuh"

namespace qdec {

namespace {

constexpr unsigned XSLOT_TAGS = 1024;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// one line {data, tag}: a single naturally aligned 64-bit store / load
__device__ __forceinline__ void st_line(uint8_t* p, uint32_t d, uint32_t tag) {
    const unsigned long long v = (unsigned long long)d | ((unsigned long long)tag << 32);
    asm volatile("st.volatile.global.u64 [%0], %1;" ::"l"(p), "l"(v) : "memory");
}
__device__ __forceinline__ unsigned long long ld_line(const uint8_t* p) {
    unsigned long long v;
    asm volatile("ld.volatile.global.u64 %0, [%1];" : "=l"(v) : "l"(p) : "memory");
    return v;
}
__device__ __forceinline__ bool line_has(unsigned long long v, unsigned tag) { return (unsigned)(v >> 32) == tag; }

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
    // push: this rank's slice, 8 bytes (two lines) per thread step, to every other rank; and into its own
    // receive buffer
    const int upr = rb / 8;
    for (long long u = tid; u < (long long)upr * a.rows; u += nthr) {
        const int row = (int)(u / upr);
        int o = (int)(u % upr) * 8;
        const int s = seg_of(a, o);
        const uint2 d = *reinterpret_cast<const uint2*>(a.src + row * a.src_ld + a.seg_src[s] + o);
        const long long pos = row * a.dst_ld + a.seg_dst[s] + o;  // byte offset in the full rows
        *reinterpret_cast<uint2*>(a.out + pos) = d;
        for (int k = 0; k < a.world; k++)
            if (k != a.rank) {
                st_line(a.ll[k] + pos * 2, d.x, tag);
                st_line(a.ll[k] + pos * 2 + 8, d.y, tag);
            }
    }
    const unsigned long long t1 = globaltimer_ns();
    const unsigned long long lim = a.wait_ns ? a.wait_ns : EXCHANGE_WAIT_NS;
    // poll: every line of the full rows outside this rank's own slice
    const int lpr = (int)(a.dst_ld / 4);
    bool ok = true;
    for (long long u = tid; u < (long long)lpr * a.rows && ok; u += nthr) {
        const int row = (int)(u / lpr);
        const int b = (int)(u % lpr) * 4;
        bool mine = false;
        for (int s = 0; s < a.nseg; s++) mine |= b >= a.seg_dst[s] && b < a.seg_dst[s] + a.seg_len[s];
        if (mine) continue;
        const long long pos = row * a.dst_ld + b;
        unsigned long long v = ld_line(a.ll_local + pos * 2);
        if (!line_has(v, tag)) {
            const unsigned long long w0 = globaltimer_ns();
            do {
                __nanosleep(32);
                v = ld_line(a.ll_local + pos * 2);
                if (globaltimer_ns() - w0 > lim) {
                    atomicCAS(a.err, 0u, 0x10000u | (unsigned)a.slot);
                    ok = false;
                    break;
                }
            } while (!line_has(v, tag));
        }
        if (ok) *reinterpret_cast<uint32_t*>(a.out + pos) = (uint32_t)v;
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
    const long long lines = a.dst_ld / 4 * a.rows;
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

int selftest_exchange(unsigned long long wait_ns) {
    // rank 0 of 2; rows of 64 bytes, this rank's slice the first 32 of each, the "peer's" the last 32
    const int rows = 2, ld = 64, half = 32, slot = 5;
    const unsigned epoch = 7, tag = epoch * XSLOT_TAGS + slot + 1;
    uint8_t *src = nullptr, *out = nullptr, *ll_local = nullptr, *ll_peer = nullptr;
    unsigned* words = nullptr;  // {epoch, err}
    cudaStream_t st = nullptr;
    int rc = 0;
    if (cudaMalloc(&src, rows * half) || cudaMalloc(&out, rows * ld) || cudaMalloc(&ll_local, rows * ld * 2) ||
        cudaMalloc(&ll_peer, rows * ld * 2) || cudaMalloc(&words, 8) || cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking))
        rc = 1;
    uint8_t h_src[rows * half], h_peer[rows * half], h_out[rows * ld];
    unsigned long long lines[rows * ld / 4];
    for (int i = 0; i < rows * half; i++) h_src[i] = (uint8_t)(3 * i + 1), h_peer[i] = (uint8_t)(200 - i);
    auto fill_lines = [&](unsigned t) {  // the lines the peer would have written: its slice under tag t
        for (int r = 0; r < rows; r++)
            for (int b = 0; b < ld; b += 4) {
                uint32_t d = 0;
                if (b >= half) memcpy(&d, h_peer + r * half + (b - half), 4);
                lines[(r * ld + b) / 4] = b >= half ? ((unsigned long long)d | ((unsigned long long)t << 32)) : 0ull;
            }
        return cudaMemcpy(ll_local, lines, sizeof lines, cudaMemcpyHostToDevice);
    };
    XArgs a{};
    a.src = src;
    a.src_ld = half;
    a.ll[1] = ll_peer;
    a.ll_local = ll_local;
    a.out = out;
    a.dst_ld = ld;
    a.seg_src[0] = 0, a.seg_dst[0] = 0, a.seg_len[0] = half;
    a.nseg = 1, a.rows = rows;
    a.epoch = words;
    a.err = words + 1;
    a.slot = slot, a.rank = 0, a.world = 2;
    const unsigned w0[2] = {epoch, 0};
    unsigned hw[2] = {0, 0};
    if (!rc && (cudaMemcpy(src, h_src, sizeof h_src, cudaMemcpyHostToDevice) || cudaMemcpy(words, w0, 8, cudaMemcpyHostToDevice) ||
                fill_lines(tag - 1)))
        rc = 1;
    if (!rc) {  // the peer's lines carry the previous step's tag: the poll must give up
        a.wait_ns = wait_ns;
        if (launch_exchange(a, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess) rc = 2;
        else if (cudaMemcpy(hw, words, 8, cudaMemcpyDeviceToHost) != cudaSuccess || hw[1] != (0x10000u | slot)) rc = 3;
    }
    if (!rc) {  // the peer's lines in place: the step completes with the full rows and no error
        a.wait_ns = 0;
        if (cudaMemcpy(words, w0, 8, cudaMemcpyHostToDevice) || fill_lines(tag) || cudaMemset(out, 0, rows * ld) ||
            launch_exchange(a, st) != cudaSuccess || cudaStreamSynchronize(st) != cudaSuccess)
            rc = 4;
        else if (cudaMemcpy(hw, words, 8, cudaMemcpyDeviceToHost) || cudaMemcpy(h_out, out, sizeof h_out, cudaMemcpyDeviceToHost))
            rc = 4;
        else if (hw[1] != 0)
            rc = 5;
        else
            for (int r = 0; r < rows && !rc; r++)
                if (memcmp(h_out + r * ld, h_src + r * half, half) || memcmp(h_out + r * ld + half, h_peer + r * half, half)) rc = 6;
    }
    if (!rc) {  // and the lines it pushed to the peer: this rank's slice under this step's tag
        unsigned long long pl[rows * ld / 4];
        if (cudaMemcpy(pl, ll_peer, sizeof pl, cudaMemcpyDeviceToHost)) rc = 4;
        for (int r = 0; r < rows && !rc; r++)
            for (int b = 0; b < half && !rc; b += 4) {
                uint32_t d;
                memcpy(&d, h_src + r * half + b, 4);
                if (pl[(r * ld + b) / 4] != ((unsigned long long)d | ((unsigned long long)tag << 32))) rc = 7;
            }
    }
    if (st) cudaStreamDestroy(st);
    cudaFree(src);
    cudaFree(out);
    cudaFree(ll_local);
    cudaFree(ll_peer);
    cudaFree(words);
    return rc;
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
