// qdec_matvec_noalloc: qdec_matvec for callers that cannot allocate device memory.
//
// qdec_matvec quantises its f32 input columns into a device buffer that the library allocates (and grows) on
// demand.  Some callers cannot let a library call cudaMalloc: an application whose device memory is owned by
// another allocator (a framework's caching allocator that has reserved the GPU), or a decode loop that must
// stay allocation-free once it is running (the rule the reference enforces for its own decode step).  This
// entry point keeps the quantised columns in a fixed array in the library's own device memory instead, so it
// allocates nothing.
//
// The array is a file-scope __device__ object of NOALLOC_SCRATCH_BYTES; every GPU that loads the library holds
// one copy until the process exits.  Host code cannot use the array's name as a device address, so the first
// call on each device looks the address up with cudaGetSymbolAddress (with that device current) and caches it;
// make that first call before any stream capture.  The cached address belongs to the device's primary context:
// cudaDeviceReset destroys that context (and the module copy of the array with it), after which the cached value
// is stale, so a process that resets a device must not call this entry point on that device again.  All calls on a device share the one array and it keeps the
// last call's contents: two calls whose kernels overlap on the GPU (different streams, or host threads) race on
// it.  Nothing in it has to start at zero: every call overwrites the bytes it reads.
#include <cuda_runtime.h>

#include <mutex>

#include "../../include/qdec.h"
#include "capi_util.h"
#include "common.cuh"
#include "kernels.cuh"

namespace qdec {

namespace {

constexpr size_t NOALLOC_SCRATCH_BYTES = 256 * 1024;
__device__ __align__(256) uint8_t g_noalloc_scratch[NOALLOC_SCRATCH_BYTES];

constexpr int MAX_DEVICES = 64;
std::mutex g_mu;
void* g_addr[MAX_DEVICES] = {nullptr};

// The device address of g_noalloc_scratch on the current device (looked up once per device).
int scratch_address(void** out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "qdec_matvec_noalloc: cudaGetDevice");
    if (dev < 0 || dev >= MAX_DEVICES) return fail(QDEC_EINVAL, "qdec_matvec_noalloc: device %d out of range", dev);
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_addr[dev]) {
        void* p = nullptr;
        e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "qdec_matvec_noalloc: cudaGetSymbolAddress");
        g_addr[dev] = p;
    }
    *out = g_addr[dev];
    return QDEC_OK;
}

}  // namespace
}  // namespace qdec

using namespace qdec;

extern "C" size_t qdec_matvec_noalloc_max_bytes(void) { return NOALLOC_SCRATCH_BYTES; }

extern "C" size_t qdec_matvec_scratch_bytes(int ggml_type, const void *w_dev, int cols, int n_cols) {
    if (!supported_type(ggml_type) || cols <= 0 || n_cols < 0 || cols % block_elems(ggml_type)) return (size_t)-1;
    return matvec_scratch_bytes(ggml_type, w_dev, cols, n_cols);
}

extern "C" int qdec_matvec_noalloc(int ggml_type, const void* w_dev, int rows, int cols, const float* x_dev, int n_cols,
                                   float* y_dev, void* stream) {
    int rc = check_gemv_shape(ggml_type, rows, cols, n_cols);
    if (rc) return rc;
    if (!w_dev || !x_dev || !y_dev) return fail(QDEC_EINVAL, "qdec_matvec_noalloc: null pointer");
    if (n_cols == 0) return QDEC_OK;
    cudaStream_t s = (cudaStream_t)stream;
    const size_t need = matvec_scratch_bytes(ggml_type, w_dev, cols, n_cols);
    if (need == 0)  // F32 weights take the f32 columns as they are: no scratch
        return matvec_run(ggml_type, w_dev, rows, cols, x_dev, n_cols, y_dev, s, nullptr, "qdec_matvec_noalloc");
    if (need > NOALLOC_SCRATCH_BYTES)
        return fail(QDEC_EINVAL,
                    "qdec_matvec_noalloc: %d columns of %d values need %zu bytes of quantised activations; the fixed "
                    "scratch holds %zu (use qdec_matvec, or fewer columns per call)",
                    n_cols, cols, need, NOALLOC_SCRATCH_BYTES);
    void* act = nullptr;
    rc = scratch_address(&act);
    if (rc) return rc;
    return matvec_run(ggml_type, w_dev, rows, cols, x_dev, n_cols, y_dev, s, act, "qdec_matvec_noalloc");
}
