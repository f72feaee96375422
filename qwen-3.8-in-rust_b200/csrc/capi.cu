// The kernel-level C ABI (include/qdec.h): argument checks in the reference's terms, error strings, and the
// library-owned activation buffer of qdec_matvec.
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/qdec.h"
#include "capi_util.h"
#include "common.cuh"
#include "kernels.cuh"
#include "tp.cuh"

namespace qdec {

static thread_local std::string g_last_error;

int fail(int code, const char *fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int cuda_fail(cudaError_t e, const char *what) {
    return fail(QDEC_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

void clear_error() { g_last_error.clear(); }

bool supported_type(int t) {
    return t == T_F32 || t == T_Q4_0 || t == T_Q8_0 || t == T_Q4_K || t == T_Q5_K || t == T_Q6_K || t == T_Q6_K_SPLIT ||
           t == T_Q4_K_TILE || t == T_Q5_K_TILE || t == T_Q6_K_TILE || t == T_Q8_0_TILE || t == T_Q4_0_TILE;
}

// Shape checks of the reference's assert!s (matvec.rs:73-77, :300, :338; kdot.rs:179-191).
int check_gemv_shape(int type, int rows, int cols, int ncols) {
    if (!supported_type(type)) return fail(QDEC_EINVAL, "unsupported weight type %d", type);
    if (rows < 0 || cols <= 0 || ncols < 0) return fail(QDEC_EINVAL, "bad shape rows=%d cols=%d n_cols=%d", rows, cols, ncols);
    const int be = block_elems(type);
    if (cols % be) return fail(QDEC_EINVAL, "cols %d not a multiple of block size %d for type %d", cols, be, type);
    if ((type == T_Q8_0 || type == T_Q4_0) && cols % 64)
        return fail(QDEC_EINVAL, "cols %d: Q8_0/Q4_0 rows must hold an even number of 32-blocks", cols);
    if (tile_base_type(type) != type && rows % 8)
        return fail(QDEC_EINVAL, "rows %d: the tile layout holds a multiple of 8 rows", rows);
    if ((type == T_Q8_0_TILE || type == T_Q4_0_TILE) && cols % 256)
        return fail(QDEC_EINVAL, "cols %d: the Q8_0/Q4_0 tile layout holds a multiple of 256 columns", cols);
    if (is_kquant(type)) {
        const size_t smem = (size_t)4 * (cols / 256) * 324 + 64;  // the raw-activation kernel stages 4 columns
        if (smem > 220 * 1024) return fail(QDEC_EINVAL, "cols %d too wide for the staged activations", cols);
    }
    return QDEC_OK;
}

// Library-owned activation buffer per device for qdec_matvec.
struct ActPool {
    std::mutex mu;
    std::vector<void *> buf;
    std::vector<size_t> cap;
};
static ActPool g_act;

static int act_buffer(size_t bytes, void **out) {
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
    std::lock_guard<std::mutex> lk(g_act.mu);
    if ((int)g_act.buf.size() <= dev) g_act.buf.resize(dev + 1, nullptr), g_act.cap.resize(dev + 1, 0);
    if (g_act.cap[dev] < bytes) {
        if (g_act.buf[dev]) cudaFree(g_act.buf[dev]);
        g_act.buf[dev] = nullptr;
        g_act.cap[dev] = 0;
        e = cudaMalloc(&g_act.buf[dev], bytes);
        if (e != cudaSuccess) return fail(QDEC_ENOMEM, "activation buffer of %zu bytes: %s", bytes, cudaGetErrorString(e));
        g_act.cap[dev] = bytes;
    }
    *out = g_act.buf[dev];
    return QDEC_OK;
}

bool uses_image(int type, const void *w_dev) {
    return gemv_impl() != 2 && v6_gemv_supported(type) && ((uintptr_t)w_dev & 15) == 0;
}

size_t image_bytes(int cols, int n_cols) { return (size_t)(cols / QK_K) * Q8K_IMG_BYTES * n_cols; }

size_t matvec_scratch_bytes(int type, const void *w_dev, int cols, int n_cols) {
    if (type == T_F32) return 0;
    if (type == T_Q8_0_TILE || type == T_Q4_0_TILE) return (size_t)(cols / 32) * Q80_IMG_BYTES * n_cols;
    if (uses_image(type, w_dev)) return image_bytes(cols, n_cols);
    return act_row_bytes(type, cols) * n_cols;
}

int matvec_run(int type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols, float *y_dev, cudaStream_t s,
               void *scratch, const char *who) {
    const uint8_t *w = (const uint8_t *)w_dev;
    cudaError_t e;
    if (type == T_F32) {
        e = launch_gemv(type, w, rows, cols, x_dev, n_cols, y_dev, s);
        return e == cudaSuccess ? QDEC_OK : cuda_fail(e, who);
    }
    if (type == T_Q8_0_TILE || type == T_Q4_0_TILE) {
        e = launch_quantize_q80_image(x_dev, cols, n_cols, (uint8_t *)scratch, s);
        if (e != cudaSuccess) return cuda_fail(e, who);
        e = launch_gemv_q80_img(type, w, rows, cols, scratch, n_cols, y_dev, s, false);
        return e == cudaSuccess ? QDEC_OK : cuda_fail(e, who);
    }
    if (uses_image(type, w_dev)) {
        e = launch_quantize_q8k_image(x_dev, cols, n_cols, (uint8_t *)scratch, s);
        if (e != cudaSuccess) return cuda_fail(e, who);
        e = launch_gemv_img(type, w, rows, cols, scratch, n_cols, y_dev, s, false);
        return e == cudaSuccess ? QDEC_OK : cuda_fail(e, who);
    }
    e = is_kquant(type) ? launch_quantize_q8k(x_dev, cols, n_cols, (uint8_t *)scratch, s)
                        : launch_quantize_q8_0(x_dev, cols, n_cols, (uint8_t *)scratch, s);
    if (e != cudaSuccess) return cuda_fail(e, who);
    e = launch_gemv(type, w, rows, cols, scratch, n_cols, y_dev, s);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, who);
}

}  // namespace qdec

using namespace qdec;

extern "C" {

const char *qdec_version(void) { return "qdec 0.1.0 sm_100a"; }

const char *qdec_last_error(void) { return g_last_error.c_str(); }

int qdec_quantize_q8k(const float *x_dev, int n, int rows, void *q8k_dev, void *stream) {
    if (n <= 0 || n % 256 || rows < 0) return fail(QDEC_EINVAL, "qdec_quantize_q8k: length %d is not a multiple of 256", n);
    if (!x_dev || !q8k_dev) return fail(QDEC_EINVAL, "qdec_quantize_q8k: null pointer");
    cudaError_t e = launch_quantize_q8k(x_dev, n, rows, (uint8_t *)q8k_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_quantize_q8k");
}

int qdec_quantize_q8_0(const float *x_dev, int n, int rows, void *q8_dev, void *stream) {
    if (n <= 0 || n % 32 || rows < 0) return fail(QDEC_EINVAL, "qdec_quantize_q8_0: length %d is not a multiple of 32", n);
    if (!x_dev || !q8_dev) return fail(QDEC_EINVAL, "qdec_quantize_q8_0: null pointer");
    cudaError_t e = launch_quantize_q8_0(x_dev, n, rows, (uint8_t *)q8_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_quantize_q8_0");
}

size_t qdec_act_row_bytes(int ggml_type, int cols) {
    if (!supported_type(ggml_type) || cols <= 0 || cols % block_elems(ggml_type)) return 0;
    return act_row_bytes(ggml_type, cols);
}

int qdec_gemv(int ggml_type, const void *w_dev, int rows, int cols, const void *act_dev, int n_cols, float *y_dev,
              void *stream) {
    int rc = check_gemv_shape(ggml_type, rows, cols, n_cols);
    if (rc) return rc;
    if (!w_dev || !act_dev || !y_dev) return fail(QDEC_EINVAL, "qdec_gemv: null pointer");
    if (n_cols == 0 || rows == 0) return QDEC_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (ggml_type == T_Q8_0_TILE || ggml_type == T_Q4_0_TILE) {  // block_q8_0 rows -> the Q8_0 row image
        void *img = nullptr;
        rc = act_buffer((size_t)(cols / 32) * Q80_IMG_BYTES * n_cols, &img);
        if (rc) return rc;
        cudaError_t e = launch_q80_raw_to_image((const uint8_t *)act_dev, cols, n_cols, (uint8_t *)img, s);
        if (e != cudaSuccess) return cuda_fail(e, "qdec_gemv: activation image");
        e = launch_gemv_q80_img(ggml_type, (const uint8_t *)w_dev, rows, cols, img, n_cols, y_dev, s, false);
        return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_gemv");
    }
    if (uses_image(ggml_type, w_dev)) {  // rearrange the block_q8_K rows into the image the kernel reads
        void *img = nullptr;
        rc = act_buffer(image_bytes(cols, n_cols), &img);
        if (rc) return rc;
        cudaError_t e = launch_q8k_raw_to_image((const uint8_t *)act_dev, (long long)n_cols * (cols / QK_K), (uint8_t *)img, s);
        if (e != cudaSuccess) return cuda_fail(e, "qdec_gemv: activation image");
        e = launch_gemv_img(ggml_type, (const uint8_t *)w_dev, rows, cols, img, n_cols, y_dev, s, false);
        return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_gemv");
    }
    cudaError_t e = launch_gemv(ggml_type, (const uint8_t *)w_dev, rows, cols, act_dev, n_cols, y_dev, s);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_gemv");
}

int qdec_matvec(int ggml_type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols, float *y_dev,
                void *stream) {
    int rc = check_gemv_shape(ggml_type, rows, cols, n_cols);
    if (rc) return rc;
    if (!w_dev || !x_dev || !y_dev) return fail(QDEC_EINVAL, "qdec_matvec: null pointer");
    if (n_cols == 0) return QDEC_OK;
    void *act = nullptr;
    const size_t need = matvec_scratch_bytes(ggml_type, w_dev, cols, n_cols);
    if (need) {
        rc = act_buffer(need, &act);
        if (rc) return rc;
    }
    return matvec_run(ggml_type, w_dev, rows, cols, x_dev, n_cols, y_dev, (cudaStream_t)stream, act, "qdec_matvec");
}

size_t qdec_image_row_bytes(int ggml_type, int cols) {
    if (cols <= 0) return 0;
    if (is_q80(ggml_type)) return cols % 32 ? 0 : (size_t)(cols / 32) * Q80_IMG_BYTES;
    if (is_kquant(ggml_type)) return cols % QK_K ? 0 : (size_t)(cols / QK_K) * Q8K_IMG_BYTES;
    return 0;
}

int qdec_quantize_image(int ggml_type, const float *x_dev, int n, int rows, void *img_dev, void *stream) {
    if (!x_dev || !img_dev || rows < 0 || !qdec_image_row_bytes(ggml_type, n))
        return fail(QDEC_EINVAL, "qdec_quantize_image: bad argument (type %d, length %d)", ggml_type, n);
    cudaError_t e = is_q80(ggml_type) ? launch_quantize_q80_image(x_dev, n, rows, (uint8_t *)img_dev, (cudaStream_t)stream)
                                      : launch_quantize_q8k_image(x_dev, n, rows, (uint8_t *)img_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_quantize_image");
}

int qdec_gemv_image(int ggml_type, const void *w_dev, int rows, int cols, const void *img_dev, int n_cols, float *y_dev,
                    void *stream) {
    int rc = check_gemv_shape(ggml_type, rows, cols, n_cols);
    if (rc) return rc;
    if (!w_dev || !img_dev || !y_dev) return fail(QDEC_EINVAL, "qdec_gemv_image: null pointer");
    if (((uintptr_t)w_dev & 15) != 0) return fail(QDEC_EINVAL, "qdec_gemv_image: weights must be 16-byte aligned");
    if (((uintptr_t)img_dev & 15) != 0) return fail(QDEC_EINVAL, "qdec_gemv_image: the image must be 16-byte aligned");
    cudaError_t e;
    if (ggml_type == T_Q8_0_TILE || ggml_type == T_Q4_0_TILE)
        e = launch_gemv_q80_img(ggml_type, (const uint8_t *)w_dev, rows, cols, img_dev, n_cols, y_dev, (cudaStream_t)stream, false);
    else if (v6_gemv_supported(ggml_type))
        e = launch_gemv_img(ggml_type, (const uint8_t *)w_dev, rows, cols, img_dev, n_cols, y_dev, (cudaStream_t)stream, false);
    else
        return fail(QDEC_EINVAL, "qdec_gemv_image: type %d does not read the activation image", ggml_type);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_gemv_image");
}

int qdec_gemv_image_pair(int ggml_type, const void *w1_dev, const void *w2_dev, int rows, int cols, const void *img_dev,
                         int n_cols, float *y1_dev, float *y2_dev, void *stream) {
    int rc = check_gemv_shape(ggml_type, rows, cols, n_cols);
    if (rc) return rc;
    if (!w1_dev || !w2_dev || !img_dev || !y1_dev || !y2_dev) return fail(QDEC_EINVAL, "qdec_gemv_image_pair: null pointer");
    if (ggml_type != T_Q4_K_TILE && ggml_type != T_Q5_K_TILE && ggml_type != T_Q6_K_TILE)
        return fail(QDEC_EINVAL, "qdec_gemv_image_pair: type %d is not a K-quant tile type", ggml_type);
    if ((((uintptr_t)w1_dev | (uintptr_t)w2_dev | (uintptr_t)img_dev) & 15) != 0)
        return fail(QDEC_EINVAL, "qdec_gemv_image_pair: weights and image must be 16-byte aligned");
    if (n_cols == 0 || rows == 0) return QDEC_OK;
    const cudaError_t e = launch_gemv_img_pair(ggml_type, (const uint8_t *)w1_dev, rows, y1_dev, (const uint8_t *)w2_dev, rows,
                                               y2_dev, cols, img_dev, n_cols, (cudaStream_t)stream, false);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_gemv_image_pair");
}

int qdec_tune_gemv(int impl, int config) {
    if (impl == 8) {  // the Q8_0 / Q4_0 tile kernel: 0 automatic, 1 one warp per tile, 2 split group range,
                      // 3 split group range with two tiles per CTA
        if (config < 0 || config > 3) return fail(QDEC_EINVAL, "Q8_0 gemv configuration must be 0..3");
        set_q80_split(config - 1);
        return QDEC_OK;
    }
    if (impl == 9) {  // the tensor-core prefill GEMM: the smallest column count routed to it (0 = never)
        if (config < 0) return fail(QDEC_EINVAL, "prefill GEMM minimum column count must be >= 0");
        set_gemm_tc_min_cols(config);
        return QDEC_OK;
    }
    if (impl == 10) {  // the warp-MMA form of the Q4_K tile GEMV: the smallest column group routed to it (0 = never)
        if (config < 0 || config > 4) return fail(QDEC_EINVAL, "warp-MMA minimum column count must be 0..4");
        set_gemv7_mma_min_cols(config);
        return QDEC_OK;
    }
    if (impl == 7) {  // the decode GEMV of tile matrices: 0 automatic by shape, 1..8 a fixed configuration
        if (config < 0 || config > 8) return fail(QDEC_EINVAL, "tile gemv configuration must be 0..8");
        set_gemv_impl(0);
        set_gemv7_config(config);
        return QDEC_OK;
    }
    if (impl != 0 && impl != 2 && impl != 6) return fail(QDEC_EINVAL, "gemv kernel must be 0, 2, 6, 7, 8, 9 or 10");
    if (impl == 0) set_gemv7_config(0);
    if (config < 0 || config > 8) return fail(QDEC_EINVAL, "gemv configuration must be 0..8");
    set_gemv_impl(impl);
    set_gemv_v6_config(config);
    return QDEC_OK;
}

int qdec_selftest_wait(int which, int wait_ms) {
    if (which < 0 || which > 1 || wait_ms <= 0 || wait_ms > 10000)
        return fail(QDEC_EINVAL, "qdec_selftest_wait: which must be 0 or 1 and wait_ms in 1..10000");
    const unsigned long long ns = (unsigned long long)wait_ms * 1000000ull;
    const int rc = which == 0 ? selftest_exchange(ns) : selftest_gemv7_timeout(ns);
    if (rc == 0) return QDEC_OK;
    static const char *what[] = {"", "setting up", "the timed-out run did not complete as a kernel",
                                 "the wait did not report that it gave up", "the normal run afterwards failed",
                                 "the normal run afterwards reported an error", "the normal run afterwards gave wrong data",
                                 "the pushed lines are wrong"};
    return fail(QDEC_ECUDA, "qdec_selftest_wait(%s): %s", which == 0 ? "exchange poll" : "GEMV stage wait",
                rc > 0 && rc < 8 ? what[rc] : "?");
}

int qdec_repack_q6k(const void *src_dev, int rows, int cols, void *dst_dev, void *stream) {
    if (!src_dev || !dst_dev || rows < 0 || cols <= 0 || cols % 256)
        return fail(QDEC_EINVAL, "qdec_repack_q6k: bad argument (cols %d must be a multiple of 256)", cols);
    if (src_dev == dst_dev) return fail(QDEC_EINVAL, "qdec_repack_q6k: source and destination must differ");
    cudaError_t e = launch_repack_q6k((const uint8_t *)src_dev, (size_t)rows * (cols / 256), (uint8_t *)dst_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_repack_q6k");
}

int qdec_repack_tiles(int ggml_type, const void *src_dev, int rows, int cols, void *dst_dev, void *stream) {
    if (ggml_type != T_Q4_K && ggml_type != T_Q5_K && ggml_type != T_Q6_K && ggml_type != T_Q8_0 && ggml_type != T_Q4_0)
        return fail(QDEC_EINVAL, "qdec_repack_tiles: type %d has no tile layout", ggml_type);
    if (!src_dev || !dst_dev || rows < 0 || rows % 8 || cols <= 0 || cols % 256)
        return fail(QDEC_EINVAL, "qdec_repack_tiles: bad argument (rows %d must be a multiple of 8, cols %d of 256)", rows, cols);
    if (src_dev == dst_dev) return fail(QDEC_EINVAL, "qdec_repack_tiles: source and destination must differ");
    if (((uintptr_t)dst_dev & 15) != 0) return fail(QDEC_EINVAL, "qdec_repack_tiles: destination must be 16-byte aligned");
    const bool q80 = ggml_type == T_Q8_0 || ggml_type == T_Q4_0;
    if (q80 && cols % 256) return fail(QDEC_EINVAL, "qdec_repack_tiles: Q8_0/Q4_0 tiles hold a multiple of 256 columns");
    cudaError_t e = q80 ? launch_repack_q80_tiles(ggml_type, (const uint8_t *)src_dev, rows, cols, (uint8_t *)dst_dev, (cudaStream_t)stream)
                        : launch_repack_tiles(ggml_type, (const uint8_t *)src_dev, rows, cols, (uint8_t *)dst_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_repack_tiles");
}

int qdec_dequant_rows(int ggml_type, const void *w_dev, int rows, int cols, const int32_t *ids_dev, int n_ids,
                      float *out_dev, void *stream) {
    if (!supported_type(ggml_type) || ggml_type == T_Q6_K_SPLIT || tile_base_type(ggml_type) != ggml_type || cols <= 0 || cols % block_elems(ggml_type) || rows < 0 || n_ids < 0)
        return fail(QDEC_EINVAL, "qdec_dequant_rows: bad type %d or shape %d x %d", ggml_type, rows, cols);
    if (!w_dev || (!ids_dev && n_ids) || (!out_dev && n_ids)) return fail(QDEC_EINVAL, "qdec_dequant_rows: null pointer");
    const size_t rb = (size_t)(cols / block_elems(ggml_type)) * block_bytes(ggml_type);
    cudaError_t e = launch_dequant_rows(ggml_type, (const uint8_t *)w_dev, rb, cols, ids_dev, n_ids, out_dev, (cudaStream_t)stream);
    return e == cudaSuccess ? QDEC_OK : cuda_fail(e, "qdec_dequant_rows");
}

}  // extern "C"
