// Kernel and launcher declarations shared by the qdec translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qdec {

__global__ void q8k_quantize_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ out);
__global__ void q8k_image_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ img);
__global__ void q8k_raw_to_image_kernel(const uint8_t* __restrict__ raw, long long nblocks, uint8_t* __restrict__ img);
__global__ void q80_image_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ img);
__global__ void q80_raw_to_image_kernel(const uint8_t* __restrict__ raw, int nb, int rows, uint8_t* __restrict__ img);
__global__ void q8_0_quantize_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ out);
__global__ void dequant_rows_kernel(int type, const uint8_t* __restrict__ w, size_t row_bytes, int n,
                                    const int32_t* __restrict__ ids, int nids, float* __restrict__ out);

// Host launchers (return cudaError_t of the launch).
cudaError_t launch_quantize_q8k(const float* x, int n, int rows, uint8_t* out, cudaStream_t s);
cudaError_t launch_quantize_q8_0(const float* x, int n, int rows, uint8_t* out, cudaStream_t s);
cudaError_t launch_dequant_rows(int type, const uint8_t* w, size_t row_bytes, int n, const int32_t* ids, int nids,
                                float* out, cudaStream_t s);

// y[c * rows + r] = W[r] . act_c for c in [0, ncols); act in the form the weight type consumes:
// block_q8_K rows (K-quants), block_q8_0 rows (Q8_0, Q4_0) or f32 rows (F32), `ncols` rows back to back.
cudaError_t launch_gemv(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y,
                        cudaStream_t s);
// F32 weights: rows of w_a then rows of w_b (w_b may be null) against the same f32 columns, y_a / y_b laid out
// [column][row]; cols <= 16384.
// early: x was written two or more kernels back (not by the kernel right before), so the product may run
// before griddepcontrol.wait, alongside its predecessor (launched as a programmatic dependent)
cudaError_t launch_gemv_f32_pair(const float* w_a, int rows_a, float* y_a, const float* w_b, int rows_b, float* y_b, int cols,
                                 const float* x, int ncols, cudaStream_t s, bool early = false);
// Bytes of one activation row of `cols` values in the form `type` consumes (reference layouts).
size_t act_row_bytes(int type, int cols);
int num_sms();

// The engine's Q8_K device image (common.cuh): quantise f32 rows into it, or rearrange block_q8_K rows.
cudaError_t launch_quantize_q8k_image(const float* x, int n, int rows, uint8_t* img, cudaStream_t s);
cudaError_t launch_q8k_raw_to_image(const uint8_t* raw, long long nblocks, uint8_t* img, cudaStream_t s);
// K-quant GEMV over the Q8_K device image (gemv_v6.cu): Q4_K, Q5_K and Q6_K in the split layout, weights
// 16-byte aligned.  `img` holds `ncols` rows of cols/256 image blocks back to back.
// `pdl`: launch as a programmatic dependent of the previous kernel in the stream; the GEMV then streams its
// first weight bytes before that kernel finishes, so the weights must not be written by it.
bool v6_gemv_supported(int type);
cudaError_t launch_gemv_img(int type, const uint8_t* w, int rows, int cols, const void* img, int ncols, float* y,
                            cudaStream_t s, bool pdl);
// Two K-quant tile matrices of one type reading the same image columns (e.g. ffn_gate and ffn_up) in one
// launch: y_a = W_a x, y_b = W_b x; rows % 8 == 0.
cudaError_t launch_gemv_img_pair(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                                 int cols, const void* img, int ncols, cudaStream_t s, bool pdl);
// Tuning: the K-quant GEMV implementation (0 = automatic, 2 = the raw-Q8_K register path, 6 = the image kernel)
// and the image kernel's configuration (0 = automatic, 1..8).
void set_gemv_impl(int impl);
int gemv_impl();
void set_gemv_v6_config(int cfg);
// ggml Q6_K blocks -> the split layout the image kernel reads (nblocks blocks; dst holds the same bytes).
cudaError_t launch_repack_q6k(const uint8_t* src, size_t nblocks, uint8_t* dst, cudaStream_t s);
// ggml Q4_K / Q5_K / Q6_K rows (rows % 8 == 0) -> the tile layout (gemv_v6.cu); dst holds the same bytes.
cudaError_t launch_repack_tiles(int ggml_type, const uint8_t* src, int rows, int cols, uint8_t* dst, cudaStream_t s);
// Q8_0 / Q4_0: the engine's Q8_0 row image (common.cuh), the tile layout, and the GEMV over both (gemv_q80.cu).
cudaError_t launch_quantize_q80_image(const float* x, int n, int rows, uint8_t* img, cudaStream_t s);
cudaError_t launch_q80_raw_to_image(const uint8_t* raw, int n, int rows, uint8_t* img, cudaStream_t s);
cudaError_t launch_repack_q80_tiles(int ggml_type, const uint8_t* src, int rows, int cols, uint8_t* dst, cudaStream_t s);
// Tuning: -1 = automatic, 0 = one warp per tile, 1 = the group range split over 4 warps.
void set_q80_split(int mode);
cudaError_t launch_gemv_q80_img(int type, const uint8_t* w, int rows, int cols, const void* img, int ncols, float* y,
                                cudaStream_t s, bool pdl);
// The decode GEMV of K-quant tile matrices (gemv7.cu): one matrix, or two reading the same image columns (w_b
// non-null, e.g. ffn_gate and ffn_up), against `ncols` Q8_K image columns (groups of at most 4 per launch).
// Bit-exact with crates/core/src/kernels/kdot.rs.  rows % 8 == 0, cols % 256 == 0.
bool gemv7_supported(int type);
void set_gemv7_config(int cfg);  // 0 = automatic by shape; 1..8 a fixed configuration (tests, sweeps)
void set_gemv7_mma_min_cols(int n);  // Q4_K column groups of at least n take the warp-MMA form (0 = never)
cudaError_t launch_gemv7(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                         int cols, const void* img, int ncols, cudaStream_t s, bool pdl);
// The MLP's gate and up tile matrices (rows x cols each, rows % 256 == 0) against the image columns, fused with
// h = silu(gate) * up (written to h_out, [column][row]) and its quantisation into the Q8_K image img_out
// ([column][rows / 256 blocks]); blk_cnt: rows / 256 zeroed counters, left zeroed.
cudaError_t launch_gemv7_swiglu(int type, const uint8_t* w_gate, const uint8_t* w_up, int rows, int cols, const void* img,
                                int ncols, float* h_out, uint8_t* img_out, unsigned* blk_cnt, cudaStream_t s, bool pdl);
unsigned read_gemv7_error(bool clear);  // the error word of gemv7.cu's bounded waits (0 = none)
int selftest_gemv7_timeout(unsigned long long wait_ns);  // failure-handling self-test of the stage wait (0 = as designed)
// The device error word set by bounded waits that gave up (0 = none); optionally cleared.
unsigned read_kernel_error(bool clear);
// The same two error words (prefill GEMM, tile GEMV) copied into pinned host memory in stream order, so that the
// stream's synchronisation also delivers them; read_kernel_error(true) clears them after one was set.
cudaError_t enqueue_kernel_error_read(unsigned* host2, cudaStream_t s);
cudaError_t enqueue_gemv7_error_read(unsigned* host_dst, cudaStream_t s);
cudaError_t enqueue_gemm_tc_error_read(unsigned* host_dst, cudaStream_t s);
// Prompt-prefill GEMM on the tensor cores (gemm_tc.cu): K-quant tile matrices (one, or two reading the same
// image columns) against `ncols` Q8_K image columns, bit-exact with the GEMV.  launch_gemv_img and
// launch_gemv_img_pair route there when gemm_tc_applies(type, ncols): tile types and ncols >= the minimum
// column count (16 by default; 0 disables the path).
bool gemm_tc_applies(int type, int ncols);
void set_gemm_tc_min_cols(int n);
int gemm_tc_min_cols();
cudaError_t launch_gemm_tc(int type, const uint8_t* w_a, int rows_a, float* y_a, const uint8_t* w_b, int rows_b, float* y_b,
                           int cols, const void* img, int ncols, cudaStream_t s, bool pdl);
unsigned read_gemm_tc_error(bool clear);

}  // namespace qdec
