// Kernel and launcher declarations shared by the qdec translation units.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>
#include <stddef.h>

namespace qdec {

__global__ void q8k_quantize_kernel(const float* __restrict__ x, int n, int rows, uint8_t* __restrict__ out);
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
// `pdl`: launch as a programmatic dependent of the previous kernel in the stream; the GEMV then streams its
// first weight bytes before that kernel finishes, so the weights must not be written by it.
cudaError_t launch_gemv(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y,
                        cudaStream_t s, bool pdl = false);
// Bytes of one activation row of `cols` values in the form `type` consumes.
size_t act_row_bytes(int type, int cols);
int num_sms();
// Bulk-copy pipelined K-quant GEMV (gemv_tma.cu) for Q4_K / Q5_K when its staging fits shared memory.
bool tma_gemv_supported(int type, int cols, int ncols);
cudaError_t launch_gemv_tma(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y,
                            cudaStream_t s);
// Register-streamed K-quant GEMV (gemv_v5.cu) for Q4_K / Q5_K / Q6_K split.
bool v5_gemv_supported(int type, int cols, int ncols);
cudaError_t launch_gemv_v5(int type, const uint8_t* w, int rows, int cols, const void* act, int ncols, float* y,
                           cudaStream_t s, bool pdl);
// Tuning: GEMV implementation (0 = automatic, 2 = register path with super-block slots, 4 = bulk-copy,
// 5 = register-streamed) and the register-streamed kernel's lanes per thread (0, 1, 2) and depth (0, 4, 8).
void set_gemv_impl(int impl);
void set_gemv_v5_tuning(int gl, int depth);
// ggml Q6_K blocks -> the split layout the bulk-copy GEMV reads (nblocks blocks; dst holds the same bytes).
cudaError_t launch_repack_q6k(const uint8_t* src, size_t nblocks, uint8_t* dst, cudaStream_t s);
// Force the bulk-copy GEMV's lanes per row (1, 2, 4, 8; 0 = chosen from the row count).
void set_gemv_lanes_per_row(int lpr);
// The device error word set by bounded waits that gave up (0 = none); optionally cleared.
unsigned read_kernel_error(bool clear);

}  // namespace qdec
