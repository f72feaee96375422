// Error plumbing shared by the C-ABI translation units.
#pragma once
#include <cstdarg>
#include <cstddef>
#include <cuda_runtime.h>

namespace qdec {
// Record a message for qdec_last_error() and return `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char *what);
void clear_error();
bool supported_type(int t);
int check_gemv_shape(int type, int rows, int cols, int ncols);
// Whether a K-quant GEMV on these weights reads the Q8_K device image (else the reference-layout activations).
bool uses_image(int type, const void *w_dev);
size_t image_bytes(int cols, int n_cols);
// Device scratch a matvec of n_cols columns needs for its quantised columns (0 for F32 weights).
size_t matvec_scratch_bytes(int type, const void *w_dev, int cols, int n_cols);
// Quantise x into `scratch` in the form the GEMV reads, then the GEMV; a status code.
int matvec_run(int type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols, float *y_dev, cudaStream_t s,
               void *scratch, const char *who);
}  // namespace qdec
