// Error plumbing shared by the C-ABI translation units.
#pragma once
#include <cstdarg>
#include <cuda_runtime.h>

namespace qdec {
// Record a message for qdec_last_error() and return `code`.
int fail(int code, const char *fmt, ...) __attribute__((format(printf, 2, 3)));
int cuda_fail(cudaError_t e, const char *what);
void clear_error();
bool supported_type(int t);
int check_gemv_shape(int type, int rows, int cols, int ncols);
}  // namespace qdec
