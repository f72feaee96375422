/*
 * qdec -- a B200 (sm_100a) decode engine for Qwen3.8-class hybrid models stored as K-quant GGUF files.
 *
 * C ABI.  Every function returns an int status: QDEC_OK (0) or a negative QDEC_E* code; qdec_last_error()
 * returns the message of the calling thread's last failure.  No C++ exception crosses this boundary.
 * Pointers named *_dev are device pointers; `stream` is a cudaStream_t (NULL = the legacy default stream).
 *
 * The reference engine (`aqueduct`, ManeeshJupalle/Qwen-3.8-in-Rust) is a Rust workspace with no FFI layer;
 * each entry point below names the crate API it replaces (paths relative to that project's root).
 */
#ifndef QDEC_H
#define QDEC_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define QDEC_OK 0
#define QDEC_EINVAL (-1)   /* bad argument: shape, type, size (the reference's assert! panics) */
#define QDEC_ECUDA (-2)    /* a CUDA call failed */
#define QDEC_ENOMEM (-3)   /* device or host allocation failed */
#define QDEC_EIO (-4)      /* file I/O failed */
#define QDEC_EFORMAT (-5)  /* malformed GGUF or config contract violated (GgufError / ConfigError) */
#define QDEC_ESTATE (-6)   /* call out of order (e.g. spec_round before spec_prefill) */
#define QDEC_ETIMEOUT (-7) /* a device-side wait gave up; the kernel returned an error word */

/* ggml tensor types accepted by the kernels (GGUF type ids; crates/core/src/gguf.rs GgmlType) */
#define QDEC_TYPE_F32 0
#define QDEC_TYPE_Q4_0 2
#define QDEC_TYPE_Q8_0 8
#define QDEC_TYPE_Q4_K 12
#define QDEC_TYPE_Q5_K 13
#define QDEC_TYPE_Q6_K 14

/* Library version string, e.g. "qdec 0.1.0 sm_100a". */
const char *qdec_version(void);
/* Message of the calling thread's last failed call ("" if none). */
const char *qdec_last_error(void);

/* ------------------------------------------------------------------------------------- kernel level */

/* Quantise `rows` rows of `n` f32 values (n % 256 == 0) into ggml block_q8_K rows
 * (per 256 values: f32 d, 256 x i8, 16 x i16 bsums; 292 bytes), bit-exact with the reference.
 * Replaces Q8KRow::quantize_into (crates/core/src/kernels/q8k.rs:51, :76-114). */
int qdec_quantize_q8k(const float *x_dev, int n, int rows, void *q8k_dev, void *stream);

/* Quantise into ggml block_q8_0 rows (per 32 values: f16 d, 32 x i8; 34 bytes), n % 32 == 0.
 * Replaces Q8Row::quantize_into (crates/core/src/kernels/q8.rs:65-103). */
int qdec_quantize_q8_0(const float *x_dev, int n, int rows, void *q8_dev, void *stream);

/* Size in bytes of one activation row of `cols` values in the form weights of `ggml_type` consume
 * (Q8_K for K-quants, Q8_0 for Q8_0/Q4_0, f32 for F32); 0 for an unsupported type.
 * Mirrors act_kind (crates/core/src/kernels/matvec.rs:147-160). */
size_t qdec_act_row_bytes(int ggml_type, int cols);

/* y[c * rows + r] = W[r] . act_c for c in [0, n_cols): the dequant-GEMV over pre-quantised activations.
 * `w_dev` is rows x cols in ggml row layout; `act_dev` holds n_cols activation rows of
 * qdec_act_row_bytes(type, cols) bytes each.  Every weight byte is read once per 4 columns.  Bit-exact with
 * matmul_fn / dot_q8k_t (crates/core/src/kernels/matvec.rs:377, :511-539; kdot.rs:314). */
int qdec_gemv(int ggml_type, const void *w_dev, int rows, int cols, const void *act_dev, int n_cols, float *y_dev,
              void *stream);

/* As qdec_gemv, from f32 activation rows (`x_dev`, n_cols x cols): each column is quantised into the form
 * the weight type consumes, then multiplied.  The quantised rows live in a device buffer the library owns
 * (one per device, grown on demand).  Replaces matvec_f32_in / matmul over ActVec
 * (crates/core/src/kernels/matvec.rs:541-545, :369-371). */
int qdec_matvec(int ggml_type, const void *w_dev, int rows, int cols, const float *x_dev, int n_cols, float *y_dev,
                void *stream);

/* out[i * cols + e] = dequantised element e of row ids[i] of `w_dev` (ids on the device, n_ids of them):
 * the embedding gather.  Replaces Model::embed_token_into (crates/core/src/model.rs:364-368) and
 * dequantize_into (crates/core/src/quant.rs:229). */
int qdec_dequant_rows(int ggml_type, const void *w_dev, int rows, int cols, const int32_t *ids_dev, int n_ids,
                      float *out_dev, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* QDEC_H */
