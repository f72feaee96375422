/*
 * CPU ORACLE -- test infrastructure only, never part of the product path.
 *
 * A plain-C restatement of the CPU arithmetic of the reference engine `aqueduct`
 * (ManeeshJupalle/Qwen-3.8-in-Rust, crates/core).  Every function cites the reference
 * file:line it follows.  It is used by tests/ (as the checker), by __graft_entry__.smoke()
 * and by bench.py's cpu_baseline / --impl reference legs, and by nothing else.
 *
 * Build: oracle/Makefile (gcc -O2 -ffp-contract=off: no FMA contraction, as
 * crates/core/src/kernels/kdot.rs:18 requires "multiply then add").
 *
 * Transcendentals.  The reference calls Rust's f32::exp / f32::ln_1p, which lower to the
 * platform libm.  `oracle_set_libm(ORACLE_LIBM_GLIBC)` uses glibc expf/log1pf, i.e. what a
 * Linux build of the reference computes.  `ORACLE_LIBM_CR` (the default) evaluates them in
 * double and rounds once to f32 -- correctly rounded on every f32 input for exp (checked
 * exhaustively), and the same formula the CUDA kernels use, so oracle and GPU compare
 * bit for bit.  glibc's expf differs from correct rounding on 7.6e-5 of inputs in
 * (-104, 89) and log1pf on 0.47 % of positive inputs, each by one ulp.
 */
#ifndef QDEC_ORACLE_H
#define QDEC_ORACLE_H
#include <stdint.h>
#include <stddef.h>

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_LIBM_CR = 0, ORACLE_LIBM_GLIBC = 1 };
void oracle_set_libm(int mode);
int oracle_get_libm(void);
void oracle_set_threads(int n);

/* ggml type ids (GGUF tensor types), crates/core/src/gguf.rs GgmlType */
enum { OT_F32 = 0, OT_F16 = 1, OT_Q4_0 = 2, OT_Q8_0 = 8, OT_Q4_K = 12, OT_Q5_K = 13, OT_Q6_K = 14 };

float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);
float oracle_expf(float x);
float oracle_log1pf(float x);
float oracle_silu(float x);
float oracle_sigmoid(float x);
float oracle_softplus(float x);

/* block geometry: elements per block and bytes per block; 0 on an unknown type */
int oracle_block_layout(int type, int *block_elems, int *block_bytes);
size_t oracle_row_bytes(int type, int cols);

/* dequantisation (quant.rs:67-229); returns 0, or -1 on a size mismatch */
int oracle_dequantize(int type, const uint8_t *src, size_t src_len, float *dst, size_t n);

/* Q8_K activation rows in ggml block_q8_K layout: per 256 values f32 d, 256 x i8, 16 x i16 (292 B). */
void oracle_quantize_q8k(const float *x, int n, uint8_t *out);
/* Q8_0 activation rows in ggml block_q8_0 layout: per 32 values f16 d, 32 x i8 (34 B). */
void oracle_quantize_q8_0(const float *x, int n, uint8_t *out);

/* One weight row (ggml bytes) times one activation row.  K-quants take Q8_K, Q8_0/Q4_0 take Q8_0,
 * F32 takes f32. */
float oracle_dot(int type, const uint8_t *wrow, const void *act, int cols);

/* y[c*rows + r] = w[r] . x_c for c in 0..ncols (matvec.rs:364-369 layout).  `x` holds ncols activation
 * rows of `cols` f32 values; they are quantised here into the form `type` consumes (matvec.rs:147-160). */
void oracle_matmul_f32in(int type, const uint8_t *w, int rows, int cols, const float *x, int ncols, float *y);
/* Same, on pre-quantised activations (Q8_K / Q8_0 bytes, or f32 for F32 weights), `act_stride` bytes apart. */
void oracle_matmul_act(int type, const uint8_t *w, int rows, int cols, const void *act, size_t act_stride,
                       int ncols, float *y);

/* The matmuls run the AVX2 kernels (bit-identical to the scalar ones, blocked over up to 16 columns) when the CPU
 * has AVX2; oracle_set_simd(0) forces the scalar kernels, 1 the AVX2 ones, -1 back to detection. */
void oracle_set_simd(int on);

float oracle_reduce8(const float *l);
float oracle_sum_squares_8lane(const float *x, int n);
float oracle_inv_rms(const float *x, int n, float eps);
void oracle_rmsnorm(const float *x, const float *w, int n, float eps, float *y);
void oracle_rmsnorm_gated(const float *x, const float *gate, const float *w, int n, float eps, float *y);
void oracle_swiglu(const float *g, const float *u, int n, float *y);
void oracle_softmax(const float *x, int n, float *y);
void oracle_inv_freq(int rope_dim, float theta, float *out);
void oracle_cos_sin(uint32_t pos, const float *inv_freq, int half, float *cos, float *sin);
void oracle_apply_rope(float *x, int len, int head_dim, int rope_dim, const float *cos, const float *sin);
void oracle_conv1d_step(float *state, const float *w, int kernel, const float *x_new, int channels, float *out,
                        int act_silu);
void oracle_l2norm(float *x, int n, float eps);
float oracle_gate_g(float a, float dt_bias, float big_a);
float oracle_gate_beta(float b);
void oracle_deltanet_step(const float *q, const float *k, const float *v, int dk, int dv, float g, float beta,
                          float *s, float *out);
uint32_t oracle_argmax(const float *v, int n);
uint32_t oracle_crc32(const uint8_t *p, size_t n);

/* the sampler (sample.c, crates/core/src/sample.rs) */
typedef struct {
    float temperature;  /* <= 0: greedy */
    int top_k;          /* 0: off */
    float top_p, min_p;
    uint64_t seed;
} OSamplerCfg;
typedef struct oracle_sampler OSampler;
void oracle_rng_seed(uint64_t s_out[4], uint64_t seed);
uint64_t oracle_rng_next(uint64_t s[4]);
float oracle_rng_f32(uint64_t s[4]);
OSampler *oracle_sampler_new(const OSamplerCfg *cfg, int vocab);
void oracle_sampler_free(OSampler *s);
int oracle_sampler_greedy(const OSampler *s);
int oracle_sampler_process(OSampler *s, const float *logits, uint32_t *ids_out, float *probs_out);
uint32_t oracle_sampler_draw(OSampler *s);
uint32_t oracle_sampler_sample(OSampler *s, const float *logits);
int oracle_sampler_accept(OSampler *s, const float *target_logits, const float *q_dense, uint32_t d, uint32_t *tok_out);
void oracle_sampler_write_dense(const OSampler *s, float *out);


/* --- model level (model.c) --- */
/* the carried state of one layer of an oracle state: what = 0 DeltaNet S, 1 conv window, 2 / 3 K / V rows [0, pos);
 * returns the floats written (or needed, out NULL), 0 when the layer has no such state */
typedef struct oracle_state OState;
long oracle_state_get(OState *s, int layer, int what, float *out);

/* one layer on caller-held F32 weights (crates/core/tests/layers.rs): weight slots and kinds */
enum { OW_ATTN_NORM, OW_POST_NORM, OW_QKV, OW_GATE_Z, OW_ALPHA, OW_BETA, OW_SSM_A, OW_DT_BIAS, OW_CONV, OW_SSM_NORM,
       OW_SSM_OUT, OW_Q, OW_K, OW_V, OW_O, OW_Q_NORM, OW_K_NORM, OW_FFN_GATE, OW_FFN_UP, OW_FFN_DOWN, OW_COUNT };
enum { OL_DELTANET = 0, OL_ATTENTION = 1, OL_MLP = 2, OL_DECODER_DELTANET = 3, OL_DECODER_ATTENTION = 4 };
int oracle_layer_f32(const int *dims, const float *fdims, const float *const *w, int kind, const float *x, int t,
                     int pos0, float *S, float *conv, float *K, float *V, float *y);

#ifdef __cplusplus
}
#endif
#endif
