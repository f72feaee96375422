/*
 * CPU ORACLE (test infrastructure; see oracle.h).  Kernel-level restatement of the reference's scalar
 * paths.  Paths are relative to the reference project root.
 */
#include "oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static int g_libm = ORACLE_LIBM_CR;
static int g_threads = 0;

void oracle_set_libm(int mode) { g_libm = mode; }
int oracle_get_libm(void) { return g_libm; }
void oracle_set_threads(int n) { g_threads = n; }

/* ---------------------------------------------------------------- f16 (crates/core/src/quant.rs:34-37) */

/* IEEE binary16 -> f32, exact (the `half` crate's to_f32). */
float oracle_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t exp = (h >> 10) & 0x1f;
    uint32_t man = h & 0x3ff;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else { /* subnormal: renormalise */
            int e = -1;
            do {
                man <<= 1;
                e++;
            } while ((man & 0x400) == 0);
            man &= 0x3ff;
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | (man << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    memcpy(&f, &bits, 4);
    return f;
}

/* f32 -> binary16, round to nearest even (`half::f16::from_f32`, used by kernels/q8.rs:97). */
uint16_t oracle_f32_to_f16(float f) {
    uint32_t x;
    memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t exp = (x >> 23) & 0xff;
    uint32_t man = x & 0x7fffff;
    if (exp == 0xff) return (uint16_t)(sign | 0x7c00u | (man ? (0x200u | (man >> 13)) : 0));
    int32_t e = (int32_t)exp - 127 + 15;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        man |= 0x800000u;
        uint32_t shift = (uint32_t)(14 - e);
        uint32_t half_m = man >> shift;
        uint32_t rem = man & ((1u << shift) - 1);
        uint32_t mid = 1u << (shift - 1);
        if (rem > mid || (rem == mid && (half_m & 1))) half_m++;
        return (uint16_t)(sign | half_m);
    }
    uint32_t half_m = man >> 13;
    uint32_t rem = man & 0x1fff;
    uint32_t out = sign | ((uint32_t)e << 10) | half_m;
    if (rem > 0x1000 || (rem == 0x1000 && (half_m & 1))) out++; /* may carry into the exponent: still RNE */
    return (uint16_t)out;
}

/* ------------------------------------------------------- activations (crates/core/src/kernels/act.rs:7-40) */

float oracle_expf(float x) { return g_libm == ORACLE_LIBM_GLIBC ? expf(x) : (float)exp((double)x); }
float oracle_log1pf(float x) { return g_libm == ORACLE_LIBM_GLIBC ? log1pf(x) : (float)log1p((double)x); }

/* act.rs:10: x / (1 + exp(-x)) */
float oracle_silu(float x) { return x / (1.0f + oracle_expf(-x)); }
/* act.rs:15 */
float oracle_sigmoid(float x) { return 1.0f / (1.0f + oracle_expf(-x)); }
/* act.rs:33-40: threshold 20 */
float oracle_softplus(float x) { return x > 20.0f ? x : oracle_log1pf(oracle_expf(x)); }

/* act.rs:24 */
void oracle_swiglu(const float *g, const float *u, int n, float *y) {
    for (int i = 0; i < n; i++) y[i] = oracle_silu(g[i]) * u[i];
}

/* ------------------------------------------------------------------------ block layouts (quant.rs:20-29) */

int oracle_block_layout(int type, int *be, int *bb) {
    switch (type) {
    case OT_F32: *be = 1; *bb = 4; return 1;
    case OT_Q4_0: *be = 32; *bb = 18; return 1;
    case OT_Q8_0: *be = 32; *bb = 34; return 1;
    case OT_Q4_K: *be = 256; *bb = 144; return 1;
    case OT_Q5_K: *be = 256; *bb = 176; return 1;
    case OT_Q6_K: *be = 256; *bb = 210; return 1;
    default: return 0;
    }
}

size_t oracle_row_bytes(int type, int cols) {
    int be, bb;
    if (!oracle_block_layout(type, &be, &bb)) return 0;
    return (size_t)(cols / be) * (size_t)bb;
}

static inline float f16_at(const uint8_t *b, int off) {
    return oracle_f16_to_f32((uint16_t)(b[off] | (b[off + 1] << 8)));
}

/* quant.rs:45-51 (ggml get_scale_min_k4) */
static inline void scale_min_k4(int j, const uint8_t *q, int *sc, int *m) {
    if (j < 4) {
        *sc = q[j] & 63;
        *m = q[j + 4] & 63;
    } else {
        *sc = (q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4);
        *m = (q[j + 4] >> 4) | ((q[j] >> 6) << 4);
    }
}

/* ------------------------------------------------------------------------ dequant (quant.rs:67-229) */

static void dq_q4_0(const uint8_t *src, size_t nb, float *y) { /* quant.rs:67-82 */
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * 18;
        float d = f16_at(b, 0);
        for (int j = 0; j < 16; j++) {
            int x0 = (b[2 + j] & 0x0F) - 8, x1 = (b[2 + j] >> 4) - 8;
            y[i * 32 + j] = (float)x0 * d;
            y[i * 32 + j + 16] = (float)x1 * d;
        }
    }
}

static void dq_q8_0(const uint8_t *src, size_t nb, float *y) { /* quant.rs:85-96 */
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * 34;
        float d = f16_at(b, 0);
        for (int j = 0; j < 32; j++) y[i * 32 + j] = (float)(int8_t)b[2 + j] * d;
    }
}

static void dq_q4_k(const uint8_t *src, size_t nb, float *dst) { /* quant.rs:102-133 */
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * 144;
        float d = f16_at(b, 0), mn = f16_at(b, 2);
        const uint8_t *scales = b + 4, *qs = b + 16;
        float *y = dst + i * 256;
        for (int g = 0; g < 4; g++) {
            int sc, m;
            scale_min_k4(2 * g, scales, &sc, &m);
            float d1 = d * (float)sc, m1 = mn * (float)m;
            scale_min_k4(2 * g + 1, scales, &sc, &m);
            float d2 = d * (float)sc, m2 = mn * (float)m;
            for (int l = 0; l < 32; l++) y[g * 64 + l] = d1 * (float)(qs[g * 32 + l] & 0xF) - m1;
            for (int l = 0; l < 32; l++) y[g * 64 + 32 + l] = d2 * (float)(qs[g * 32 + l] >> 4) - m2;
        }
    }
}

static void dq_q5_k(const uint8_t *src, size_t nb, float *dst) { /* quant.rs:137-175 */
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * 176;
        float d = f16_at(b, 0), mn = f16_at(b, 2);
        const uint8_t *scales = b + 4, *qh = b + 16, *ql = b + 48;
        float *y = dst + i * 256;
        for (int g = 0; g < 4; g++) {
            int sc, m;
            scale_min_k4(2 * g, scales, &sc, &m);
            float d1 = d * (float)sc, m1 = mn * (float)m;
            scale_min_k4(2 * g + 1, scales, &sc, &m);
            float d2 = d * (float)sc, m2 = mn * (float)m;
            uint8_t u1 = (uint8_t)(1u << (2 * g)), u2 = (uint8_t)(2u << (2 * g));
            for (int l = 0; l < 32; l++)
                y[g * 64 + l] = d1 * (float)((ql[g * 32 + l] & 0xF) + ((qh[l] & u1) ? 16 : 0)) - m1;
            for (int l = 0; l < 32; l++)
                y[g * 64 + 32 + l] = d2 * (float)((ql[g * 32 + l] >> 4) + ((qh[l] & u2) ? 16 : 0)) - m2;
        }
    }
}

static void dq_q6_k(const uint8_t *src, size_t nb, float *dst) { /* quant.rs:182-210 */
    for (size_t i = 0; i < nb; i++) {
        const uint8_t *b = src + i * 210;
        float d = f16_at(b, 208);
        float *yb = dst + i * 256;
        for (int half = 0; half < 2; half++) {
            const uint8_t *ql = b + half * 64, *qh = b + 128 + half * 32;
            const int8_t *sc = (const int8_t *)(b + 192 + half * 8);
            float *y = yb + half * 128;
            for (int l = 0; l < 32; l++) {
                int is = l / 16;
                int q1 = ((ql[l] & 0xF) | ((qh[l] & 3) << 4)) - 32;
                int q2 = ((ql[l + 32] & 0xF) | (((qh[l] >> 2) & 3) << 4)) - 32;
                int q3 = ((ql[l] >> 4) | (((qh[l] >> 4) & 3) << 4)) - 32;
                int q4 = ((ql[l + 32] >> 4) | (((qh[l] >> 6) & 3) << 4)) - 32;
                y[l] = d * (float)sc[is] * (float)q1;
                y[l + 32] = d * (float)sc[is + 2] * (float)q2;
                y[l + 64] = d * (float)sc[is + 4] * (float)q3;
                y[l + 96] = d * (float)sc[is + 6] * (float)q4;
            }
        }
    }
}

int oracle_dequantize(int type, const uint8_t *src, size_t src_len, float *dst, size_t n) {
    int be, bb;
    if (!oracle_block_layout(type, &be, &bb)) return -1;
    if (n % (size_t)be) return -1;
    size_t nb = n / (size_t)be;
    if (src_len != nb * (size_t)bb) return -1;
    switch (type) {
    case OT_F32: memcpy(dst, src, n * 4); break; /* quant.rs:213-219 (little-endian host) */
    case OT_Q4_0: dq_q4_0(src, nb, dst); break;
    case OT_Q8_0: dq_q8_0(src, nb, dst); break;
    case OT_Q4_K: dq_q4_k(src, nb, dst); break;
    case OT_Q5_K: dq_q5_k(src, nb, dst); break;
    case OT_Q6_K: dq_q6_k(src, nb, dst); break;
    default: return -1;
    }
    return 0;
}

/* ------------------------------------------------------ Q8_K quantiser (crates/core/src/kernels/q8k.rs:76-114) */

void oracle_quantize_q8k(const float *x, int n, uint8_t *out) {
    int nb = n / 256;
    for (int b = 0; b < nb; b++) {
        const float *blk = x + (size_t)b * 256;
        uint8_t *o = out + (size_t)b * 292;
        float amax = 0.0f, mx = 0.0f;
        for (int i = 0; i < 256; i++) { /* strict > scan: the first max wins (q8k.rs:88-95) */
            float a = fabsf(blk[i]);
            if (a > amax) {
                amax = a;
                mx = blk[i];
            }
        }
        if (amax == 0.0f) {
            memset(o, 0, 292);
            continue;
        }
        float iscale = -127.0f / mx;
        int8_t q[256];
        for (int i = 0; i < 256; i++) {
            float v = rintf(iscale * blk[i]); /* round_ties_even; then `as i32` (saturating) */
            int qi = (v >= 2147483647.0f) ? 2147483647 : (v <= -2147483648.0f ? (int)-2147483647 - 1 : (int)v);
            if (qi > 127) qi = 127;
            q[i] = (int8_t)qi;
        }
        float d = 1.0f / iscale;
        memcpy(o, &d, 4);
        memcpy(o + 4, q, 256);
        for (int g = 0; g < 16; g++) {
            int s = 0;
            for (int i = 0; i < 16; i++) s += q[g * 16 + i];
            int16_t s16 = (int16_t)s;
            memcpy(o + 260 + 2 * g, &s16, 2);
        }
    }
}

/* ------------------------------------------------------ Q8_0 quantiser (crates/core/src/kernels/q8.rs:81-103) */

void oracle_quantize_q8_0(const float *x, int n, uint8_t *out) {
    int nb = n / 32;
    for (int b = 0; b < nb; b++) {
        const float *blk = x + (size_t)b * 32;
        uint8_t *o = out + (size_t)b * 34;
        float amax = 0.0f;
        for (int i = 0; i < 32; i++) {
            float a = fabsf(blk[i]);
            if (a > amax) amax = a;
        }
        float dd = amax / 127.0f;
        float id = dd != 0.0f ? 1.0f / dd : 0.0f;
        uint16_t h = oracle_f32_to_f16(dd);
        o[0] = (uint8_t)(h & 0xff);
        o[1] = (uint8_t)(h >> 8);
        for (int i = 0; i < 32; i++) {
            float v = roundf(blk[i] * id); /* round half away from zero, then `as i8` (saturating) */
            int qi = v > 127.0f ? 127 : (v < -128.0f ? -128 : (int)v);
            o[2 + i] = (uint8_t)(int8_t)qi;
        }
    }
}

/* --------------------------------------------------------------------------- reductions (rmsnorm.rs:69-76) */

float oracle_reduce8(const float *l) { return ((l[0] + l[4]) + (l[2] + l[6])) + ((l[1] + l[5]) + (l[3] + l[7])); }
static inline float reduce4(const float *m) { return (m[0] + m[2]) + (m[1] + m[3]); } /* kdot.rs:31-34 */

/* ------------------------------------------------- K-quant x Q8_K dots (crates/core/src/kernels/kdot.rs:37-141) */

static inline float q8k_d(const uint8_t *blk) {
    float d;
    memcpy(&d, blk, 4);
    return d;
}
static inline int16_t q8k_bsum(const uint8_t *blk, int g) {
    int16_t s;
    memcpy(&s, blk + 260 + 2 * g, 2);
    return s;
}

/* kdot.rs:37-76 with the Q4_K (:79-84) or Q5_K (:87-95) code extraction */
static float dot_q45_k(const uint8_t *w, const uint8_t *x, int nb, int q5) {
    float acc[8] = {0}, accm[4] = {0};
    int bbytes = q5 ? 176 : 144;
    for (int sb = 0; sb < nb; sb++) {
        const uint8_t *wb = w + (size_t)sb * bbytes;
        const uint8_t *xb = x + (size_t)sb * 292;
        float dx = q8k_d(xb);
        float d = dx * f16_at(wb, 0);
        float dmin = -dx * f16_at(wb, 2);
        const uint8_t *scales = wb + 4;
        const int8_t *xq = (const int8_t *)(xb + 4);
        int sc[8], mn[8], q8s[8];
        for (int s = 0; s < 8; s++) {
            scale_min_k4(s, scales, &sc[s], &mn[s]);
            q8s[s] = (int16_t)(q8k_bsum(xb, 2 * s) + q8k_bsum(xb, 2 * s + 1)); /* q8k.rs:185-193 */
        }
        for (int i = 0; i < 4; i++) {
            int prod = mn[2 * i] * q8s[2 * i] + mn[2 * i + 1] * q8s[2 * i + 1];
            accm[i] += dmin * (float)prod;
        }
        int sumi[8] = {0};
        for (int s = 0; s < 8; s++) {
            for (int j = 0; j < 32; j++) {
                int qw;
                if (!q5) {
                    uint8_t q = wb[16 + (s / 2) * 32 + j];
                    qw = (s % 2 == 0) ? (q & 0xF) : (q >> 4);
                } else {
                    uint8_t q = wb[48 + (s / 2) * 32 + j];
                    qw = ((s % 2 == 0) ? (q & 0xF) : (q >> 4)) + ((wb[16 + j] & (1u << s)) ? 16 : 0);
                }
                sumi[j / 4] += sc[s] * qw * xq[s * 32 + j];
            }
        }
        for (int i = 0; i < 8; i++) acc[i] += d * (float)sumi[i];
    }
    return oracle_reduce8(acc) + reduce4(accm);
}

/* kdot.rs:97-141 */
static float dot_q6_k(const uint8_t *w, const uint8_t *x, int nb) {
    float acc[8] = {0};
    for (int sb = 0; sb < nb; sb++) {
        const uint8_t *wb = w + (size_t)sb * 210;
        const uint8_t *xb = x + (size_t)sb * 292;
        const uint8_t *ql_all = wb, *qh_all = wb + 128, *sc_all = wb + 192;
        float d = q8k_d(xb) * f16_at(wb, 208);
        const int8_t *xq = (const int8_t *)(xb + 4);
        int sumi[8] = {0};
        for (int half = 0; half < 2; half++) {
            const uint8_t *ql = ql_all + half * 64, *qh = qh_all + half * 32, *sc = sc_all + half * 8;
            for (int k = 0; k < 4; k++) {
                const int8_t *xs = xq + half * 128 + k * 32;
                for (int l = 0; l < 32; l++) {
                    int lo;
                    switch (k) {
                    case 0: lo = ql[l] & 0xF; break;
                    case 1: lo = ql[l + 32] & 0xF; break;
                    case 2: lo = ql[l] >> 4; break;
                    default: lo = ql[l + 32] >> 4; break;
                    }
                    int hi = (qh[l] >> (2 * k)) & 3;
                    int qw = lo | (hi << 4);
                    int scale = (int8_t)sc[2 * k + l / 16];
                    sumi[l / 4] += scale * qw * xs[l];
                }
            }
        }
        for (int i = 0; i < 8; i++) {
            int s0 = (int8_t)sc_all[2 * i], s1 = (int8_t)sc_all[2 * i + 1];
            sumi[i] -= 32 * (q8k_bsum(xb, 2 * i) * s0 + q8k_bsum(xb, 2 * i + 1) * s1);
        }
        for (int i = 0; i < 8; i++) acc[i] += d * (float)sumi[i];
    }
    return oracle_reduce8(acc);
}

/* ---------------------------------------------- Q8_0 / Q4_0 / F32 dots (crates/core/src/kernels/dot.rs:29-64, 180-198) */

static float dot_q8_0_q8(const uint8_t *w, const uint8_t *x, int nb) { /* dot.rs:29-43 */
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *wb = w + (size_t)b * 34, *xb = x + (size_t)b * 34;
        float dw = f16_at(wb, 0);
        int isum = 0;
        for (int j = 0; j < 32; j++) isum += (int8_t)wb[2 + j] * (int8_t)xb[2 + j];
        acc += (dw * f16_at(xb, 0)) * (float)isum;
    }
    return acc;
}

static float dot_q4_0_q8(const uint8_t *w, const uint8_t *x, int nb) { /* dot.rs:46-63 */
    float acc = 0.0f;
    for (int b = 0; b < nb; b++) {
        const uint8_t *wb = w + (size_t)b * 18, *xb = x + (size_t)b * 34;
        float dw = f16_at(wb, 0);
        const int8_t *xq = (const int8_t *)(xb + 2);
        int isum = 0;
        for (int j = 0; j < 16; j++) {
            int lo = (wb[2 + j] & 0x0F) - 8, hi = (wb[2 + j] >> 4) - 8;
            isum += lo * xq[j] + hi * xq[j + 16];
        }
        acc += (dw * f16_at(xb, 0)) * (float)isum;
    }
    return acc;
}

/* dot.rs:180-198: 32-element block partials left to right, the tail as one more partial */
static float dot_f32(const float *w, const float *x, int n) {
    float acc = 0.0f;
    int i = 0;
    while (i + 32 <= n) {
        float part = 0.0f;
        for (int j = 0; j < 32; j++) part += w[i + j] * x[i + j];
        acc += part;
        i += 32;
    }
    float part = 0.0f;
    while (i < n) {
        part += w[i] * x[i];
        i++;
    }
    return acc + part;
}

/* matvec.rs:282-292 (one_row) */
float oracle_dot(int type, const uint8_t *wrow, const void *act, int cols) {
    switch (type) {
    case OT_Q4_K: return dot_q45_k(wrow, (const uint8_t *)act, cols / 256, 0);
    case OT_Q5_K: return dot_q45_k(wrow, (const uint8_t *)act, cols / 256, 1);
    case OT_Q6_K: return dot_q6_k(wrow, (const uint8_t *)act, cols / 256);
    case OT_Q8_0: return dot_q8_0_q8(wrow, (const uint8_t *)act, cols / 32);
    case OT_Q4_0: return dot_q4_0_q8(wrow, (const uint8_t *)act, cols / 32);
    case OT_F32: return dot_f32((const float *)(const void *)wrow, (const float *)act, cols);
    default: abort();
    }
}

static size_t act_bytes(int type, int cols) {
    switch (type) {
    case OT_Q4_K: case OT_Q5_K: case OT_Q6_K: return (size_t)(cols / 256) * 292;
    case OT_Q8_0: case OT_Q4_0: return (size_t)(cols / 32) * 34;
    default: return (size_t)cols * 4;
    }
}

/* matvec.rs:377-385, 511-539: every row computed once per column with the single-row arithmetic */
int oracle_matmul_fast(int type, const uint8_t *w, int rows, int cols, const void *act, size_t act_stride, int ncols, float *y);

void oracle_matmul_act(int type, const uint8_t *w, int rows, int cols, const void *act, size_t act_stride, int ncols,
                       float *y) {
    if (oracle_matmul_fast(type, w, rows, cols, act, act_stride, ncols, y)) return;
    size_t rb = oracle_row_bytes(type, cols);
#ifdef _OPENMP
    int nt = g_threads > 0 ? g_threads : omp_get_max_threads();
#pragma omp parallel for schedule(static) num_threads(nt)
#endif
    for (int r = 0; r < rows; r++) {
        for (int c = 0; c < ncols; c++)
            y[(size_t)c * rows + r] = oracle_dot(type, w + (size_t)r * rb, (const uint8_t *)act + (size_t)c * act_stride, cols);
    }
}

void oracle_matmul_f32in(int type, const uint8_t *w, int rows, int cols, const float *x, int ncols, float *y) {
    size_t ab = act_bytes(type, cols);
    uint8_t *act = (uint8_t *)malloc(ab * (size_t)ncols);
    for (int c = 0; c < ncols; c++) {
        const float *xc = x + (size_t)c * cols;
        uint8_t *a = act + (size_t)c * ab;
        switch (type) {
        case OT_Q4_K: case OT_Q5_K: case OT_Q6_K: oracle_quantize_q8k(xc, cols, a); break;
        case OT_Q8_0: case OT_Q4_0: oracle_quantize_q8_0(xc, cols, a); break;
        default: memcpy(a, xc, (size_t)cols * 4); break;
        }
    }
    oracle_matmul_act(type, w, rows, cols, act, ab, ncols, y);
    free(act);
}

/* ------------------------------------------------------------------------ RMSNorm (rmsnorm.rs:14-76) */

float oracle_sum_squares_8lane(const float *x, int n) { /* rmsnorm.rs:55-69 */
    int n8 = n / 8 * 8;
    float l[8] = {0};
    for (int i = 0; i < n8; i += 8)
        for (int k = 0; k < 8; k++) l[k] += x[i + k] * x[i + k];
    float ss = oracle_reduce8(l);
    for (int i = n8; i < n; i++) ss += x[i] * x[i];
    return ss;
}

float oracle_inv_rms(const float *x, int n, float eps) { /* rmsnorm.rs:49-53 */
    float mean = oracle_sum_squares_8lane(x, n) / (float)n;
    return 1.0f / sqrtf(mean + eps);
}

void oracle_rmsnorm(const float *x, const float *w, int n, float eps, float *y) { /* rmsnorm.rs:25-33 */
    float inv = oracle_inv_rms(x, n, eps);
    for (int i = 0; i < n; i++) y[i] = (x[i] * inv) * w[i];
}

void oracle_rmsnorm_gated(const float *x, const float *gate, const float *w, int n, float eps, float *y) {
    float inv = oracle_inv_rms(x, n, eps); /* rmsnorm.rs:36-47 */
    for (int i = 0; i < n; i++) y[i] = (w[i] * (x[i] * inv)) * oracle_silu(gate[i]);
}

/* -------------------------------------------------------------------------- softmax (softmax.rs:22-50) */

void oracle_softmax(const float *x, int n, float *y) {
    float m = -INFINITY;
    for (int i = 0; i < n; i++)
        if (x[i] > m) m = x[i];
    for (int i = 0; i < n; i++) y[i] = oracle_expf(x[i] - m);
    int n8 = n / 8 * 8;
    float l[8] = {0};
    for (int i = 0; i < n8; i += 8)
        for (int k = 0; k < 8; k++) l[k] += y[i + k];
    float s = oracle_reduce8(l);
    for (int i = n8; i < n; i++) s += y[i];
    for (int i = 0; i < n; i++) y[i] /= s;
}

/* ------------------------------------------------------------------------------ RoPE (rope.rs:10-45) */

void oracle_inv_freq(int rope_dim, float theta, float *out) {
    for (int i = 0; i < rope_dim / 2; i++) out[i] = 1.0f / powf(theta, (float)(2 * i) / (float)rope_dim);
}

void oracle_cos_sin(uint32_t pos, const float *inv_freq, int half, float *cos, float *sin) {
    float p = (float)pos;
    for (int i = 0; i < half; i++) {
        float angle = p * inv_freq[i];
        float s = sinf(angle), c = cosf(angle);
        cos[i] = c;
        cos[i + half] = c;
        sin[i] = s;
        sin[i + half] = s;
    }
}

void oracle_apply_rope(float *x, int len, int head_dim, int rope_dim, const float *cos, const float *sin) {
    int half = rope_dim / 2;
    for (int h = 0; h + head_dim <= len; h += head_dim) {
        float *v = x + h;
        for (int i = 0; i < half; i++) {
            float a = v[i], b = v[i + half];
            v[i] = a * cos[i] - b * sin[i];
            v[i + half] = b * cos[i + half] + a * sin[i + half];
        }
    }
}

/* ------------------------------------------------------------------------------ conv1d (conv.rs:11-36) */

void oracle_conv1d_step(float *state, const float *w, int kernel, const float *x_new, int channels, float *out,
                        int act_silu) {
    for (int ch = 0; ch < channels; ch++) {
        float *st = state + (size_t)ch * (kernel - 1);
        const float *wc = w + (size_t)ch * kernel;
        float acc = 0.0f;
        for (int j = 0; j < kernel - 1; j++) acc += wc[j] * st[j];
        acc += wc[kernel - 1] * x_new[ch];
        for (int j = 0; j < kernel - 2; j++) st[j] = st[j + 1];
        if (kernel >= 2) st[kernel - 2] = x_new[ch];
        out[ch] = act_silu ? oracle_silu(acc) : acc;
    }
}

/* ---------------------------------------------------------------------------- DeltaNet (deltanet.rs:19-89) */

void oracle_l2norm(float *x, int n, float eps) {
    float ss = 0.0f;
    for (int i = 0; i < n; i++) ss += x[i] * x[i];
    float inv = 1.0f / sqrtf(ss + eps);
    for (int i = 0; i < n; i++) x[i] *= inv;
}

float oracle_gate_g(float a, float dt_bias, float big_a) { return big_a * oracle_softplus(a + dt_bias); }
float oracle_gate_beta(float b) { return oracle_sigmoid(b); }

void oracle_deltanet_step(const float *q, const float *k, const float *v, int dk, int dv, float g, float beta,
                          float *s, float *out) {
    float decay = oracle_expf(g);
    for (int i = 0; i < dk * dv; i++) s[i] *= decay;
    for (int j = 0; j < dv; j++) out[j] = 0.0f;
    for (int kk = 0; kk < dk; kk++)
        for (int j = 0; j < dv; j++) out[j] += s[kk * dv + j] * k[kk];
    for (int j = 0; j < dv; j++) out[j] = (v[j] - out[j]) * beta;
    for (int kk = 0; kk < dk; kk++)
        for (int j = 0; j < dv; j++) s[kk * dv + j] += k[kk] * out[j];
    for (int j = 0; j < dv; j++) out[j] = 0.0f;
    for (int kk = 0; kk < dk; kk++)
        for (int j = 0; j < dv; j++) out[j] += s[kk * dv + j] * q[kk];
}

/* ---------------------------------------------------------------------------- misc */

uint32_t oracle_argmax(const float *v, int n) { /* model.rs:505-513: first index on ties */
    int best = 0;
    for (int i = 1; i < n; i++)
        if (v[i] > v[best]) best = i;
    return (uint32_t)best;
}

uint32_t oracle_crc32(const uint8_t *p, size_t n) { /* quant.rs:234-249 */
    uint32_t table[256];
    for (uint32_t i = 0; i < 256; i++) {
        uint32_t c = i;
        for (int k = 0; k < 8; k++) c = (c & 1) ? 0xEDB88320u ^ (c >> 1) : c >> 1;
        table[i] = c;
    }
    uint32_t crc = 0xFFFFFFFFu;
    for (size_t i = 0; i < n; i++) crc = table[(crc ^ p[i]) & 0xFF] ^ (crc >> 8);
    return crc ^ 0xFFFFFFFFu;
}

/* ------------------------------------------------------------------------------------------------------------
 * The timed CPU baseline's kernels: an AVX2 restatement of the reference's SIMD dots
 * (crates/core/src/kernels/avx2.rs:934-1087, the blocked form of kdot.rs:176-333 that matmul_t runs:
 * one weight row decoded once per super-block for up to 16 activation rows), bit-identical to the scalar
 * kernels above -- the exact integer lanes come from maddubs (u8 x s8 pair sums, no saturation at these
 * magnitudes) and madd (the pair sums times the chunk scale, adjacent pairs added: i32 lane k = positions
 * 4k .. 4k+3 of the chunk, the reference's lane), and the f32 steps are the same multiply-then-add per lane in
 * the same order.  Q8_0 / Q4_0 blocks use the sign trick for the signed x signed byte products; F32 stays
 * scalar (its 32-term partial sums are sequential chains).  Rows are split over OpenMP threads, as the
 * reference splits them over its pool (kernels/matvec.rs:446-467).  oracle_set_simd(0) routes every matmul to
 * the scalar kernels.
 * ------------------------------------------------------------------------------------------------------------ */
#if defined(__x86_64__)
#include <immintrin.h>
#define OR_AVX2 __attribute__((target("avx2")))

static int g_simd = -1; /* -1: use AVX2 when the CPU has it */
void oracle_set_simd(int on) { g_simd = on; }
static int simd_on(void) {
    if (g_simd < 0) g_simd = __builtin_cpu_supports("avx2") ? 1 : 0;
    return g_simd;
}

OR_AVX2 static inline float hsum_lane_order8(__m256 v) { /* reduce8 in the reference order */
    float l[8];
    _mm256_storeu_ps(l, v);
    return oracle_reduce8(l);
}
OR_AVX2 static inline float hsum_lane_order4(__m128 v) {
    float m[4];
    _mm_storeu_ps(m, v);
    return reduce4(m);
}
OR_AVX2 static inline int hsum_epi32(__m256i v) { /* an exact integer sum: any order */
    __m128i s = _mm_add_epi32(_mm256_castsi256_si128(v), _mm256_extracti128_si256(v, 1));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0x4e));
    s = _mm_add_epi32(s, _mm_shuffle_epi32(s, 0xb1));
    return _mm_cvtsi128_si32(s);
}

/* Q4_K / Q5_K row x t Q8_K rows (kdot.rs:194-260, avx2.rs dot_q4_k_q8k_t / dot_q5_k_q8k_t) */
OR_AVX2 static void dot_q45_k_t_avx2(const uint8_t *w, const uint8_t *const *x, int t, int nb, int q5, float *out) {
    __m256 acc[16];
    __m128 accm[16];
    for (int c = 0; c < t; c++) acc[c] = _mm256_setzero_ps(), accm[c] = _mm_setzero_ps();
    const int bbytes = q5 ? 176 : 144;
    const __m256i m4 = _mm256_set1_epi8(0x0F), one = _mm256_set1_epi8(1);
    for (int sb = 0; sb < nb; sb++) {
        const uint8_t *wb = w + (size_t)sb * bbytes;
        const float dw = f16_at(wb, 0), dminw = f16_at(wb, 2);
        int sc[8], mn[8];
        for (int s = 0; s < 8; s++) scale_min_k4(s, wb + 4, &sc[s], &mn[s]);
        __m256i q[8], scv[8];
        const uint8_t *qs = wb + (q5 ? 48 : 16);
        __m256i qh = q5 ? _mm256_loadu_si256((const __m256i *)(wb + 16)) : _mm256_setzero_si256();
        for (int p = 0; p < 4; p++) {
            const __m256i raw = _mm256_loadu_si256((const __m256i *)(qs + 32 * p));
            q[2 * p] = _mm256_and_si256(raw, m4);
            q[2 * p + 1] = _mm256_and_si256(_mm256_srli_epi16(raw, 4), m4);
        }
        if (q5)
            for (int s = 0; s < 8; s++)
                q[s] = _mm256_or_si256(q[s], _mm256_slli_epi16(_mm256_and_si256(_mm256_srli_epi16(qh, s), one), 4));
        for (int s = 0; s < 8; s++) scv[s] = _mm256_set1_epi16((short)sc[s]);
        const __m128i mins = _mm_setr_epi16((short)mn[0], (short)mn[1], (short)mn[2], (short)mn[3], (short)mn[4], (short)mn[5],
                                            (short)mn[6], (short)mn[7]);
        for (int c = 0; c < t; c++) {
            const uint8_t *xb = x[c] + (size_t)sb * 292;
            const float dx = q8k_d(xb);
            const int8_t *xq = (const int8_t *)(xb + 4);
            __m256i sumi = _mm256_setzero_si256();
            for (int s = 0; s < 8; s++) {
                const __m256i xs = _mm256_loadu_si256((const __m256i *)(xq + 32 * s));
                sumi = _mm256_add_epi32(sumi, _mm256_madd_epi16(_mm256_maddubs_epi16(q[s], xs), scv[s]));
            }
            /* q8s[s] = bsums[2s] + bsums[2s+1] (q8k.rs:185-193), then mn . q8s pairwise: 4 exact i32 lanes */
            const __m128i bs0 = _mm_loadu_si128((const __m128i *)(xb + 260)), bs1 = _mm_loadu_si128((const __m128i *)(xb + 276));
            const __m128i q8s = _mm_hadd_epi16(bs0, bs1);
            const __m128i prod = _mm_madd_epi16(q8s, mins);
            const float d = dx * dw, dmin = -dx * dminw;
            accm[c] = _mm_add_ps(accm[c], _mm_mul_ps(_mm_set1_ps(dmin), _mm_cvtepi32_ps(prod)));
            acc[c] = _mm256_add_ps(acc[c], _mm256_mul_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi)));
        }
    }
    for (int c = 0; c < t; c++) out[c] = hsum_lane_order8(acc[c]) + hsum_lane_order4(accm[c]);
}

/* Q6_K row x t Q8_K rows (kdot.rs:262-312, avx2.rs dot_q6_k_q8k_t) */
OR_AVX2 static void dot_q6_k_t_avx2(const uint8_t *w, const uint8_t *const *x, int t, int nb, float *out) {
    __m256 acc[16];
    for (int c = 0; c < t; c++) acc[c] = _mm256_setzero_ps();
    const __m256i m4 = _mm256_set1_epi8(0x0F), m2 = _mm256_set1_epi8(0x03);
    for (int sb = 0; sb < nb; sb++) {
        const uint8_t *wb = w + (size_t)sb * 210;
        const float dw = f16_at(wb, 208);
        __m256i q[8], scv[8];
        for (int h = 0; h < 2; h++) {
            const __m256i ql0 = _mm256_loadu_si256((const __m256i *)(wb + 64 * h));
            const __m256i ql1 = _mm256_loadu_si256((const __m256i *)(wb + 64 * h + 32));
            const __m256i qh = _mm256_loadu_si256((const __m256i *)(wb + 128 + 32 * h));
            const __m256i lo[4] = {_mm256_and_si256(ql0, m4), _mm256_and_si256(ql1, m4), _mm256_and_si256(_mm256_srli_epi16(ql0, 4), m4),
                                   _mm256_and_si256(_mm256_srli_epi16(ql1, 4), m4)};
            for (int k = 0; k < 4; k++) {
                const __m256i hi = _mm256_and_si256(_mm256_srli_epi16(qh, 2 * k), m2);
                q[4 * h + k] = _mm256_or_si256(lo[k], _mm256_slli_epi16(hi, 4));
                const int8_t *sc = (const int8_t *)(wb + 192 + 8 * h + 2 * k);
                scv[4 * h + k] = _mm256_setr_m128i(_mm_set1_epi16(sc[0]), _mm_set1_epi16(sc[1]));
            }
        }
        /* the 16 scales as i16, for the -32 * (bsums . scales) correction of each lane */
        const __m256i sc16 = _mm256_cvtepi8_epi16(_mm_loadu_si128((const __m128i *)(wb + 192)));
        for (int c = 0; c < t; c++) {
            const uint8_t *xb = x[c] + (size_t)sb * 292;
            const int8_t *xq = (const int8_t *)(xb + 4);
            __m256i sumi = _mm256_setzero_si256();
            for (int s = 0; s < 8; s++) {
                const __m256i xs = _mm256_loadu_si256((const __m256i *)(xq + 32 * s));
                sumi = _mm256_add_epi32(sumi, _mm256_madd_epi16(_mm256_maddubs_epi16(q[s], xs), scv[s]));
            }
            const __m256i bs = _mm256_loadu_si256((const __m256i *)(xb + 260));
            sumi = _mm256_sub_epi32(sumi, _mm256_slli_epi32(_mm256_madd_epi16(bs, sc16), 5));
            const float d = q8k_d(xb) * dw;
            acc[c] = _mm256_add_ps(acc[c], _mm256_mul_ps(_mm256_set1_ps(d), _mm256_cvtepi32_ps(sumi)));
        }
    }
    for (int c = 0; c < t; c++) out[c] = hsum_lane_order8(acc[c]);
}

/* Q8_0 / Q4_0 row x one Q8_0 row (dot.rs:29-64): per 32-block an exact i32 sum, then the f32 chain */
OR_AVX2 static float dot_q80_avx2(const uint8_t *w, const uint8_t *x, int nb, int q4) {
    float acc = 0.0f;
    const __m256i m4 = _mm256_set1_epi8(0x0F), eight = _mm256_set1_epi8(8), ones = _mm256_set1_epi16(1);
    for (int b = 0; b < nb; b++) {
        const uint8_t *wb = w + (size_t)b * (q4 ? 18 : 34), *xb = x + (size_t)b * 34;
        __m256i wv;
        if (q4) {
            const __m128i raw = _mm_loadu_si128((const __m128i *)(wb + 2));
            wv = _mm256_sub_epi8(_mm256_and_si256(_mm256_setr_m128i(raw, _mm_srli_epi16(raw, 4)), m4), eight);
        } else {
            wv = _mm256_loadu_si256((const __m256i *)(wb + 2));
        }
        const __m256i xv = _mm256_loadu_si256((const __m256i *)(xb + 2));
        const __m256i p16 = _mm256_maddubs_epi16(_mm256_sign_epi8(wv, wv), _mm256_sign_epi8(xv, wv));
        const int isum = hsum_epi32(_mm256_madd_epi16(p16, ones));
        acc += (f16_at(wb, 0) * f16_at(xb, 0)) * (float)isum;
    }
    return acc;
}

int oracle_matmul_fast(int type, const uint8_t *w, int rows, int cols, const void *act, size_t act_stride, int ncols, float *y) {
    if (!simd_on() || type == OT_F32) return 0;
    const size_t rb = oracle_row_bytes(type, cols);
    const int nt = g_threads > 0 ? g_threads : omp_get_max_threads();
    for (int c0 = 0; c0 < ncols; c0 += 16) {
        const int tc = ncols - c0 < 16 ? ncols - c0 : 16;
        const uint8_t *xs[16];
        for (int c = 0; c < tc; c++) xs[c] = (const uint8_t *)act + (size_t)(c0 + c) * act_stride;
#pragma omp parallel for schedule(static) num_threads(nt)
        for (int r = 0; r < rows; r++) {
            const uint8_t *wr = w + (size_t)r * rb;
            float o[16];
            switch (type) {
            case OT_Q4_K: dot_q45_k_t_avx2(wr, xs, tc, cols / 256, 0, o); break;
            case OT_Q5_K: dot_q45_k_t_avx2(wr, xs, tc, cols / 256, 1, o); break;
            case OT_Q6_K: dot_q6_k_t_avx2(wr, xs, tc, cols / 256, o); break;
            default:
                for (int c = 0; c < tc; c++) o[c] = dot_q80_avx2(wr, xs[c], cols / 32, type == OT_Q4_0);
            }
            for (int c = 0; c < tc; c++) y[(size_t)(c0 + c) * rows + r] = o[c];
        }
    }
    return 1;
}
#else
void oracle_set_simd(int on) { (void)on; }
int oracle_matmul_fast(int type, const uint8_t *w, int rows, int cols, const void *act, size_t act_stride, int ncols, float *y) {
    return 0;
}
#endif
