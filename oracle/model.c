/*
 * CPU ORACLE (test infrastructure; see oracle.h): the model-level restatement of the reference engine.
 *
 *   GGUF reader           crates/core/src/gguf.rs:483-600 (header, KV, tensor index, aligned data section)
 *   config                crates/core/src/config.rs:146-260 (the keys this path needs)
 *   forward_token         crates/core/src/model.rs:364-438, :486-490; layers/mod.rs:295-330
 *   Gated DeltaNet        layers/gated_deltanet.rs:548-602 (token form)
 *   gated GQA             layers/gqa_attention.rs:155-234 (token form)
 *   MLP                   layers/mlp.rs:53-64
 *   MTP head              layers/mtp.rs:95-137
 *   speculative loop      spec.rs:229-433: verify of k+1 rows, greedy accept, snapshot/restore of the
 *                         DeltaNet states + KV truncation, MTP re-feed, chained drafts
 *
 * The reference's batched forms (forward_batch_in, prefill, matmul_t) are bit-identical to its token form
 * (its own tests/matmul_t.rs, spec_identity.rs); this oracle uses the token form throughout.  Weights are read
 * through mmap of the GGUF file.
 */
#include <errno.h>
#include <fcntl.h>
#include <math.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>
#include <time.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include "oracle.h"

#define MAXT 2048
#define MAXB 16 /* rows of one batched forward (the reference's matmul_t tile, kdot.rs T_MAX) */

typedef struct {
    char *name;
    int type;
    uint64_t ne[4];
    int nd;
    uint64_t off, bytes;
} OTensor;

typedef struct {
    int type, rows, cols;
    const uint8_t *data;
} OMat;

typedef struct {
    int attn;
    const float *attn_norm, *post_norm;
    OMat qkv, gate_z, alpha, beta, ssm_out;
    const float *ssm_a, *dt_bias, *conv_w, *ssm_norm;
    OMat q, k, v, o;
    const float *q_norm, *k_norm;
    OMat gate, up, down;
} OLayer;

typedef struct oracle_model {
    int fd;
    uint8_t *map;
    size_t map_len;
    uint64_t data_off;
    int n_tensors;
    OTensor *t;
    /* config */
    int n_layer, hidden, ffn, vocab, n_head, n_kv, hd, rope_dim, interval, conv_k, dk, n_k, n_v, dv, kd, vd, conv_dim;
    float eps, theta, scaling;
    uint32_t eos, stop2;
    OLayer *layers;
    OMat embed, lm_head;
    const float *out_norm;
    int has_mtp;
    OLayer mtp_block;
    OMat eh_proj;
    const float *enorm, *hnorm, *head_norm;
    char err[512];
} OModel;

typedef struct {
    float *S, *conv;  /* DeltaNet */
    float *K, *V;     /* attention: [max_pos][n_kv*hd] */
    /* the projections of the last batched call of a DeltaNet layer (the reference's DeltaBatch, spec.rs replay):
     * mixed [MAXB][conv_dim], z [MAXB][vd], a / b [MAXB][n_v] */
    float *sv_mixed, *sv_z, *sv_ga, *sv_gb;
} OLayerState;

typedef struct oracle_state {
    OModel *m;
    int max_pos, pos;
    OLayerState *ls;
    float *mtpK, *mtpV;
    int mtp_len;
} OState;

/* ------------------------------------------------------------------------------------------ GGUF */

typedef struct {
    const uint8_t *p, *end;
    int ok;
} Rd;

static uint64_t rd_u(Rd *r, int n) {
    if (r->p + n > r->end) { r->ok = 0; return 0; }
    uint64_t v = 0;
    memcpy(&v, r->p, n);
    r->p += n;
    return v;
}
static void rd_skip_value(Rd *r, uint32_t t);
static void rd_skip_value(Rd *r, uint32_t t) {
    static const int sz[] = {1, 1, 2, 2, 4, 4, 4, 1, 0, 0, 8, 8, 8};
    if (t == 8) { uint64_t n = rd_u(r, 8); if (r->p + n > r->end) { r->ok = 0; return; } r->p += n; return; }
    if (t == 9) {
        uint32_t et = (uint32_t)rd_u(r, 4);
        uint64_t n = rd_u(r, 8);
        for (uint64_t i = 0; i < n && r->ok; i++) rd_skip_value(r, et);
        return;
    }
    if (t > 12) { r->ok = 0; return; }
    r->p += sz[t];
}

typedef struct {
    char key[128];
    uint32_t type;
    const uint8_t *val; /* pointer at the value */
} OKv;

static int kv_find(OKv *kv, int n, const char *key) {
    for (int i = 0; i < n; i++)
        if (!strcmp(kv[i].key, key)) return i;
    return -1;
}
static int kv_u32(OKv *kv, int n, const char *key, uint32_t *out) {
    int i = kv_find(kv, n, key);
    if (i < 0 || kv[i].type != 4) return -1;
    memcpy(out, kv[i].val, 4);
    return 0;
}
static int kv_f32(OKv *kv, int n, const char *key, float *out) {
    int i = kv_find(kv, n, key);
    if (i < 0 || kv[i].type != 6) return -1;
    memcpy(out, kv[i].val, 4);
    return 0;
}

static OTensor *find_t(OModel *m, const char *name) {
    for (int i = 0; i < m->n_tensors; i++)
        if (!strcmp(m->t[i].name, name)) return &m->t[i];
    return NULL;
}

static int get_mat(OModel *m, const char *name, int rows, int cols, OMat *out) {
    OTensor *t = find_t(m, name);
    if (!t || t->nd != 2 || (int)t->ne[0] != cols || (int)t->ne[1] != rows) {
        snprintf(m->err, sizeof m->err, "tensor %s missing or not [%d, %d]", name, rows, cols);
        return -1;
    }
    out->type = t->type;
    out->rows = rows;
    out->cols = cols;
    out->data = m->map + m->data_off + t->off;
    return 0;
}
static const float *get_vec(OModel *m, const char *name, int len) {
    OTensor *t = find_t(m, name);
    uint64_t n = 1;
    if (!t) { snprintf(m->err, sizeof m->err, "tensor %s missing", name); return NULL; }
    for (int d = 0; d < t->nd; d++) n *= t->ne[d];
    if ((int)n != len || t->type != OT_F32) { snprintf(m->err, sizeof m->err, "tensor %s: %llu elements or not F32", name, (unsigned long long)n); return NULL; }
    return (const float *)(m->map + m->data_off + t->off);
}

static int load_layer(OModel *m, int i, int attn, OLayer *L) {
    char p[64], n[160];
    snprintf(p, sizeof p, "blk.%d.", i);
    memset(L, 0, sizeof *L);
    L->attn = attn;
#define V(field, suffix, len) do { snprintf(n, sizeof n, "%s%s", p, suffix); if (!(L->field = get_vec(m, n, len))) return -1; } while (0)
#define M(field, suffix, r, c) do { snprintf(n, sizeof n, "%s%s", p, suffix); if (get_mat(m, n, r, c, &L->field)) return -1; } while (0)
    V(attn_norm, "attn_norm.weight", m->hidden);
    V(post_norm, "post_attention_norm.weight", m->hidden);
    if (attn) {
        M(q, "attn_q.weight", 2 * m->n_head * m->hd, m->hidden);
        M(k, "attn_k.weight", m->n_kv * m->hd, m->hidden);
        M(v, "attn_v.weight", m->n_kv * m->hd, m->hidden);
        M(o, "attn_output.weight", m->hidden, m->n_head * m->hd);
        V(q_norm, "attn_q_norm.weight", m->hd);
        V(k_norm, "attn_k_norm.weight", m->hd);
    } else {
        M(qkv, "attn_qkv.weight", m->conv_dim, m->hidden);
        M(gate_z, "attn_gate.weight", m->vd, m->hidden);
        M(alpha, "ssm_alpha.weight", m->n_v, m->hidden);
        M(beta, "ssm_beta.weight", m->n_v, m->hidden);
        V(ssm_a, "ssm_a", m->n_v);
        V(dt_bias, "ssm_dt.bias", m->n_v);
        V(conv_w, "ssm_conv1d.weight", m->conv_dim * m->conv_k);
        V(ssm_norm, "ssm_norm.weight", m->dv);
        M(ssm_out, "ssm_out.weight", m->hidden, m->vd);
    }
    M(gate, "ffn_gate.weight", m->ffn, m->hidden);
    M(up, "ffn_up.weight", m->ffn, m->hidden);
    M(down, "ffn_down.weight", m->hidden, m->ffn);
#undef V
#undef M
    return 0;
}

void oracle_model_close(OModel *m);

OModel *oracle_model_open(const char *path, char *err, int errlen) {
    OModel *m = (OModel *)calloc(1, sizeof *m);
    OKv *kv = NULL;
    m->fd = open(path, O_RDONLY);
    if (m->fd < 0) { snprintf(err, errlen, "cannot open %s: %s", path, strerror(errno)); free(m); return NULL; }
    struct stat st;
    fstat(m->fd, &st);
    m->map_len = (size_t)st.st_size;
    m->map = (uint8_t *)mmap(NULL, m->map_len, PROT_READ, MAP_PRIVATE, m->fd, 0);
    if (m->map == MAP_FAILED) { snprintf(err, errlen, "mmap failed"); close(m->fd); free(m); return NULL; }
    Rd r = {m->map, m->map + m->map_len, 1};
    uint32_t magic = (uint32_t)rd_u(&r, 4), ver = (uint32_t)rd_u(&r, 4);
    if (magic != 0x46554747u || ver != 3) { snprintf(err, errlen, "not a GGUF v3 file"); goto fail; }
    uint64_t nt = rd_u(&r, 8), nkv = rd_u(&r, 8);
    kv = (OKv *)calloc(nkv ? nkv : 1, sizeof *kv);
    for (uint64_t i = 0; i < nkv && r.ok; i++) {
        uint64_t kl = rd_u(&r, 8);
        if (kl >= sizeof kv[i].key || r.p + kl > r.end) { r.ok = 0; break; }
        memcpy(kv[i].key, r.p, kl);
        r.p += kl;
        kv[i].type = (uint32_t)rd_u(&r, 4);
        kv[i].val = r.p;
        rd_skip_value(&r, kv[i].type);
    }
    m->n_tensors = (int)nt;
    m->t = (OTensor *)calloc(nt ? nt : 1, sizeof *m->t);
    for (uint64_t i = 0; i < nt && r.ok; i++) {
        uint64_t nl = rd_u(&r, 8);
        if (r.p + nl > r.end) { r.ok = 0; break; }
        m->t[i].name = (char *)calloc(nl + 1, 1);
        memcpy(m->t[i].name, r.p, nl);
        r.p += nl;
        m->t[i].nd = (int)rd_u(&r, 4);
        uint64_t n = 1;
        for (int d = 0; d < m->t[i].nd && d < 4; d++) n *= (m->t[i].ne[d] = rd_u(&r, 8));
        m->t[i].type = (int)rd_u(&r, 4);
        m->t[i].off = rd_u(&r, 8);
        int be, bb;
        if (!oracle_block_layout(m->t[i].type, &be, &bb)) { snprintf(err, errlen, "unsupported type of %s", m->t[i].name); goto fail; }
        m->t[i].bytes = n / be * bb;
    }
    if (!r.ok) { snprintf(err, errlen, "header truncated"); goto fail; }
    uint32_t align = 32;
    kv_u32(kv, (int)nkv, "general.alignment", &align);
    uint64_t hdr = (uint64_t)(r.p - m->map);
    m->data_off = (hdr + align - 1) / align * align;
    uint32_t u;
#define U(field, key) do { if (kv_u32(kv, (int)nkv, key, &u)) { snprintf(err, errlen, "metadata key missing: %s", key); goto fail; } m->field = (int)u; } while (0)
    uint32_t bc, nn;
    if (kv_u32(kv, (int)nkv, "qwen35.block_count", &bc) || kv_u32(kv, (int)nkv, "qwen35.nextn_predict_layers", &nn)) {
        snprintf(err, errlen, "metadata key missing: block_count");
        goto fail;
    }
    m->n_layer = (int)(bc - nn);
    U(hidden, "qwen35.embedding_length");
    U(ffn, "qwen35.feed_forward_length");
    U(n_head, "qwen35.attention.head_count");
    U(n_kv, "qwen35.attention.head_count_kv");
    U(hd, "qwen35.attention.key_length");
    U(rope_dim, "qwen35.rope.dimension_count");
    U(interval, "qwen35.full_attention_interval");
    U(conv_k, "qwen35.ssm.conv_kernel");
    U(dk, "qwen35.ssm.state_size");
    U(n_k, "qwen35.ssm.group_count");
    U(n_v, "qwen35.ssm.time_step_rank");
    U(vd, "qwen35.ssm.inner_size");
#undef U
    if (kv_f32(kv, (int)nkv, "qwen35.attention.layer_norm_rms_epsilon", &m->eps) || kv_f32(kv, (int)nkv, "qwen35.rope.freq_base", &m->theta)) {
        snprintf(err, errlen, "metadata key missing: eps / freq_base");
        goto fail;
    }
    kv_u32(kv, (int)nkv, "tokenizer.ggml.eos_token_id", &m->eos);
    m->stop2 = 248044; /* the architecture's extra stop id (crates/core/src/arch.rs:71) */
    {
        int ti = kv_find(kv, (int)nkv, "tokenizer.ggml.tokens");
        if (ti < 0) { snprintf(err, errlen, "metadata key missing: tokenizer.ggml.tokens"); goto fail; }
        uint64_t cnt;
        memcpy(&cnt, kv[ti].val + 4, 8);
        m->vocab = (int)cnt;
    }
    m->dv = m->vd / m->n_v;
    m->kd = m->n_k * m->dk;
    m->conv_dim = 2 * m->kd + m->vd;
    m->scaling = powf((float)m->hd, -0.5f);
    m->layers = (OLayer *)calloc(m->n_layer, sizeof *m->layers);
    for (int i = 0; i < m->n_layer; i++) {
        char nm[64];
        snprintf(nm, sizeof nm, "blk.%d.attn_q.weight", i);
        int attn = find_t(m, nm) != NULL;
        if (load_layer(m, i, attn, &m->layers[i])) { snprintf(err, errlen, "%s", m->err); goto fail; }
    }
    if (get_mat(m, "token_embd.weight", m->vocab, m->hidden, &m->embed) ||
        get_mat(m, find_t(m, "output.weight") ? "output.weight" : "token_embd.weight", m->vocab, m->hidden, &m->lm_head) ||
        !(m->out_norm = get_vec(m, "output_norm.weight", m->hidden))) {
        snprintf(err, errlen, "%s", m->err);
        goto fail;
    }
    if (nn > 0) {
        char nm[96];
        int mi = m->n_layer;
        if (load_layer(m, mi, 1, &m->mtp_block)) { snprintf(err, errlen, "%s", m->err); goto fail; }
        snprintf(nm, sizeof nm, "blk.%d.nextn.eh_proj.weight", mi);
        if (get_mat(m, nm, m->hidden, 2 * m->hidden, &m->eh_proj)) { snprintf(err, errlen, "%s", m->err); goto fail; }
        snprintf(nm, sizeof nm, "blk.%d.nextn.enorm.weight", mi);
        m->enorm = get_vec(m, nm, m->hidden);
        snprintf(nm, sizeof nm, "blk.%d.nextn.hnorm.weight", mi);
        m->hnorm = get_vec(m, nm, m->hidden);
        snprintf(nm, sizeof nm, "blk.%d.nextn.shared_head_norm.weight", mi);
        m->head_norm = get_vec(m, nm, m->hidden);
        if (!m->enorm || !m->hnorm || !m->head_norm) { snprintf(err, errlen, "%s", m->err); goto fail; }
        m->has_mtp = 1;
    }
    free(kv);
    return m;
fail:
    free(kv);
    oracle_model_close(m);
    return NULL;
}

void oracle_model_close(OModel *m) {
    if (!m) return;
    if (m->map && m->map != MAP_FAILED) munmap(m->map, m->map_len);
    if (m->fd >= 0) close(m->fd);
    for (int i = 0; i < m->n_tensors; i++) free(m->t[i].name);
    free(m->t);
    free(m->layers);
    free(m);
}

int oracle_model_dims(OModel *m, int *out8) {
    out8[0] = m->n_layer;
    out8[1] = m->hidden;
    out8[2] = m->vocab;
    out8[3] = m->has_mtp;
    out8[4] = (int)m->eos;
    out8[5] = m->ffn;
    out8[6] = m->n_head;
    out8[7] = m->hd;
    return 0;
}

/* ----------------------------------------------------------------------------------------- state */

OState *oracle_state_new(OModel *m, int max_pos) {
    OState *s = (OState *)calloc(1, sizeof *s);
    s->m = m;
    s->max_pos = max_pos;
    s->ls = (OLayerState *)calloc(m->n_layer, sizeof *s->ls);
    size_t kvd = (size_t)m->n_kv * m->hd;
    for (int i = 0; i < m->n_layer; i++) {
        if (m->layers[i].attn) {
            s->ls[i].K = (float *)calloc((size_t)max_pos * kvd, 4);
            s->ls[i].V = (float *)calloc((size_t)max_pos * kvd, 4);
        } else {
            s->ls[i].S = (float *)calloc((size_t)m->n_v * m->dk * m->dv, 4);
            s->ls[i].conv = (float *)calloc((size_t)m->conv_dim * (m->conv_k - 1), 4);
            s->ls[i].sv_mixed = (float *)calloc((size_t)MAXB * m->conv_dim, 4);
            s->ls[i].sv_z = (float *)calloc((size_t)MAXB * m->vd, 4);
            s->ls[i].sv_ga = (float *)calloc((size_t)MAXB * m->n_v, 4);
            s->ls[i].sv_gb = (float *)calloc((size_t)MAXB * m->n_v, 4);
        }
    }
    if (m->has_mtp) {
        s->mtpK = (float *)calloc((size_t)max_pos * kvd, 4);
        s->mtpV = (float *)calloc((size_t)max_pos * kvd, 4);
    }
    return s;
}

void oracle_state_free(OState *s) {
    if (!s) return;
    for (int i = 0; i < s->m->n_layer; i++) {
        free(s->ls[i].S);
        free(s->ls[i].conv);
        free(s->ls[i].sv_mixed);
        free(s->ls[i].sv_z);
        free(s->ls[i].sv_ga);
        free(s->ls[i].sv_gb);
        free(s->ls[i].K);
        free(s->ls[i].V);
    }
    free(s->ls);
    free(s->mtpK);
    free(s->mtpV);
    free(s);
}

/* snapshot / restore of the DeltaNet states (spec.rs:154-179); KV caches roll back by length */
static float *snapshot(OState *s) {
    OModel *m = s->m;
    size_t per = (size_t)m->n_v * m->dk * m->dv + (size_t)m->conv_dim * (m->conv_k - 1), n = 0;
    for (int i = 0; i < m->n_layer; i++) n += m->layers[i].attn ? 0 : per;
    float *snap = (float *)malloc((n ? n : 1) * 4), *p = snap;
    for (int i = 0; i < m->n_layer; i++) {
        if (m->layers[i].attn) continue;
        memcpy(p, s->ls[i].S, (size_t)m->n_v * m->dk * m->dv * 4);
        p += (size_t)m->n_v * m->dk * m->dv;
        memcpy(p, s->ls[i].conv, (size_t)m->conv_dim * (m->conv_k - 1) * 4);
        p += (size_t)m->conv_dim * (m->conv_k - 1);
    }
    return snap;
}
static void restore(OState *s, const float *snap) {
    OModel *m = s->m;
    const float *p = snap;
    for (int i = 0; i < m->n_layer; i++) {
        if (m->layers[i].attn) continue;
        memcpy(s->ls[i].S, p, (size_t)m->n_v * m->dk * m->dv * 4);
        p += (size_t)m->n_v * m->dk * m->dv;
        memcpy(s->ls[i].conv, p, (size_t)m->conv_dim * (m->conv_k - 1) * 4);
        p += (size_t)m->conv_dim * (m->conv_k - 1);
    }
}

/* ---------------------------------------------------------------------------------------- layers */

static void matvec(const OMat *w, const float *x, float *y) { oracle_matmul_f32in(w->type, w->data, w->rows, w->cols, x, 1, y); }

static void matmul_rows(const OMat *w, const float *x, int t, float *y) {
    oracle_matmul_f32in(w->type, w->data, w->rows, w->cols, x, t, y);
}

/* The DeltaNet recurrence of one row from its projections (gated_deltanet.rs:562-598): the conv step, then per V
 * head p (K head p % n_k) l2norm, the gates, the delta rule and the gated RMSNorm into heads.  The heads are
 * independent (each has its own state), so they are spread over the threads. */
static void deltanet_recur(OModel *m, const OLayer *L, OLayerState *st, const float *mixed, const float *z, const float *ga,
                           const float *gb, float *heads) {
    float *conved = (float *)malloc((size_t)m->conv_dim * 4);
    oracle_conv1d_step(st->conv, L->conv_w, m->conv_k, mixed, m->conv_dim, conved, 1);
    const float scale = 1.0f / sqrtf((float)m->dk);
#pragma omp parallel for schedule(static) if (m->n_v >= 16)
    for (int p = 0; p < m->n_v; p++) {
        float qn[256], kn[256], o[256];
        int kh = p % m->n_k;
        memcpy(qn, conved + kh * m->dk, (size_t)m->dk * 4);
        memcpy(kn, conved + m->kd + kh * m->dk, (size_t)m->dk * 4);
        oracle_l2norm(qn, m->dk, 1e-6f);
        oracle_l2norm(kn, m->dk, 1e-6f);
        for (int i = 0; i < m->dk; i++) qn[i] *= scale;
        float g = oracle_gate_g(ga[p], L->dt_bias[p], L->ssm_a[p]);
        float beta = oracle_gate_beta(gb[p]);
        oracle_deltanet_step(qn, kn, conved + 2 * m->kd + p * m->dv, m->dk, m->dv, g, beta, st->S + (size_t)p * m->dk * m->dv, o);
        if (heads) oracle_rmsnorm_gated(o, z + p * m->dv, L->ssm_norm, m->dv, m->eps, heads + p * m->dv);
    }
    free(conved);
}

/* gated_deltanet.rs:548-602 */
static void deltanet_token(OModel *m, const OLayer *L, OLayerState *st, const float *x, float *y) {
    float *mixed = (float *)malloc((size_t)m->conv_dim * 4), *z = (float *)malloc((size_t)m->vd * 4);
    float *ga = (float *)malloc((size_t)m->n_v * 4), *gb = (float *)malloc((size_t)m->n_v * 4), *heads = (float *)malloc((size_t)m->vd * 4);
    matmul_rows(&L->qkv, x, 1, mixed);
    matmul_rows(&L->gate_z, x, 1, z);
    matmul_rows(&L->alpha, x, 1, ga);
    matmul_rows(&L->beta, x, 1, gb);
    deltanet_recur(m, L, st, mixed, z, ga, gb, heads);
    matmul_rows(&L->ssm_out, heads, 1, y);
    free(mixed); free(z); free(ga); free(gb); free(heads);
}

/* The attention of one row at `pos` from its projections (gqa_attention.rs:170-228): q/k RMSNorm, RoPE on the
 * first rope_dim dims, the K/V append, scores over the cache, softmax, the value sum and the sigmoid gate into
 * attn (n_head * head_dim).  k is normed and rotated in place.  The query heads are spread over the threads. */
static void attention_recur(OModel *m, const OLayer *L, float *K, float *V, int pos, const float *qg, float *k, const float *v,
                            float *attn) {
    const int nh = m->n_head, nkv = m->n_kv, hd = m->hd, rd = m->rope_dim, group = nh / nkv;
    float inv[128], cs[256], sn[256], tmp[512];
    const int len = pos + 1;
    oracle_inv_freq(rd, m->theta, inv);
    oracle_cos_sin((uint32_t)pos, inv, rd / 2, cs, sn);
    for (int h = 0; h < nkv; h++) {
        oracle_rmsnorm(k + (size_t)h * hd, L->k_norm, hd, m->eps, tmp);
        oracle_apply_rope(tmp, hd, hd, rd, cs, sn);
        memcpy(k + (size_t)h * hd, tmp, (size_t)hd * 4);
    }
    memcpy(K + (size_t)pos * nkv * hd, k, (size_t)nkv * hd * 4);
    memcpy(V + (size_t)pos * nkv * hd, v, (size_t)nkv * hd * 4);
#pragma omp parallel for schedule(static) if (nh >= 8 && len >= 64)
    for (int h = 0; h < nh; h++) {
        float qh[512];
        float *sc = (float *)malloc((size_t)len * 4), *pr = (float *)malloc((size_t)len * 4);
        oracle_rmsnorm(qg + (size_t)h * 2 * hd, L->q_norm, hd, m->eps, qh);
        oracle_apply_rope(qh, hd, hd, rd, cs, sn);
        int kvh = h / group;
        for (int t = 0; t < len; t++) {
            const float *kt = K + ((size_t)t * nkv + kvh) * hd;
            float s = 0.0f;
            for (int d = 0; d < hd; d++) s += qh[d] * kt[d];
            sc[t] = s * m->scaling;
        }
        oracle_softmax(sc, len, pr);
        float *out = attn + (size_t)h * hd;
        for (int d = 0; d < hd; d++) out[d] = 0.0f;
        for (int t = 0; t < len; t++) {
            const float *vt = V + ((size_t)t * nkv + kvh) * hd;
            for (int d = 0; d < hd; d++) out[d] += pr[t] * vt[d];
        }
        for (int d = 0; d < hd; d++) out[d] *= oracle_sigmoid(qg[(size_t)h * 2 * hd + hd + d]);
        free(sc);
        free(pr);
    }
}

/* gqa_attention.rs:155-234 */
static void attention_token(OModel *m, const OLayer *L, float *K, float *V, int pos, const float *x, float *y) {
    const int nh = m->n_head, nkv = m->n_kv, hd = m->hd;
    float *qg = (float *)malloc((size_t)2 * nh * hd * 4), *k = (float *)malloc((size_t)nkv * hd * 4), *v = (float *)malloc((size_t)nkv * hd * 4);
    float *attn = (float *)malloc((size_t)nh * hd * 4);
    matmul_rows(&L->q, x, 1, qg);
    matmul_rows(&L->k, x, 1, k);
    matmul_rows(&L->v, x, 1, v);
    attention_recur(m, L, K, V, pos, qg, k, v, attn);
    matmul_rows(&L->o, attn, 1, y);
    free(qg); free(k); free(v); free(attn);
}

/* layers/mlp.rs:53-64: y = down(swiglu(gate(x), up(x))) */
static void mlp_token(OModel *m, const OLayer *L, const float *x, float *y) {
    float *g = (float *)malloc((size_t)m->ffn * 4), *u = (float *)malloc((size_t)m->ffn * 4), *hh = (float *)malloc((size_t)m->ffn * 4);
    matvec(&L->gate, x, g);
    matvec(&L->up, x, u);
    oracle_swiglu(g, u, m->ffn, hh);
    matvec(&L->down, hh, y);
    free(g); free(u); free(hh);
}

/* layers/mod.rs:295-330: h = x + mixer(norm(x)); y = h + mlp(norm(h)) */
static void layer_token(OModel *m, const OLayer *L, OLayerState *st, float *K, float *V, int pos, const float *x, float *y) {
    const int H = m->hidden;
    float *normed = (float *)malloc((size_t)H * 4), *mixed = (float *)malloc((size_t)H * 4), *resid = (float *)malloc((size_t)H * 4);
    oracle_rmsnorm(x, L->attn_norm, H, m->eps, normed);
    if (L->attn) attention_token(m, L, K, V, pos, normed, mixed);
    else deltanet_token(m, L, st, normed, mixed);
    for (int i = 0; i < H; i++) resid[i] = x[i] + mixed[i];
    oracle_rmsnorm(resid, L->post_norm, H, m->eps, normed);
    mlp_token(m, L, normed, mixed);
    for (int i = 0; i < H; i++) y[i] = resid[i] + mixed[i];
    free(normed); free(mixed); free(resid);
}

/* layers/mod.rs:335-377 (DecoderLayer::forward_batch_in): t rows at positions pos0 .. pos0 + t - 1.  Every matrix
 * multiplies the t rows in one pass over its weights (matmul_t), the recurrences (conv + DeltaNet state, K/V append
 * + attention) run row by row in order -- the reference's batched form, bit-identical to its token form.  A
 * DeltaNet layer keeps its projections for the replay of a rolled-back verify (st->sv_*). */
static void layer_rows(OModel *m, const OLayer *L, OLayerState *st, float *K, float *V, int pos0, int t, const float *x, float *y) {
    const size_t H = (size_t)m->hidden;
    float *normed = (float *)malloc(t * H * 4), *out = (float *)malloc(t * H * 4), *resid = (float *)malloc(t * H * 4);
    for (int i = 0; i < t; i++) oracle_rmsnorm(x + i * H, L->attn_norm, (int)H, m->eps, normed + i * H);
    if (L->attn) {
        const size_t qd = (size_t)2 * m->n_head * m->hd, kvd = (size_t)m->n_kv * m->hd, ad = (size_t)m->n_head * m->hd;
        float *qg = (float *)malloc(t * qd * 4), *k = (float *)malloc(t * kvd * 4), *v = (float *)malloc(t * kvd * 4);
        float *attn = (float *)malloc(t * ad * 4);
        matmul_rows(&L->q, normed, t, qg);
        matmul_rows(&L->k, normed, t, k);
        matmul_rows(&L->v, normed, t, v);
        for (int i = 0; i < t; i++) attention_recur(m, L, K, V, pos0 + i, qg + i * qd, k + i * kvd, v + i * kvd, attn + i * ad);
        matmul_rows(&L->o, attn, t, out);
        free(qg); free(k); free(v); free(attn);
    } else {
        const size_t cd = (size_t)m->conv_dim, vd = (size_t)m->vd, nv = (size_t)m->n_v;
        float *mixed = (float *)malloc(t * cd * 4), *z = (float *)malloc(t * vd * 4), *ga = (float *)malloc(t * nv * 4);
        float *gb = (float *)malloc(t * nv * 4), *heads = (float *)malloc(t * vd * 4);
        matmul_rows(&L->qkv, normed, t, mixed);
        matmul_rows(&L->gate_z, normed, t, z);
        matmul_rows(&L->alpha, normed, t, ga);
        matmul_rows(&L->beta, normed, t, gb);
        if (st->sv_mixed && t <= MAXB) {
            memcpy(st->sv_mixed, mixed, t * cd * 4);
            memcpy(st->sv_z, z, t * vd * 4);
            memcpy(st->sv_ga, ga, t * nv * 4);
            memcpy(st->sv_gb, gb, t * nv * 4);
        }
        for (int i = 0; i < t; i++) deltanet_recur(m, L, st, mixed + i * cd, z + i * vd, ga + i * nv, gb + i * nv, heads + i * vd);
        matmul_rows(&L->ssm_out, heads, t, out);
        free(mixed); free(z); free(ga); free(gb); free(heads);
    }
    for (size_t i = 0; i < t * H; i++) resid[i] = x[i] + out[i];
    for (int i = 0; i < t; i++) oracle_rmsnorm(resid + i * H, L->post_norm, (int)H, m->eps, normed + i * H);
    const size_t F = (size_t)m->ffn;
    float *g = (float *)malloc(t * F * 4), *u = (float *)malloc(t * F * 4), *hh = (float *)malloc(t * F * 4);
    matmul_rows(&L->gate, normed, t, g);
    matmul_rows(&L->up, normed, t, u);
    oracle_swiglu(g, u, (int)(t * F), hh);
    matmul_rows(&L->down, hh, t, out);
    for (size_t i = 0; i < t * H; i++) y[i] = resid[i] + out[i];
    free(g); free(u); free(hh); free(normed); free(out); free(resid);
}

static void embed_row(OModel *m, uint32_t id, float *out) {
    size_t rb = oracle_row_bytes(m->embed.type, m->hidden);
    oracle_dequantize(m->embed.type, m->embed.data + (size_t)id * rb, rb, out, (size_t)m->hidden);
}

/* Model::forward_token (model.rs:486-490): logits [vocab]; optional capture [n_layer + 1][hidden] of the
 * residual after each layer and the post-final-norm row; `normed_out` receives the post-final-norm row. */
int oracle_forward_token(OState *s, uint32_t id, float *logits, float *capture, float *normed_out) {
    OModel *m = s->m;
    const int H = m->hidden;
    if (id >= (uint32_t)m->vocab || s->pos >= s->max_pos) return -1;
    float *x = (float *)malloc((size_t)H * 4), *y = (float *)malloc((size_t)H * 4), *nrm = (float *)malloc((size_t)H * 4);
    embed_row(m, id, x);
    for (int i = 0; i < m->n_layer; i++) {
        layer_token(m, &m->layers[i], &s->ls[i], s->ls[i].K, s->ls[i].V, s->pos, x, y);
        memcpy(x, y, (size_t)H * 4);
        if (capture) memcpy(capture + (size_t)i * H, x, (size_t)H * 4);
    }
    oracle_rmsnorm(x, m->out_norm, H, m->eps, nrm);
    if (capture) memcpy(capture + (size_t)m->n_layer * H, nrm, (size_t)H * 4);
    if (normed_out) memcpy(normed_out, nrm, (size_t)H * 4);
    if (logits) matvec(&m->lm_head, nrm, logits);
    s->pos++;
    free(x); free(y); free(nrm);
    return 0;
}

/* Model::prefill / forward_batch (model.rs:401-461, spec.rs:301): t <= MAXB rows from s->pos; logits of every row
 * (logits_rows = t) or of the last one (1) or none (0); normed_out: the t post-final-norm rows. */
static int forward_rows(OState *s, const uint32_t *ids, int t, float *logits, int logits_rows, float *normed_out) {
    OModel *m = s->m;
    const size_t H = (size_t)m->hidden;
    if (t <= 0 || t > MAXB || s->pos + t > s->max_pos) return -1;
    for (int i = 0; i < t; i++)
        if (ids[i] >= (uint32_t)m->vocab) return -1;
    float *x = (float *)malloc(t * H * 4), *y = (float *)malloc(t * H * 4), *nrm = (float *)malloc(t * H * 4);
    for (int i = 0; i < t; i++) embed_row(m, ids[i], x + i * H);
    for (int l = 0; l < m->n_layer; l++) {
        layer_rows(m, &m->layers[l], &s->ls[l], s->ls[l].K, s->ls[l].V, s->pos, t, x, y);
        float *tmp = x;
        x = y;
        y = tmp;
    }
    for (int i = 0; i < t; i++) oracle_rmsnorm(x + i * H, m->out_norm, (int)H, m->eps, nrm + i * H);
    if (normed_out) memcpy(normed_out, nrm, t * H * 4);
    if (logits && logits_rows == t) matmul_rows(&m->lm_head, nrm, t, logits);
    else if (logits && logits_rows == 1) matmul_rows(&m->lm_head, nrm + (t - 1) * H, 1, logits);
    s->pos += t;
    free(x); free(y); free(nrm);
    return 0;
}

/* The prompt through forward_rows in chunks of MAXB rows (Model::prefill); logits of the last row, the post-norm
 * rows of every prompt position into normed_all when given. */
static int prefill_rows(OState *s, const uint32_t *ids, int n, float *logits, float *normed_all) {
    const size_t H = (size_t)s->m->hidden;
    for (int off = 0; off < n; off += MAXB) {
        const int t = n - off < MAXB ? n - off : MAXB;
        if (forward_rows(s, ids + off, t, off + t == n ? logits : NULL, off + t == n ? 1 : 0, normed_all ? normed_all + off * H : NULL))
            return -1;
    }
    return 0;
}

/* The MTP block over t rows (layers/mtp.rs:95-130, rows_in): row i = [enorm(embed(toks[i])) | hnorm(h_i)] ->
 * eh_proj -> the block's attention decoder layer at MTP positions mtp_len .. -> shared_head_norm into hout. */
static void mtp_rows_batch(OState *s, const uint32_t *toks, const float *h, int t, float *hout) {
    OModel *m = s->m;
    const size_t H = (size_t)m->hidden;
    float *e = (float *)malloc(H * 4), *cat = (float *)malloc(t * 2 * H * 4), *u = (float *)malloc(t * H * 4);
    float *yy = (float *)malloc(t * H * 4);
    for (int i = 0; i < t; i++) {
        embed_row(m, toks[i], e);
        oracle_rmsnorm(e, m->enorm, (int)H, m->eps, cat + i * 2 * H);
        oracle_rmsnorm(h + i * H, m->hnorm, (int)H, m->eps, cat + i * 2 * H + H);
    }
    matmul_rows(&m->eh_proj, cat, t, u);
    OLayerState none;
    memset(&none, 0, sizeof none);
    layer_rows(m, &m->mtp_block, &none, s->mtpK, s->mtpV, s->mtp_len, t, u, yy);
    for (int i = 0; i < t; i++) oracle_rmsnorm(yy + i * H, m->head_norm, (int)H, m->eps, hout + i * H);
    s->mtp_len += t;
    free(e); free(cat); free(u); free(yy);
}

/* One MTP row (layers/mtp.rs:95-137): hout = head_norm(block([enorm(embed(tok)) | hnorm(h)] @ eh_proj)),
 * at MTP position s->mtp_len; returns the greedy draft from the shared lm_head when want_draft. */
static uint32_t mtp_row(OState *s, uint32_t tok, const float *h, float *hout, int want_draft) {
    OModel *m = s->m;
    const int H = m->hidden;
    float *e = (float *)malloc((size_t)H * 4), *cat = (float *)malloc((size_t)2 * H * 4), *u = (float *)malloc((size_t)H * 4);
    float *yy = (float *)malloc((size_t)H * 4);
    embed_row(m, tok, e);
    oracle_rmsnorm(e, m->enorm, H, m->eps, cat);
    oracle_rmsnorm(h, m->hnorm, H, m->eps, cat + H);
    matvec(&m->eh_proj, cat, u);
    layer_token(m, &m->mtp_block, NULL, s->mtpK, s->mtpV, s->mtp_len, u, yy);
    oracle_rmsnorm(yy, m->head_norm, H, m->eps, hout);
    s->mtp_len++;
    uint32_t d = 0;
    if (want_draft) {
        float *lg = (float *)malloc((size_t)m->vocab * 4);
        matvec(&m->lm_head, hout, lg);
        d = oracle_argmax(lg, m->vocab);
        free(lg);
    }
    free(e); free(cat); free(u); free(yy);
    return d;
}

static int is_stop(OModel *m, uint32_t id) { return id == m->eos || id == m->stop2; }

/* The plain greedy loop (crates/cli/src/run.rs:329-350): prefill the prompt, then one token per step;
 * stops after a stop id when `stop` is set.  Returns the number of ids written. */
/* smp (optional): the sampler; greedy (argmax) without one or at temperature <= 0, else sample() on every
 * token (run.rs:313-318, :348) */
int oracle_generate_s(OState *s, const uint32_t *prompt, int n, int n_out, int stop, OSampler *smp, uint32_t *out) {
    OModel *m = s->m;
    float *lg = (float *)malloc((size_t)m->vocab * 4);
    const int greedy = !smp || oracle_sampler_greedy(smp);
    if (prefill_rows(s, prompt, n, lg, NULL)) { free(lg); return -1; }  /* batched, as Model::prefill */
    int c = 0;
    out[c++] = greedy ? oracle_argmax(lg, m->vocab) : oracle_sampler_sample(smp, lg);
    while (c < n_out && !(stop && is_stop(m, out[c - 1]))) {
        if (oracle_forward_token(s, out[c - 1], lg, NULL, NULL)) break;
        out[c++] = greedy ? oracle_argmax(lg, m->vocab) : oracle_sampler_sample(smp, lg);
    }
    free(lg);
    return c;
}

int oracle_generate(OState *s, const uint32_t *prompt, int n, int n_out, int stop, uint32_t *out) {
    return oracle_generate_s(s, prompt, n, n_out, stop, NULL, out);
}

/* The --spec k loop (spec.rs:229-433, run.rs:353-383), greedy: spec_prefill, then rounds of verify
 * [x_p, d_1..d_k] (token by token on the snapshot), accept, restore + replay of the kept rows, MTP re-feed,
 * chained drafts.  forced_drafts (optional, n_forced_rounds x k) replaces the MTP drafts of the first rounds,
 * as spec_set_drafts does in the reference's identity test.  stats4 = rounds, drafted, accepted, emitted. */
static double g_round_seconds = 0.0;  /* wall time the last oracle_spec_generate spent in its rounds */

double oracle_last_round_seconds(void) { return g_round_seconds; }

static double now_s(void) {
    struct timespec ts;
    clock_gettime(CLOCK_MONOTONIC, &ts);
    return (double)ts.tv_sec + 1e-9 * (double)ts.tv_nsec;
}

/* One draft from the MTP's post-norm row hout through the shared lm_head (spec.rs:190-203): greedy argmax, or
 * process + draw with the processed distribution written densely to q_dense (the acceptance rule's q). */
static uint32_t draft_token(OState *s, OSampler *smp, const float *hout, float *q_dense) {
    OModel *m = s->m;
    float *lg = (float *)malloc((size_t)m->vocab * 4);
    matvec(&m->lm_head, hout, lg);
    uint32_t d;
    if (!smp || oracle_sampler_greedy(smp)) {
        d = oracle_argmax(lg, m->vocab);
    } else {
        oracle_sampler_process(smp, lg, NULL, NULL);
        d = oracle_sampler_draw(smp);
        oracle_sampler_write_dense(smp, q_dense);
    }
    free(lg);
    return d;
}

int oracle_spec_generate_s(OState *s, const uint32_t *prompt, int n, int n_out, int k, int stop, const uint32_t *forced,
                           int n_forced, OSampler *smp, uint32_t *out, uint64_t *stats4, uint32_t *drafts_log);

int oracle_spec_generate(OState *s, const uint32_t *prompt, int n, int n_out, int k, int stop, const uint32_t *forced,
                         int n_forced, uint32_t *out, uint64_t *stats4, uint32_t *drafts_log) {
    return oracle_spec_generate_s(s, prompt, n, n_out, k, stop, forced, n_forced, NULL, out, stats4, drafts_log);
}

int oracle_spec_generate_s(OState *s, const uint32_t *prompt, int n, int n_out, int k, int stop, const uint32_t *forced,
                           int n_forced, OSampler *smp, uint32_t *out, uint64_t *stats4, uint32_t *drafts_log) {
    OModel *m = s->m;
    const int H = m->hidden, t = k + 1;
    if (!m->has_mtp || k < 1 || k + 1 > MAXT) return -1;
    const int greedy = !smp || oracle_sampler_greedy(smp);
    float *q_dense = greedy ? NULL : (float *)malloc((size_t)m->vocab * 4 * k);
    float *lg = (float *)malloc((size_t)m->vocab * 4 * t);
    float *normed = (float *)malloc((size_t)H * 4 * (n > t ? n : t));
    float *hout = (float *)malloc((size_t)H * 4), *hprev = (float *)malloc((size_t)H * 4);
    uint32_t *drafts = (uint32_t *)malloc(sizeof(uint32_t) * k), *emitted = (uint32_t *)malloc(sizeof(uint32_t) * t);
    int c = 0, round = 0;
    /* spec_prefill (spec.rs:229-285): the batched prefill, x_T, the MTP over the prompt rows (x_{j+1}, h_j) */
    int p = s->pos;
    if (prefill_rows(s, prompt, n, lg, normed)) goto fail;
    uint32_t x_t = greedy ? oracle_argmax(lg, m->vocab) : oracle_sampler_sample(smp, lg);
    s->mtp_len = p;
    {
        uint32_t xs[MAXB];
        float *ho = (float *)malloc((size_t)MAXB * H * 4);
        for (int off = 0; off < n; off += MAXB) {
            const int tt = n - off < MAXB ? n - off : MAXB;
            for (int j = 0; j < tt; j++) xs[j] = (off + j + 1 < n) ? prompt[off + j + 1] : x_t;
            mtp_rows_batch(s, xs, normed + (size_t)off * H, tt, ho);
            if (off + tt == n) memcpy(hout, ho + (size_t)(tt - 1) * H, (size_t)H * 4);
        }
        free(ho);
    }
    drafts[0] = draft_token(s, smp, hout, q_dense);
    for (int i = 1; i < k; i++) {
        memcpy(hprev, hout, (size_t)H * 4);
        mtp_row(s, drafts[i - 1], hprev, hout, 0);
        drafts[i] = draft_token(s, smp, hout, q_dense ? q_dense + (size_t)i * m->vocab : NULL);
    }
    out[c++] = x_t;
    uint32_t x_p = x_t;
    const double t_rounds = now_s();
    while (c < n_out && !(stop && is_stop(m, out[c - 1]))) {
        if (forced && round < n_forced) memcpy(drafts, forced + (size_t)round * k, sizeof(uint32_t) * k);
        if (drafts_log) memcpy(drafts_log + (size_t)round * k, drafts, sizeof(uint32_t) * k);
        p = s->pos;
        if (p + t > s->max_pos) break;
        float *snap = snapshot(s);
        uint32_t batch[MAXT];
        batch[0] = x_p;
        for (int i = 0; i < k; i++) batch[i + 1] = drafts[i];
        /* the verify: the t rows in one batched forward (spec.rs:337-350) */
        if (forward_rows(s, batch, t, lg, t, normed)) { free(snap); break; }
        int mm = 0, ne = 0;
        if (greedy) {
            while (mm < k) {
                uint32_t a = oracle_argmax(lg + (size_t)mm * m->vocab, m->vocab);
                emitted[ne++] = a;
                if (a != drafts[mm]) break;
                mm++;
            }
            if (mm == k) emitted[ne++] = oracle_argmax(lg + (size_t)k * m->vocab, m->vocab);
        } else {  /* spec.rs:367-379: accept_or_resample per position, then the bonus draw */
            while (mm < k) {
                uint32_t tok;
                const int ok = oracle_sampler_accept(smp, lg + (size_t)mm * m->vocab, q_dense + (size_t)mm * m->vocab,
                                                     drafts[mm], &tok);
                emitted[ne++] = tok;
                if (!ok) break;
                mm++;
            }
            if (mm == k) {
                oracle_sampler_process(smp, lg + (size_t)k * m->vocab, NULL, NULL);
                emitted[ne++] = oracle_sampler_draw(smp);
            }
        }
        int keep = mm + 1;
        if (keep < t) {
            /* spec.rs:395-415: restore the DeltaNet snapshot and replay the kept rows' recurrence (conv + delta
             * rule) from the verify's saved projections -- the states after `keep` rows, bit for bit, with no
             * second pass over the weights; the KV caches end at p + keep */
            restore(s, snap);
            for (int l = 0; l < m->n_layer; l++) {
                if (m->layers[l].attn) continue;
                OLayerState *ls = &s->ls[l];
                for (int i = 0; i < keep; i++)
                    deltanet_recur(m, &m->layers[l], ls, ls->sv_mixed + (size_t)i * m->conv_dim, ls->sv_z + (size_t)i * m->vd,
                                   ls->sv_ga + (size_t)i * m->n_v, ls->sv_gb + (size_t)i * m->n_v, NULL);
            }
            s->pos = p + keep;
        }
        free(snap);
        if (stats4) { stats4[0]++; stats4[1] += k; stats4[2] += mm; stats4[3] += keep; }
        /* the MTP: truncate to p, re-feed the kept pairs (emitted_i, normed_i), draft, chain */
        s->mtp_len = p;
        {
            float *ho = (float *)malloc((size_t)t * H * 4);
            mtp_rows_batch(s, emitted, normed, keep, ho);  /* the re-feed rows in one batch (mtp.rs rows_in) */
            memcpy(hout, ho + (size_t)(keep - 1) * H, (size_t)H * 4);
            free(ho);
        }
        drafts[0] = draft_token(s, smp, hout, q_dense);
        for (int i = 1; i < k; i++) {
            memcpy(hprev, hout, (size_t)H * 4);
            mtp_row(s, drafts[i - 1], hprev, hout, 0);
            drafts[i] = draft_token(s, smp, hout, q_dense ? q_dense + (size_t)i * m->vocab : NULL);
        }
        for (int i = 0; i < keep && c < n_out; i++) {
            out[c++] = emitted[i];
            if (stop && is_stop(m, emitted[i])) break;
        }
        x_p = emitted[keep - 1];
        round++;
    }
    g_round_seconds = now_s() - t_rounds;
    free(lg); free(normed); free(hout); free(hprev); free(drafts); free(emitted); free(q_dense);
    return c;
fail:
    free(lg); free(normed); free(hout); free(hprev); free(drafts); free(emitted); free(q_dense);
    return -1;
}

int oracle_state_pos(OState *s) { return s->pos; }

/* ------------------------------------------------------------------------- carried state, for the tests */

/* The carried state of layer `layer` (spec_identity.rs:5-9 compares it after every round): what = 0 the DeltaNet
 * recurrent state f32 [n_v][dk][dv], 1 its conv window f32 [conv_dim][conv_k - 1], 2 / 3 the attention K / V
 * cache rows [0, pos) f32 [pos][n_kv * head_dim].  Returns the number of floats written (0: not this kind of
 * layer), or the number needed when out is NULL. */
long oracle_state_get(OState *s, int layer, int what, float *out) {
    OModel *m = s->m;
    if (layer < 0 || layer >= m->n_layer) return -1;
    const OLayer *L = &m->layers[layer];
    const OLayerState *ls = &s->ls[layer];
    size_t n = 0;
    const float *src = NULL;
    if (!L->attn && what == 0) { n = (size_t)m->n_v * m->dk * m->dv; src = ls->S; }
    else if (!L->attn && what == 1) { n = (size_t)m->conv_dim * (m->conv_k - 1); src = ls->conv; }
    else if (L->attn && (what == 2 || what == 3)) { n = (size_t)s->pos * m->n_kv * m->hd; src = what == 2 ? ls->K : ls->V; }
    if (out && n) memcpy(out, src, n * 4);
    return (long)n;
}

/* --------------------------------------------------------------- one layer on caller-held F32 weights */

/* The reference checks its layer code against HF module outputs on F32 weights (crates/core/tests/layers.rs:
 * WeightMat::from_f32, a prefill of t rows, then one step on the carried state / KV cache).  This runs the
 * oracle's own layer functions -- the ones oracle_forward_token uses -- on such weights, row by row from
 * position pos0.  dims = {hidden, ffn, n_head, n_kv, head_dim, rope_dim, conv_kernel, dk, n_k, n_v, dv},
 * fdims = {eps, theta}, w = OW_COUNT weight pointers (oracle.h; the ones a kind does not use may be NULL).
 * State in and out: S [n_v][dk][dv] and conv [conv_dim][conv_kernel - 1] (DeltaNet kinds), K and V
 * [pos][n_kv * head_dim] (attention kinds, rows pos0 .. pos0 + t - 1 written).  y: t rows of hidden. */
int oracle_layer_f32(const int *dims, const float *fdims, const float *const *w, int kind, const float *x, int t,
                     int pos0, float *S, float *conv, float *K, float *V, float *y) {
    OModel m;
    memset(&m, 0, sizeof m);
    m.hidden = dims[0]; m.ffn = dims[1]; m.n_head = dims[2]; m.n_kv = dims[3]; m.hd = dims[4]; m.rope_dim = dims[5];
    m.conv_k = dims[6]; m.dk = dims[7]; m.n_k = dims[8]; m.n_v = dims[9]; m.dv = dims[10];
    m.eps = fdims[0];
    m.theta = fdims[1];
    m.kd = m.n_k * m.dk;
    m.vd = m.n_v * m.dv;
    m.conv_dim = 2 * m.kd + m.vd;
    m.scaling = m.hd > 0 ? powf((float)m.hd, -0.5f) : 0.0f;
    OLayer L;
    memset(&L, 0, sizeof L);
#define FMAT(field, idx, r, c) do { L.field.type = OT_F32; L.field.rows = (r); L.field.cols = (c); L.field.data = (const uint8_t *)w[idx]; } while (0)
    L.attn_norm = w[OW_ATTN_NORM];
    L.post_norm = w[OW_POST_NORM];
    FMAT(qkv, OW_QKV, m.conv_dim, m.hidden);
    FMAT(gate_z, OW_GATE_Z, m.vd, m.hidden);
    FMAT(alpha, OW_ALPHA, m.n_v, m.hidden);
    FMAT(beta, OW_BETA, m.n_v, m.hidden);
    L.ssm_a = w[OW_SSM_A];
    L.dt_bias = w[OW_DT_BIAS];
    L.conv_w = w[OW_CONV];
    L.ssm_norm = w[OW_SSM_NORM];
    FMAT(ssm_out, OW_SSM_OUT, m.hidden, m.vd);
    FMAT(q, OW_Q, 2 * m.n_head * m.hd, m.hidden);
    FMAT(k, OW_K, m.n_kv * m.hd, m.hidden);
    FMAT(v, OW_V, m.n_kv * m.hd, m.hidden);
    FMAT(o, OW_O, m.hidden, m.n_head * m.hd);
    L.q_norm = w[OW_Q_NORM];
    L.k_norm = w[OW_K_NORM];
    FMAT(gate, OW_FFN_GATE, m.ffn, m.hidden);
    FMAT(up, OW_FFN_UP, m.ffn, m.hidden);
    FMAT(down, OW_FFN_DOWN, m.hidden, m.ffn);
#undef FMAT
    OLayerState st = {S, conv, K, V, NULL, NULL, NULL, NULL};
    L.attn = kind == OL_ATTENTION || kind == OL_DECODER_ATTENTION;
    const size_t H = (size_t)m.hidden;
    for (int i = 0; i < t; i++) {
        const float *xi = x + (size_t)i * H;
        float *yi = y + (size_t)i * H;
        switch (kind) {
        case OL_DELTANET: deltanet_token(&m, &L, &st, xi, yi); break;
        case OL_ATTENTION: attention_token(&m, &L, K, V, pos0 + i, xi, yi); break;
        case OL_MLP: mlp_token(&m, &L, xi, yi); break;
        case OL_DECODER_DELTANET:
        case OL_DECODER_ATTENTION: layer_token(&m, &L, &st, K, V, pos0 + i, xi, yi); break;
        default: return -1;
        }
    }
    return 0;
}
