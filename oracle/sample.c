/* CPU oracle (test infrastructure, never the product path): the reference's sampler restated in C.
 *
 *   crates/core/src/sample.rs:14-55   the RNG: xoshiro256** (Blackman & Vigna 2018) seeded by splitmix64;
 *                                     f32() = (next >> 40) * 2^-24, a uniform in [0, 1) with 24 random bits
 *   crates/core/src/sample.rs:182-243 process(): candidates = the top-k by logit (ties: the lower id first),
 *                                     or the whole vocabulary, sorted descending; softmax at the temperature
 *                                     (sum left to right in that order); top-p (keep while the mass above is
 *                                     below top_p, the crossing token stays, at least one); min-p (drop below
 *                                     min_p x the top probability); renormalise the kept set
 *   crates/core/src/sample.rs:246-257 draw(): the first kept candidate whose running mass exceeds u
 *   crates/core/src/sample.rs:279-313 accept_or_resample(): accept d with probability min(1, p(d) / q(d)),
 *                                     else draw from norm(max(0, p - q)) over the kept set of p
 *
 * Pinned by tests/test_oracle_golden.py against the reference's own sampler tests (sample.rs:492-529).
 * exp is oracle_expf (the oracle's libm convention).  NaN logits are outside the contract (the reference's
 * comparator treats NaN as equal to everything; its order is then not total).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include "oracle.h"

static uint64_t rotl(uint64_t x, int k) { return (x << k) | (x >> (64 - k)); }

void oracle_rng_seed(uint64_t s_out[4], uint64_t seed) {
    uint64_t x = seed;
    for (int i = 0; i < 4; i++) {
        x += 0x9E3779B97F4A7C15ull;
        uint64_t z = x;
        z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
        z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
        s_out[i] = z ^ (z >> 31);
    }
}

uint64_t oracle_rng_next(uint64_t s[4]) {
    const uint64_t result = rotl(s[1] * 5, 7) * 9;
    const uint64_t t = s[1] << 17;
    s[2] ^= s[0];
    s[3] ^= s[1];
    s[1] ^= s[2];
    s[0] ^= s[3];
    s[2] ^= t;
    s[3] = rotl(s[3], 45);
    return result;
}

float oracle_rng_f32(uint64_t s[4]) { return (float)(oracle_rng_next(s) >> 40) * (1.0f / 16777216.0f); }

struct oracle_sampler {
    OSamplerCfg cfg;
    uint64_t rng[4];
    int vocab, n;
    uint32_t *idx;
    float *probs;
};

OSampler *oracle_sampler_new(const OSamplerCfg *cfg, int vocab) {
    OSampler *s = (OSampler *)calloc(1, sizeof(OSampler));
    s->cfg = *cfg;
    s->vocab = vocab;
    s->idx = (uint32_t *)malloc(sizeof(uint32_t) * (size_t)vocab);
    s->probs = (float *)malloc(sizeof(float) * (size_t)vocab);
    oracle_rng_seed(s->rng, cfg->seed);
    return s;
}

void oracle_sampler_free(OSampler *s) {
    if (!s) return;
    free(s->idx);
    free(s->probs);
    free(s);
}

int oracle_sampler_greedy(const OSampler *s) { return s->cfg.temperature <= 0.0f; }

static const float *g_sort_logits;
static int by_logit_desc(const void *pa, const void *pb) {
    const uint32_t a = *(const uint32_t *)pa, b = *(const uint32_t *)pb;
    const float la = g_sort_logits[a], lb = g_sort_logits[b];
    if (lb > la) return 1;  /* b first */
    if (lb < la) return -1;
    return a < b ? -1 : (a > b ? 1 : 0);
}

int oracle_sampler_process(OSampler *s, const float *logits, uint32_t *ids_out, float *probs_out) {
    const int vocab = s->vocab;
    const OSamplerCfg *c = &s->cfg;
    if (c->temperature <= 0.0f) {
        s->idx[0] = oracle_argmax(logits, vocab);
        s->probs[0] = 1.0f;
        s->n = 1;
    } else {
        for (int i = 0; i < vocab; i++) s->idx[i] = (uint32_t)i;
        const int n_cand = (c->top_k > 0 && c->top_k < vocab) ? c->top_k : vocab;
        /* a full sort by (logit desc, id asc): its prefix is the reference's select_nth + sort of the top-k */
        g_sort_logits = logits;
        qsort(s->idx, (size_t)vocab, sizeof(uint32_t), by_logit_desc);
        const float inv_t = 1.0f / c->temperature;
        const float m = logits[s->idx[0]] * inv_t;
        float sum = 0.0f;
        for (int i = 0; i < n_cand; i++) {
            const float e = oracle_expf(logits[s->idx[i]] * inv_t - m);
            s->probs[i] = e;
            sum += e;
        }
        for (int i = 0; i < n_cand; i++) s->probs[i] /= sum;
        int n = n_cand;
        if (c->top_p < 1.0f) {
            float cum = 0.0f;
            n = 0;
            while (n < n_cand && cum < c->top_p) {
                cum += s->probs[n];
                n++;
            }
            if (n < 1) n = 1;
        }
        if (c->min_p > 0.0f) {
            const float thr = c->min_p * s->probs[0];
            int keep = 1;
            while (keep < n && s->probs[keep] >= thr) keep++;
            n = keep;
        }
        float t = 0.0f;
        for (int i = 0; i < n; i++) t += s->probs[i];
        for (int i = 0; i < n; i++) s->probs[i] /= t;
        s->n = n;
    }
    if (ids_out) memcpy(ids_out, s->idx, sizeof(uint32_t) * (size_t)s->n);
    if (probs_out) memcpy(probs_out, s->probs, sizeof(float) * (size_t)s->n);
    return s->n;
}

uint32_t oracle_sampler_draw(OSampler *s) {
    const float u = oracle_rng_f32(s->rng);
    float cum = 0.0f;
    for (int i = 0; i < s->n; i++) {
        cum += s->probs[i];
        if (u < cum) return s->idx[i];
    }
    return s->idx[s->n - 1];
}

uint32_t oracle_sampler_sample(OSampler *s, const float *logits) { /* sample.rs:260-263: process, then draw */
    oracle_sampler_process(s, logits, NULL, NULL);
    return oracle_sampler_draw(s);
}

/* q_dense: the draft's processed distribution, dense over the vocabulary (write_dense, sample.rs:266-275) */
int oracle_sampler_accept(OSampler *s, const float *target_logits, const float *q_dense, uint32_t d, uint32_t *tok_out) {
    oracle_sampler_process(s, target_logits, NULL, NULL);
    if (oracle_sampler_greedy(s)) {
        *tok_out = s->idx[0];
        return s->idx[0] == d;
    }
    float pd = 0.0f;
    for (int i = 0; i < s->n; i++)
        if (s->idx[i] == d) {
            pd = s->probs[i];
            break;
        }
    const float qd = q_dense[d];
    const float u = oracle_rng_f32(s->rng);
    if (qd > 0.0f && (pd >= qd || u < pd / qd)) {
        *tok_out = d;
        return 1;
    }
    float sum = 0.0f;
    for (int i = 0; i < s->n; i++) {
        const float r = fmaxf(s->probs[i] - q_dense[s->idx[i]], 0.0f);
        s->probs[i] = r;
        sum += r;
    }
    if (sum <= 0.0f) {
        oracle_sampler_process(s, target_logits, NULL, NULL);
        *tok_out = oracle_sampler_draw(s);
        return 0;
    }
    for (int i = 0; i < s->n; i++) s->probs[i] /= sum;
    *tok_out = oracle_sampler_draw(s);
    return 0;
}

void oracle_sampler_write_dense(const OSampler *s, float *out) {
    memset(out, 0, sizeof(float) * (size_t)s->vocab);
    for (int i = 0; i < s->n; i++) out[s->idx[i]] = s->probs[i];
}
