// Synthetic Qwen3.8-style GGUF checkpoints (the stand-in for the real 17.8 GB file, which is not available):
// the qwen35 metadata keys that crates/core/src/config.rs:146-260 requires, dummy vocabulary strings, and
// seeded random weights ~ N(0, 0.02) quantised by a simple K-quant encoder into the per-role type recipe of
// bartowski's Q4_K_M file (llama.cpp's "use more bits" rule: Q6_K on attn_qkv, on half of ffn_down and of
// attn_q/attn_v, Q8_0 on half of ssm_out, Q5_K on attn_k/attn_output, Q4_0 on the MTP block, F32 vectors).
//
// Every value is a pure function of (seed, tensor index, block index), so the file is identical for any
// thread count and the oracle and the engine read the same bytes.
#include "synth.h"

#include <fcntl.h>
#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <thread>
#include <vector>

#include "gguf.h"

namespace qdec {

namespace {

// ------------------------------------------------------------------------------------------- seeded RNG

inline uint64_t mix64(uint64_t z) {  // splitmix64 finaliser
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

struct Rng {
    uint64_t s;
    float spare = 0.f;
    bool has_spare = false;
    explicit Rng(uint64_t seed, uint64_t a, uint64_t b) : s(mix64(seed ^ mix64(a * 0x100000001B3ull ^ mix64(b)))) {}
    uint64_t next() { return s = mix64(s); }
    double uniform() { return ((next() >> 11) + 0.5) * (1.0 / 9007199254740992.0); }  // (0, 1)
    float normal() {  // Box-Muller in f32, two values per pair of uniforms
        if (has_spare) {
            has_spare = false;
            return spare;
        }
        const uint64_t r = next();
        const float u1 = ((float)(r >> 40) + 0.5f) * (1.0f / 16777216.0f);
        const float u2 = (float)((r >> 16) & 0xffffff) * (1.0f / 16777216.0f);
        const float rad = sqrtf(-2.0f * logf(u1));
        float sn, cs;
        sincosf(6.2831853f * u2, &sn, &cs);
        spare = rad * sn;
        has_spare = true;
        return rad * cs;
    }
};

inline uint16_t f16_rn(float f) {
    // round-to-nearest-even f32 -> f16 (finite inputs in range here)
    uint32_t x;
    memcpy(&x, &f, 4);
    const uint32_t sign = (x >> 16) & 0x8000u;
    int e = (int)((x >> 23) & 0xff) - 127 + 15;
    uint32_t m = x & 0x7fffff;
    if (((x >> 23) & 0xff) == 0 && m == 0) return (uint16_t)sign;
    if (e >= 31) return (uint16_t)(sign | 0x7c00u);
    if (e <= 0) {
        if (e < -10) return (uint16_t)sign;
        m |= 0x800000u;
        const uint32_t sh = (uint32_t)(14 - e);
        uint32_t h = m >> sh;
        const uint32_t rem = m & ((1u << sh) - 1), mid = 1u << (sh - 1);
        if (rem > mid || (rem == mid && (h & 1))) h++;
        return (uint16_t)(sign | h);
    }
    uint32_t out = sign | ((uint32_t)e << 10) | (m >> 13);
    const uint32_t rem = m & 0x1fff;
    if (rem > 0x1000 || (rem == 0x1000 && (out & 1))) out++;
    return (uint16_t)out;
}
inline float f16_to_f32(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1f, m = h & 0x3ff, bits;
    if (e == 0) {
        if (m == 0) bits = sign;
        else {
            int k = -1;
            do { m <<= 1; k++; } while (!(m & 0x400));
            bits = sign | ((uint32_t)(112 - k) << 23) | ((m & 0x3ff) << 13);
        }
    } else if (e == 31) bits = sign | 0x7f800000u | (m << 13);
    else bits = sign | ((e + 112) << 23) | (m << 13);
    float f;
    memcpy(&f, &bits, 4);
    return f;
}
inline void put16(uint8_t *p, uint16_t v) { p[0] = v & 0xff; p[1] = v >> 8; }
inline int clampi(int v, int lo, int hi) { return v < lo ? lo : (v > hi ? hi : v); }
inline long lroundf_fast(float v) { return (long)(v + (v >= 0.f ? 0.5f : -0.5f)); }

// ------------------------------------------------------------------------------- block encoders

void enc_q4k_q5k(const float *x, uint8_t *b, bool q5) {
    const int levels = q5 ? 31 : 15;
    float scale[8], mins[8];
    for (int s = 0; s < 8; s++) {
        float mn = x[s * 32], mx = x[s * 32];
        for (int j = 1; j < 32; j++) mn = std::min(mn, x[s * 32 + j]), mx = std::max(mx, x[s * 32 + j]);
        if (mn > 0) mn = 0;
        scale[s] = (mx - mn) / levels;
        mins[s] = -mn;
    }
    const float ms = *std::max_element(scale, scale + 8), mm = *std::max_element(mins, mins + 8);
    const uint16_t dh = f16_rn(ms / 63.f), mh = f16_rn(mm / 63.f);
    const float d = f16_to_f32(dh), dmin = f16_to_f32(mh);
    int ls[8], lm[8];
    for (int s = 0; s < 8; s++) {
        ls[s] = d > 0 ? clampi((int)lroundf_fast(scale[s] / d), 0, 63) : 0;
        lm[s] = dmin > 0 ? clampi((int)lroundf_fast(mins[s] / dmin), 0, 63) : 0;
    }
    memset(b, 0, q5 ? 176 : 144);
    put16(b, dh);
    put16(b + 2, mh);
    uint8_t *q = b + 4;  // inverse of get_scale_min_k4 (crates/core/src/quant.rs:45-51)
    for (int j = 0; j < 8; j++) {
        if (j < 4) {
            q[j] = (uint8_t)ls[j];
            q[j + 4] = (uint8_t)lm[j];
        } else {
            q[j + 4] = (uint8_t)((ls[j] & 0xF) | ((lm[j] & 0xF) << 4));
            q[j - 4] |= (uint8_t)((ls[j] >> 4) << 6);
            q[j] |= (uint8_t)((lm[j] >> 4) << 6);
        }
    }
    for (int s = 0; s < 8; s++) {
        const float ds = d * ls[s], off = dmin * lm[s];
        for (int j = 0; j < 32; j++) {
            const int v = ds > 0 ? clampi((int)lroundf_fast((x[s * 32 + j] + off) / ds), 0, levels) : 0;
            if (!q5) {
                b[16 + (s / 2) * 32 + j] |= (uint8_t)((v & 0xF) << ((s & 1) * 4));
            } else {
                b[48 + (s / 2) * 32 + j] |= (uint8_t)((v & 0xF) << ((s & 1) * 4));
                if (v & 16) b[16 + j] |= (uint8_t)(1u << s);
            }
        }
    }
}

void enc_q6k(const float *x, uint8_t *b) {
    float sc[16];
    for (int g = 0; g < 16; g++) {
        float a = 0;
        for (int j = 0; j < 16; j++) a = std::max(a, std::fabs(x[g * 16 + j]));
        sc[g] = a / 31.f;
    }
    const float msc = *std::max_element(sc, sc + 16);
    const uint16_t dh = f16_rn(msc / 127.f);
    const float d = f16_to_f32(dh);
    memset(b, 0, 210);
    int8_t isc[16];
    for (int g = 0; g < 16; g++) isc[g] = (int8_t)(d > 0 ? clampi((int)lroundf_fast(sc[g] / d), -128, 127) : 0);
    for (int e = 0; e < 256; e++) {
        const int g = e / 16;
        const float ds = d * isc[g];
        const int v = ds != 0 ? clampi((int)lroundf_fast(x[e] / ds) + 32, 0, 63) : 32;
        const int h = e / 128, r = e % 128, k = r / 32, l = r % 32;
        b[h * 64 + l + 32 * (k & 1)] |= (uint8_t)((v & 0xF) << (4 * (k >> 1)));
        b[128 + h * 32 + l] |= (uint8_t)(((v >> 4) & 3) << (2 * k));
    }
    memcpy(b + 192, isc, 16);
    put16(b + 208, dh);
}

void enc_q8_0(const float *x, uint8_t *b) {
    float amax = 0;
    for (int j = 0; j < 32; j++) amax = std::max(amax, std::fabs(x[j]));
    const float d = amax / 127.f, id = d != 0 ? 1.f / d : 0.f;
    put16(b, f16_rn(d));
    for (int j = 0; j < 32; j++) b[2 + j] = (uint8_t)(int8_t)clampi((int)lroundf_fast(x[j] * id), -128, 127);
}

void enc_q4_0(const float *x, uint8_t *b) {
    float amax = 0, mx = 0;
    for (int j = 0; j < 32; j++)
        if (std::fabs(x[j]) > amax) amax = std::fabs(x[j]), mx = x[j];
    const float d = mx / -8.f, id = d != 0 ? 1.f / d : 0.f;
    put16(b, f16_rn(d));
    for (int j = 0; j < 16; j++) {
        const int lo = std::min(15, (int)(x[j] * id + 8.5f)), hi = std::min(15, (int)(x[j + 16] * id + 8.5f));
        b[2 + j] = (uint8_t)(clampi(lo, 0, 15) | (clampi(hi, 0, 15) << 4));
    }
}

// ----------------------------------------------------------------------------------- tensor recipe

enum Dist { D_MATRIX, D_NORM, D_SSM_A, D_DT_BIAS, D_CONV };

struct TSpec {
    std::string name;
    int type;
    std::vector<uint64_t> ne;  // GGUF order (ne0 = cols)
    Dist dist;
    uint64_t bytes = 0, off = 0;
};

// llama.cpp's Q4_K_M "use more bits" rule over the n layers of one role
bool more_bits(int i, int n) { return i < n / 8 || i >= 7 * n / 8 || (i - n / 8) % 3 == 2; }

struct Dims {
    uint32_t hidden, n_layer, ffn, vocab, n_head, n_kv, head_dim, rope_dim, interval;
    uint32_t dn_k_heads, dn_state, dn_v_heads, dn_inner, conv_kernel;
    std::vector<int32_t> rope_sections;
    std::string name;
};

bool preset(const std::string &p, Dims &d, std::string &err) {
    // "tiny": the reference's CPU-runnable toy (a few layers of small widths); "27b": docs/model-facts.md:26-76;
    // "27b-L<n>": the 27B dimensions with n layers (n a multiple of the attention interval), for parity runs.
    if (p == "tiny") {
        d = {256, 4, 768, 4096, 4, 2, 64, 16, 4, 2, 64, 4, 256, 4, {3, 3, 2, 0}, "Qwen3.8 tiny synthetic"};
        return true;
    }
    if (p == "27b" || p.rfind("27b-L", 0) == 0) {
        d = {5120, 64, 17408, 248320, 24, 4, 256, 64, 4, 16, 128, 48, 6144, 4, {11, 11, 10, 0}, "Qwen3.8 27B synthetic"};
        if (p != "27b") {
            const int n = atoi(p.c_str() + 5);
            if (n <= 0 || n % 4) { err = "27b-L<n> needs n a positive multiple of 4"; return false; }
            d.n_layer = (uint32_t)n;
        }
        return true;
    }
    err = "unknown preset '" + p + "' (tiny, 27b, 27b-L<n>)";
    return false;
}

std::vector<TSpec> recipe(const Dims &d) {
    std::vector<TSpec> ts;
    const uint64_t H = d.hidden;
    auto mat = [&](const std::string &n, int t, uint64_t rows, uint64_t cols) { ts.push_back({n, t, {cols, rows}, D_MATRIX}); };
    auto vec = [&](const std::string &n, uint64_t len, Dist dist) { ts.push_back({n, 0, {len}, dist}); };
    mat("output.weight", 14, d.vocab, H);
    vec("output_norm.weight", H, D_NORM);
    mat("token_embd.weight", 12, d.vocab, H);
    const uint32_t kd = d.dn_k_heads * d.dn_state, vd = d.dn_inner, conv_dim = 2 * kd + vd;
    int n_attn = 0, n_dn = 0;
    for (uint32_t i = 0; i < d.n_layer; i++) ((i + 1) % d.interval == 0 ? n_attn : n_dn)++;
    int ai = 0, di = 0;
    for (uint32_t i = 0; i < d.n_layer; i++) {
        const std::string p = "blk." + std::to_string(i) + ".";
        if ((i + 1) % d.interval == 0) {
            const bool more = more_bits(ai++, n_attn);
            mat(p + "attn_k.weight", 13, (uint64_t)d.n_kv * d.head_dim, H);
            vec(p + "attn_k_norm.weight", d.head_dim, D_NORM);
            vec(p + "attn_norm.weight", H, D_NORM);
            mat(p + "attn_output.weight", 13, H, (uint64_t)d.n_head * d.head_dim);
            mat(p + "attn_q.weight", more ? 14 : 12, 2ull * d.n_head * d.head_dim, H);
            vec(p + "attn_q_norm.weight", d.head_dim, D_NORM);
            mat(p + "attn_v.weight", more ? 14 : 12, (uint64_t)d.n_kv * d.head_dim, H);
        } else {
            const bool more = more_bits(di++, n_dn);
            mat(p + "attn_gate.weight", 12, vd, H);
            vec(p + "attn_norm.weight", H, D_NORM);
            mat(p + "attn_qkv.weight", 14, conv_dim, H);
            vec(p + "ssm_a", d.dn_v_heads, D_SSM_A);
            mat(p + "ssm_alpha.weight", 0, d.dn_v_heads, H);
            mat(p + "ssm_beta.weight", 0, d.dn_v_heads, H);
            ts.push_back({p + "ssm_conv1d.weight", 0, {d.conv_kernel, conv_dim}, D_CONV});
            vec(p + "ssm_dt.bias", d.dn_v_heads, D_DT_BIAS);
            vec(p + "ssm_norm.weight", vd / d.dn_v_heads, D_NORM);
            mat(p + "ssm_out.weight", more ? 8 : 12, H, vd);
        }
        mat(p + "ffn_down.weight", more_bits((int)i, (int)d.n_layer) ? 14 : 12, H, d.ffn);
        mat(p + "ffn_gate.weight", 12, d.ffn, H);
        mat(p + "ffn_up.weight", 12, d.ffn, H);
        vec(p + "post_attention_norm.weight", H, D_NORM);
    }
    // the MTP block blk.{n_layer}: one attention decoder layer, all matrices Q4_0 (docs/mtp.md:29)
    const std::string p = "blk." + std::to_string(d.n_layer) + ".";
    mat(p + "attn_k.weight", 2, (uint64_t)d.n_kv * d.head_dim, H);
    vec(p + "attn_k_norm.weight", d.head_dim, D_NORM);
    vec(p + "attn_norm.weight", H, D_NORM);
    mat(p + "attn_output.weight", 2, H, (uint64_t)d.n_head * d.head_dim);
    mat(p + "attn_q.weight", 2, 2ull * d.n_head * d.head_dim, H);
    vec(p + "attn_q_norm.weight", d.head_dim, D_NORM);
    mat(p + "attn_v.weight", 2, (uint64_t)d.n_kv * d.head_dim, H);
    mat(p + "ffn_down.weight", 2, H, d.ffn);
    mat(p + "ffn_gate.weight", 2, d.ffn, H);
    mat(p + "ffn_up.weight", 2, d.ffn, H);
    mat(p + "nextn.eh_proj.weight", 2, H, 2 * H);
    vec(p + "nextn.enorm.weight", H, D_NORM);
    vec(p + "nextn.hnorm.weight", H, D_NORM);
    vec(p + "nextn.shared_head_norm.weight", H, D_NORM);
    vec(p + "post_attention_norm.weight", H, D_NORM);
    return ts;
}

// ------------------------------------------------------------------------------------------ writer

struct Buf {
    std::vector<uint8_t> b;
    void u32(uint32_t v) { const uint8_t *p = (const uint8_t *)&v; b.insert(b.end(), p, p + 4); }
    void u64(uint64_t v) { const uint8_t *p = (const uint8_t *)&v; b.insert(b.end(), p, p + 8); }
    void f32(float v) { const uint8_t *p = (const uint8_t *)&v; b.insert(b.end(), p, p + 4); }
    void str(const std::string &s) { u64(s.size()); b.insert(b.end(), s.begin(), s.end()); }
    void key(const std::string &k, uint32_t t) { str(k); u32(t); }
};

float draw(Dist dist, Rng &r) {
    switch (dist) {
    case D_MATRIX: return 0.02f * r.normal();
    case D_NORM: return 1.0f + 0.1f * r.normal();
    case D_SSM_A: return -std::exp((float)(2.0 * r.uniform() - 1.0));
    case D_DT_BIAS: return 0.5f * r.normal();
    case D_CONV: return 0.1f * r.normal();
    }
    return 0;
}

}  // namespace

void synth_gguf(const std::string &path, const std::string &preset_name, uint64_t seed, int threads) {
    Dims d;
    std::string err;
    if (!preset(preset_name, d, err)) throw std::invalid_argument(err);
    std::vector<TSpec> ts = recipe(d);
    const uint64_t align = 32;
    Buf h;
    h.u32(0x46554747u);
    h.u32(3);
    h.u64(ts.size());
    const uint32_t eos = d.vocab >= 248320 ? 248046 : d.vocab - 1, pad = d.vocab >= 248320 ? 248044 : d.vocab - 2;
    int n_kv = 0;
    Buf kv;
    auto kv_u32 = [&](const std::string &k, uint32_t v) { kv.key(k, 4); kv.u32(v); n_kv++; };
    auto kv_f32 = [&](const std::string &k, float v) { kv.key(k, 6); kv.f32(v); n_kv++; };
    auto kv_str = [&](const std::string &k, const std::string &v) { kv.key(k, 8); kv.str(v); n_kv++; };
    kv_str("general.architecture", "qwen35");
    kv_str("general.name", d.name);
    kv_u32("general.alignment", (uint32_t)align);
    kv_u32("qwen35.block_count", d.n_layer + 1);
    kv_u32("qwen35.context_length", 262144);
    kv_u32("qwen35.embedding_length", d.hidden);
    kv_u32("qwen35.feed_forward_length", d.ffn);
    kv_u32("qwen35.attention.head_count", d.n_head);
    kv_u32("qwen35.attention.head_count_kv", d.n_kv);
    kv.key("qwen35.rope.dimension_sections", 9);
    kv.u32(5);
    kv.u64(d.rope_sections.size());
    for (int32_t s : d.rope_sections) kv.u32((uint32_t)s);
    n_kv++;
    kv_f32("qwen35.rope.freq_base", 1.0e7f);
    kv_f32("qwen35.attention.layer_norm_rms_epsilon", 1e-6f);
    kv_u32("qwen35.attention.key_length", d.head_dim);
    kv_u32("qwen35.attention.value_length", d.head_dim);
    kv_u32("qwen35.nextn_predict_layers", 1);
    kv_u32("qwen35.ssm.conv_kernel", d.conv_kernel);
    kv_u32("qwen35.ssm.state_size", d.dn_state);
    kv_u32("qwen35.ssm.group_count", d.dn_k_heads);
    kv_u32("qwen35.ssm.time_step_rank", d.dn_v_heads);
    kv_u32("qwen35.ssm.inner_size", d.dn_inner);
    kv_u32("qwen35.full_attention_interval", d.interval);
    kv_u32("qwen35.rope.dimension_count", d.rope_dim);
    kv_str("tokenizer.ggml.model", "gpt2");
    kv_str("tokenizer.ggml.pre", "qwen35");
    kv.key("tokenizer.ggml.tokens", 9);
    kv.u32(8);
    kv.u64(d.vocab);
    for (uint32_t i = 0; i < d.vocab; i++) kv.str("<t" + std::to_string(i) + ">");
    n_kv++;
    kv_u32("tokenizer.ggml.eos_token_id", eos);
    kv_u32("tokenizer.ggml.padding_token_id", pad);
    kv_u32("tokenizer.ggml.bos_token_id", pad);
    kv.key("tokenizer.ggml.add_bos_token", 7);
    kv.b.push_back(0);
    n_kv++;
    kv_u32("general.quantization_version", 2);
    kv_u32("general.file_type", 15);
    kv.key("qdec.synth.seed", 10);
    kv.u64(seed);
    n_kv++;
    kv_str("qdec.synth.preset", preset_name);
    h.u64((uint64_t)n_kv);
    h.b.insert(h.b.end(), kv.b.begin(), kv.b.end());
    uint64_t off = 0;
    for (TSpec &t : ts) {
        uint64_t n = 1;
        for (uint64_t e : t.ne) n *= e;
        auto lay = ggml_block_layout(t.type);
        t.bytes = n / lay.first * lay.second;
        t.off = off;
        off = (off + t.bytes + align - 1) / align * align;
        h.str(t.name);
        h.u32((uint32_t)t.ne.size());
        for (uint64_t e : t.ne) h.u64(e);
        h.u32((uint32_t)t.type);
        h.u64(t.off);
    }
    const uint64_t data_off = (h.b.size() + align - 1) / align * align;
    h.b.resize(data_off, 0);
    const uint64_t total = data_off + off;

    const int fd = ::open(path.c_str(), O_WRONLY | O_CREAT | O_TRUNC | O_CLOEXEC, 0644);
    if (fd < 0) throw std::runtime_error("cannot create " + path + ": " + strerror(errno));
    auto pw = [&](const void *p, uint64_t len, uint64_t at) {
        uint64_t done = 0;
        while (done < len) {
            ssize_t k = pwrite(fd, (const uint8_t *)p + done, len - done, (off_t)(at + done));
            if (k <= 0) throw std::runtime_error("write failed on " + path + ": " + strerror(errno));
            done += (uint64_t)k;
        }
    };
    pw(h.b.data(), h.b.size(), 0);
    if (ftruncate(fd, (off_t)total) != 0) {
        ::close(fd);
        throw std::runtime_error("cannot size " + path + ": " + strerror(errno));
    }
    // work items: chunks of at most 4 MiB of encoded bytes of one tensor
    struct Item { size_t t; uint64_t b0, b1; };
    std::vector<Item> items;
    for (size_t ti = 0; ti < ts.size(); ti++) {
        auto lay = ggml_block_layout(ts[ti].type);
        const uint64_t be = lay.first == 1 ? 256 : lay.first;  // F32: 256-value chunks share one RNG stream
        const uint64_t nb = (ts[ti].bytes / lay.second * lay.first + be - 1) / be;
        const uint64_t per = std::max<uint64_t>(1, (4u << 20) / (be * 4));
        for (uint64_t b = 0; b < nb; b += per) items.push_back({ti, b, std::min(nb, b + per)});
    }
    std::atomic<size_t> next{0};
    std::atomic<bool> failed{false};
    std::string ferr;
    auto worker = [&]() {
        std::vector<float> x(256);
        std::vector<uint8_t> out;
        for (size_t i; (i = next.fetch_add(1)) < items.size() && !failed;) {
            const Item &it = items[i];
            const TSpec &t = ts[it.t];
            auto lay = ggml_block_layout(t.type);
            const uint64_t n = t.bytes / lay.second * lay.first;
            const uint64_t be = lay.first == 1 ? 256 : lay.first;
            out.clear();
            for (uint64_t b = it.b0; b < it.b1; b++) {
                Rng r(seed, it.t + 1, b);
                const uint64_t cnt = std::min<uint64_t>(be, n - b * be);
                for (uint64_t j = 0; j < cnt; j++) x[j] = draw(t.dist, r);
                const size_t o = out.size();
                switch (t.type) {
                case 0: out.resize(o + cnt * 4); memcpy(out.data() + o, x.data(), cnt * 4); break;
                case 2: out.resize(o + 18); enc_q4_0(x.data(), out.data() + o); break;
                case 8: out.resize(o + 34); enc_q8_0(x.data(), out.data() + o); break;
                case 12: out.resize(o + 144); enc_q4k_q5k(x.data(), out.data() + o, false); break;
                case 13: out.resize(o + 176); enc_q4k_q5k(x.data(), out.data() + o, true); break;
                case 14: out.resize(o + 210); enc_q6k(x.data(), out.data() + o); break;
                }
            }
            const uint64_t at = data_off + t.off + (lay.first == 1 ? it.b0 * 256 * 4 : it.b0 * lay.second);
            try {
                pw(out.data(), out.size(), at);
            } catch (const std::exception &e) {
                failed = true;
                ferr = e.what();
            }
        }
    };
    const int nt = threads > 0 ? threads : (int)std::max(1u, std::thread::hardware_concurrency());
    std::vector<std::thread> pool;
    for (int i = 0; i < nt; i++) pool.emplace_back(worker);
    for (auto &th : pool) th.join();
    ::close(fd);
    if (failed) throw std::runtime_error(ferr);
}

}  // namespace qdec
