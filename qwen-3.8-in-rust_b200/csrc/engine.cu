// Model load and the decode step on the device: the forward of t rows through the 64-layer hybrid stack
// (model.rs:401-438, layers/mod.rs:295-377), plain greedy decode, prefill, and the speculative round with the
// MTP draft head (spec.rs:205-433, layers/mtp.rs:95-137).
//
// HBM layout.  The GGUF data section is copied to one device allocation unchanged (the weights keep their
// ggml block layout and 32-byte alignment); every tensor is a pointer into it.  Per sequence the State holds
// the residual rows, the quantised activation rows, the DeltaNet recurrent states (f32 [n_v][dk][dv] per layer)
// and conv windows, the f32 KV caches ([max_pos][n_kv][head_dim] per attention layer and for the MTP block),
// and the pending rows of the last DeltaNet call.
//
// Rollback without snapshots.  The reference snapshots every DeltaNet state before a verify batch and, when a
// draft is rejected, restores it and replays the accepted rows (spec.rs:337-344, :395-415).  Here the verify
// kernels never write the state past the batch: they leave the committed state in HBM and record, per row,
// the rank-one update (decay, k, delta) and the conv input.  The next call of the layer first applies exactly
// `keep` of those rows -- the same element operations in the same order as the replay -- so the state is
// bit-identical to the reference's and is read and written once per round.  KV caches roll back by position.
#include <cuda_runtime.h>

#include <algorithm>
#include <chrono>
#include <initializer_list>
#include <cmath>
#include <cstring>
#include <stdexcept>

#include "common.cuh"
#include "engine.h"
#include "gguf.h"
#include "kernels.cuh"
#include "layers.cuh"

namespace qdec {

namespace {

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

__global__ void add_rows_kernel(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

}  // namespace

// ------------------------------------------------------------------------------------------------ Model

Model::~Model() {
    if (blob_) cudaFree(blob_);
    if (rope_cos) cudaFree(rope_cos);
    if (rope_sin) cudaFree(rope_sin);
}

bool Model::is_stop(uint32_t id) const {
    return std::find(cfg.stop_ids.begin(), cfg.stop_ids.end(), id) != cfg.stop_ids.end();
}

std::unique_ptr<Model> Model::load(const std::string& path, const LoadOptions& opt) {
    const auto t0 = std::chrono::steady_clock::now();
    Gguf g(path);
    std::unique_ptr<Model> m(new Model());
    m->cfg = ModelConfig::from_gguf(g);
    m->device = opt.device;
    m->max_pos = opt.max_pos;
    ck(cudaSetDevice(opt.device), "cudaSetDevice");
    const ModelConfig& c = m->cfg;

    // the data section, unchanged, in one allocation
    const uint64_t data_bytes = g.file_size() - g.data_offset();
    ck(cudaMalloc(&m->blob_, data_bytes + 256), "weights allocation");
    m->weight_bytes = data_bytes;
    {
        const size_t CH = 256ull << 20;
        void* host = nullptr;
        ck(cudaHostAlloc(&host, 2 * CH, cudaHostAllocDefault), "pinned staging");
        cudaStream_t s;
        ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "stream");
        cudaEvent_t done[2];
        cudaEventCreateWithFlags(&done[0], cudaEventDisableTiming);
        cudaEventCreateWithFlags(&done[1], cudaEventDisableTiming);
        bool used[2] = {false, false};
        int b = 0;
        try {
            for (uint64_t off = 0; off < data_bytes; off += CH, b ^= 1) {
                const uint64_t len = std::min<uint64_t>(CH, data_bytes - off);
                if (used[b]) ck(cudaEventSynchronize(done[b]), "staging wait");
                uint8_t* hb = static_cast<uint8_t*>(host) + b * CH;
                g.read_at(g.data_offset() + off, hb, len);
                ck(cudaMemcpyAsync(m->blob_ + off, hb, len, cudaMemcpyHostToDevice, s), "weights upload");
                ck(cudaEventRecord(done[b], s), "event");
                used[b] = true;
            }
            ck(cudaStreamSynchronize(s), "weights upload");
        } catch (...) {
            cudaStreamSynchronize(s);
            cudaFreeHost(host);
            cudaStreamDestroy(s);
            throw;
        }
        cudaEventDestroy(done[0]);
        cudaEventDestroy(done[1]);
        cudaFreeHost(host);
        cudaStreamDestroy(s);
    }
    auto ptr = [&](const TensorInfo& t) { return m->blob_ + t.rel_offset; };
    // Q6_K matrices are repacked in place into the split layout the bulk-copy GEMV reads (same bytes); the
    // embedding table keeps the ggml layout because rows of it are dequantised directly
    uint8_t* repack_tmp = nullptr;
    uint64_t repack_cap = 0;
    for (const TensorInfo& t : g.tensors())
        if (t.type == T_Q6_K && t.name != "token_embd.weight") repack_cap = std::max(repack_cap, t.byte_size);
    if (repack_cap) ck(cudaMalloc(&repack_tmp, repack_cap), "repack buffer");
    auto repack = [&](const TensorInfo& t) {
        uint8_t* p = m->blob_ + t.rel_offset;
        ck(cudaMemcpy(repack_tmp, p, t.byte_size, cudaMemcpyDeviceToDevice), "repack copy");
        ck(launch_repack_q6k(repack_tmp, t.byte_size / 210, p, 0), "repack");
        ck(cudaDeviceSynchronize(), "repack");
    };
    auto mat = [&](const std::string& name, uint64_t rows, uint64_t cols) {
        const TensorInfo& t = g.tensor(name);
        const auto sh = t.shape_numpy();
        if (sh.size() != 2 || sh[0] != rows || sh[1] != cols)
            throw ConfigError("tensor " + name + ": expected shape [" + std::to_string(rows) + ", " + std::to_string(cols) + "]");
        if (!(t.type == T_F32 || t.type == T_Q4_0 || t.type == T_Q8_0 || is_kquant(t.type)))
            throw ConfigError("tensor " + name + ": no kernel for ggml type " + std::to_string(t.type));
        DevMat d;
        d.type = t.type;
        d.rows = (int)rows;
        d.cols = (int)cols;
        d.p = ptr(t);
        d.bytes = t.byte_size;
        if (t.type == T_Q6_K && name != "token_embd.weight") {
            repack(t);
            d.type = T_Q6_K_SPLIT;
        }
        return d;
    };
    auto vec = [&](const std::string& name, uint64_t len) -> const float* {
        const TensorInfo& t = g.tensor(name);
        if (t.n_elements != len) throw ConfigError("tensor " + name + ": expected " + std::to_string(len) + " elements");
        if (t.type != T_F32) throw ConfigError("tensor " + name + ": 1-D weights must be F32 here");
        return reinterpret_cast<const float*>(ptr(t));
    };
    const uint64_t H = c.hidden_size;
    m->embed = mat("token_embd.weight", c.vocab_size, H);
    m->lm_head = mat(c.tie_word_embeddings ? "token_embd.weight" : "output.weight", c.vocab_size, H);
    m->output_norm = vec("output_norm.weight", H);
    auto load_layer = [&](uint32_t i, bool attention) {
        LayerW L;
        L.index = i;
        L.attn = attention;
        const std::string p = "blk." + std::to_string(i) + ".";
        L.attn_norm = vec(p + "attn_norm.weight", H);
        L.post_norm = vec(p + "post_attention_norm.weight", H);
        if (attention) {
            const uint64_t hd = c.head_dim_k;
            L.q = mat(p + "attn_q.weight", 2ull * c.n_head * hd, H);
            L.k = mat(p + "attn_k.weight", (uint64_t)c.n_head_kv * hd, H);
            L.v = mat(p + "attn_v.weight", (uint64_t)c.n_head_kv * hd, H);
            L.o = mat(p + "attn_output.weight", H, (uint64_t)c.n_head * hd);
            L.q_norm = vec(p + "attn_q_norm.weight", hd);
            L.k_norm = vec(p + "attn_k_norm.weight", hd);
        } else {
            L.qkv = mat(p + "attn_qkv.weight", c.dn_qkv_dim, H);
            L.gate_z = mat(p + "attn_gate.weight", c.dn_v_dim, H);
            L.alpha = mat(p + "ssm_alpha.weight", c.dn_n_v_heads, H);
            L.beta = mat(p + "ssm_beta.weight", c.dn_n_v_heads, H);
            L.ssm_a = vec(p + "ssm_a", c.dn_n_v_heads);
            L.dt_bias = vec(p + "ssm_dt.bias", c.dn_n_v_heads);
            L.conv_w = vec(p + "ssm_conv1d.weight", (uint64_t)c.dn_qkv_dim * c.dn_conv_kernel);
            L.ssm_norm = vec(p + "ssm_norm.weight", c.dn_head_dim_v);
            L.ssm_out = mat(p + "ssm_out.weight", H, c.dn_v_dim);
        }
        L.ffn_gate = mat(p + "ffn_gate.weight", c.intermediate_size, H);
        L.ffn_up = mat(p + "ffn_up.weight", c.intermediate_size, H);
        L.ffn_down = mat(p + "ffn_down.weight", H, c.intermediate_size);
        return L;
    };
    for (uint32_t i = 0; i < c.n_layer; i++) m->layers.push_back(load_layer(i, c.is_attention(i)));
    if (!c.mtp_layers.empty()) {
        const uint32_t mi = c.mtp_layers[0];
        const std::string p = "blk." + std::to_string(mi) + ".nextn.";
        m->mtp.block = load_layer(mi, true);
        m->mtp.eh_proj = mat(p + "eh_proj.weight", H, 2 * H);
        m->mtp.enorm = vec(p + "enorm.weight", H);
        m->mtp.hnorm = vec(p + "hnorm.weight", H);
        m->mtp.head_norm = vec(p + "shared_head_norm.weight", H);
        m->has_mtp = true;
    }
    // RoPE tables (rope.rs:10-29): inv_freq[i] = 1 / theta^(2i / rope_dim) in f32, angle = f32(pos) * inv_freq,
    // cos/sin in f32, each half duplicated -- computed on the host with the C library, like the reference
    const int rd = (int)c.rope_dim, half = rd / 2;
    std::vector<float> inv(half), cs((size_t)opt.max_pos * rd), sn((size_t)opt.max_pos * rd);
    for (int i = 0; i < half; i++) inv[i] = 1.0f / powf(c.rope_freq_base, (float)(2 * i) / (float)rd);
    for (int pos = 0; pos < opt.max_pos; pos++) {
        const float pf = (float)pos;
        for (int i = 0; i < half; i++) {
            const float a = pf * inv[i];
            const float s = sinf(a), co = cosf(a);
            cs[(size_t)pos * rd + i] = cs[(size_t)pos * rd + i + half] = co;
            sn[(size_t)pos * rd + i] = sn[(size_t)pos * rd + i + half] = s;
        }
    }
    ck(cudaMalloc(&m->rope_cos, cs.size() * 4), "rope table");
    ck(cudaMalloc(&m->rope_sin, sn.size() * 4), "rope table");
    ck(cudaMemcpy(m->rope_cos, cs.data(), cs.size() * 4, cudaMemcpyHostToDevice), "rope upload");
    ck(cudaMemcpy(m->rope_sin, sn.data(), sn.size() * 4, cudaMemcpyHostToDevice), "rope upload");
    if (repack_tmp) cudaFree(repack_tmp);
    m->attn_scaling = powf((float)c.head_dim_k, -0.5f);  // (hd as f32).powf(-0.5) (gqa_attention.rs:186)
    uint64_t layer_total = 0;
    for (uint32_t i = 0; i < c.n_layer; i++) {
        uint64_t s0, e0;
        if (g.layer_span(i, s0, e0)) layer_total += e0 - s0;
    }
    m->decode_bytes = layer_total + m->lm_head.bytes + 4ull * H + m->embed.bytes / c.vocab_size;
    for (uint32_t mi : c.mtp_layers) {
        uint64_t s0, e0;
        if (g.layer_span(mi, s0, e0)) m->mtp_bytes += e0 - s0;
    }
    m->load_secs = std::chrono::duration<double>(std::chrono::steady_clock::now() - t0).count();
    return m;
}

// ------------------------------------------------------------------------------------------------ State

void* State::dalloc(size_t bytes) {
    void* p = nullptr;
    ck(cudaMalloc(&p, std::max<size_t>(bytes, 16)), "state allocation");
    ck(cudaMemset(p, 0, std::max<size_t>(bytes, 16)), "state init");
    allocs_.push_back(p);
    return p;
}

State::State(const Model& m, int spec_k, int max_pos, int max_rows) : m_(m), k_(spec_k), max_pos_(max_pos) {
    const ModelConfig& c = m.cfg;
    if (max_pos > m.max_pos) throw std::invalid_argument("max_pos exceeds the model's RoPE table");
    if (spec_k > 0 && !m.has_mtp) throw std::invalid_argument("the GGUF has no MTP block (no nextn tensors): speculative decoding needs one");
    T_ = std::max(max_rows, spec_k + 1);
    ck(cudaSetDevice(m.device), "cudaSetDevice");
    ck(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    const size_t H = c.hidden_size, FF = c.intermediate_size, T = T_;
    size_t maxw = std::max<size_t>(std::max<size_t>(2 * H, FF), std::max<size_t>(c.dn_v_dim, (size_t)c.n_head * c.head_dim_k));
    q8k_stride_ = maxw / 256 * 292 + 64;
    q80_stride_ = maxw / 32 * 34 + 64;
    d_ids = (int32_t*)dalloc(T * 4);
    d_argmax = (int32_t*)dalloc(T * 4);
    d_pos = (int*)dalloc(4);
    d_keep = (int*)dalloc(4);
    d_mtp_pos = (int*)dalloc(4);
    h_ = (float*)dalloc(T * H * 4);
    embed_ = (float*)dalloc(T * H * 4);
    normed_ = (float*)dalloc(T * maxw * 4);
    mix_out_ = (float*)dalloc(T * H * 4);
    mlp_out_ = (float*)dalloc(T * H * 4);
    q8k_ = (uint8_t*)dalloc(T * q8k_stride_);
    q80_ = (uint8_t*)dalloc(T * q80_stride_);
    g_ = (float*)dalloc(T * FF * 4);
    u_ = (float*)dalloc(T * FF * 4);
    final_ = (float*)dalloc(T * H * 4);
    logits_ = (float*)dalloc(T * (size_t)c.vocab_size * 4);
    if (!c.deltanet_layers.empty()) {
        qkv_ = (float*)dalloc(T * c.dn_qkv_dim * 4);
        conved_ = (float*)dalloc(T * c.dn_qkv_dim * 4);
        z_ = (float*)dalloc(T * c.dn_v_dim * 4);
        alpha_ = (float*)dalloc(T * c.dn_n_v_heads * 4);
        beta_ = (float*)dalloc(T * c.dn_n_v_heads * 4);
        heads_ = (float*)dalloc(T * c.dn_v_dim * 4);
    }
    const size_t hd = c.head_dim_k, qd = (size_t)c.n_head * hd, kvd = (size_t)c.n_head_kv * hd;
    qg_ = (float*)dalloc(T * 2 * qd * 4);
    kk_ = (float*)dalloc(T * kvd * 4);
    vv_ = (float*)dalloc(T * kvd * 4);
    qr_ = (float*)dalloc(T * qd * 4);
    gate_ = (float*)dalloc(T * qd * 4);
    attn_ = (float*)dalloc(T * qd * 4);
    for (const LayerW& L : m.layers) {
        if (L.attn) {
            kv_.push_back({(float*)dalloc((size_t)max_pos * kvd * 4), (float*)dalloc((size_t)max_pos * kvd * 4)});
            dn_.push_back({});
        } else {
            DnState d;
            d.S = (float*)dalloc(c.dn_state_elems_per_layer * 4);
            d.conv = (float*)dalloc(c.dn_conv_state_elems_per_layer * 4);
            d.pend_x = (float*)dalloc(T * c.dn_qkv_dim * 4);
            d.pend_decay = (float*)dalloc(T * c.dn_n_v_heads * 4);
            d.pend_k = (float*)dalloc(T * c.dn_n_v_heads * c.dn_head_dim_k * 4);
            d.pend_delta = (float*)dalloc(T * c.dn_n_v_heads * c.dn_head_dim_v * 4);
            dn_.push_back(d);
            kv_.push_back({});
        }
    }
    if (m.has_mtp) {
        mtp_kv_ = {(float*)dalloc((size_t)max_pos * kvd * 4), (float*)dalloc((size_t)max_pos * kvd * 4)};
        cat_ = (float*)dalloc(T * 2 * H * 4);
        mtp_h_ = (float*)dalloc(T * H * 4);
        mtp_hout_ = (float*)dalloc(T * H * 4);
    }
    counters.hist.assign(spec_k + 1, 0);
}

State::~State() {
    if (stream) cudaStreamSynchronize(stream);
    for (void* p : allocs_) cudaFree(p);
    for (float* p : capture_h_) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
}

void State::sync() {
    ck(cudaStreamSynchronize(stream), "decode step");
    const unsigned err = read_kernel_error(true);
    if (err) throw std::runtime_error("a device-side wait gave up (code " + std::to_string(err) + ")");
}

void State::upload_ids(const uint32_t* ids, int n) {
    for (int i = 0; i < n; i++)
        if (ids[i] >= m_.cfg.vocab_size) throw std::invalid_argument("token id " + std::to_string(ids[i]) + " outside the vocabulary");
    ck(cudaMemcpyAsync(d_ids, ids, (size_t)n * 4, cudaMemcpyHostToDevice, stream), "ids upload");
}

static bool needs_q8k(std::initializer_list<int> ts) {
    for (int t : ts) if (is_kquant(t)) return true;
    return false;
}
static bool needs_q80(std::initializer_list<int> ts) {
    for (int t : ts) if (t == T_Q8_0 || t == T_Q4_0) return true;
    return false;
}

void State::gemv(const DevMat& w, const float* normed_f32, int rows, float* y) {
    const void* act = is_kquant(w.type) ? (const void*)q8k_ : (w.type == T_F32 ? (const void*)normed_f32 : (const void*)q80_);
    // activation rows are laid out back to back at the stride of this weight's width
    // weights are written once at load, so the GEMV may stream them before its predecessor finishes
    ck(launch_gemv(w.type, w.p, w.rows, w.cols, act, rows, y, stream, true), "gemv");
}

void State::quant_for(int type, const float* x, int n, int rows) {
    count_launch(); ck(launch_quant_rows(x, n, rows, is_kquant(type) ? q8k_ : nullptr, (type == T_Q8_0 || type == T_Q4_0) ? q80_ : nullptr, stream),
       "quantise");
}

// One decoder layer over t rows (layers/mod.rs:335-377): the residual stream h_ enters as (h_ + mlp_out_) of
// the previous layer (or the layer input `first_in` for layer 0 / the MTP block), leaves in h_ + mlp_out_.
void State::layer_forward(const LayerW& L, int li, int t, KvState* kv, const int* pos_dev, bool commit_dn) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const float eps = c.rms_norm_eps;
    if (L.attn) {
        const bool k8 = needs_q8k({L.q.type, L.k.type, L.v.type}), k0 = needs_q80({L.q.type, L.k.type, L.v.type});
        count_launch(); ck(launch_resid_norm_quant(h_, li == 0 ? nullptr : mlp_out_, h_, L.attn_norm, eps, H, t, normed_, k8 ? q8k_ : nullptr,
                                   k0 ? q80_ : nullptr, stream), "attn_norm");
        gemv(L.q, normed_, t, qg_);
        gemv(L.k, normed_, t, kk_);
        gemv(L.v, normed_, t, vv_);
        QkArgs qa{qg_, kk_, vv_, L.q_norm, L.k_norm, m_.rope_cos, m_.rope_sin, pos_dev, qr_, gate_, kv->k, kv->v,
                  (int)c.n_head, (int)c.n_head_kv, (int)c.head_dim_k, (int)c.rope_dim, eps};
        count_launch(); ck(launch_qk_norm_rope(qa, t, stream), "qk_norm_rope");
        AttnArgs aa{qr_, gate_, kv->k, kv->v, pos_dev, attn_, (int)c.n_head, (int)c.n_head_kv, (int)c.head_dim_k, max_pos_,
                    m_.attn_scaling};
        count_launch(); ck(launch_attention(aa, t, stream), "attention");
        quant_for(L.o.type, attn_, L.o.cols, t);
        gemv(L.o, attn_, t, mix_out_);
    } else {
        const DnState& d = dn_[li];
        const bool k8 = needs_q8k({L.qkv.type, L.gate_z.type, L.alpha.type, L.beta.type});
        const bool k0 = needs_q80({L.qkv.type, L.gate_z.type, L.alpha.type, L.beta.type});
        count_launch(); ck(launch_resid_norm_quant(h_, li == 0 ? nullptr : mlp_out_, h_, L.attn_norm, eps, H, t, normed_, k8 ? q8k_ : nullptr,
                                   k0 ? q80_ : nullptr, stream), "attn_norm");
        gemv(L.qkv, normed_, t, qkv_);
        gemv(L.gate_z, normed_, t, z_);
        gemv(L.alpha, normed_, t, alpha_);
        gemv(L.beta, normed_, t, beta_);
        count_launch(); ck(launch_conv_step(d.conv, L.conv_w, (int)c.dn_conv_kernel, (int)c.dn_qkv_dim, qkv_, t, conved_, d.pend_x,
                            commit_dn ? d_keep : nullptr, T_, stream), "conv");
        DeltaArgs da{d.S, conved_, alpha_, beta_, z_, L.ssm_a, L.dt_bias, L.ssm_norm, heads_, d.pend_decay, d.pend_k, d.pend_delta,
                     commit_dn ? d_keep : nullptr, t, T_, (int)c.dn_n_k_heads, (int)c.dn_n_v_heads, (int)c.dn_head_dim_k,
                     (int)c.dn_head_dim_v, (int)c.dn_k_dim, (int)c.dn_qkv_dim, eps};
        count_launch(); ck(launch_deltanet_heads(da, stream), "deltanet");
        quant_for(L.ssm_out.type, heads_, L.ssm_out.cols, t);
        gemv(L.ssm_out, heads_, t, mix_out_);
    }
    // h = x + mixer(x); then the MLP on post_attention_norm(h) (mlp.rs:53-64)
    const bool k8 = needs_q8k({L.ffn_gate.type, L.ffn_up.type}), k0 = needs_q80({L.ffn_gate.type, L.ffn_up.type});
    count_launch(); ck(launch_resid_norm_quant(h_, mix_out_, h_, L.post_norm, eps, H, t, normed_, k8 ? q8k_ : nullptr, k0 ? q80_ : nullptr, stream),
       "post_attention_norm");
    gemv(L.ffn_gate, normed_, t, g_);
    gemv(L.ffn_up, normed_, t, u_);
    const int dt = L.ffn_down.type;
    count_launch(); ck(launch_swiglu_quant(g_, u_, (int)c.intermediate_size, t, nullptr, is_kquant(dt) ? q8k_ : nullptr,
                           (dt == T_Q8_0 || dt == T_Q4_0) ? q80_ : nullptr, stream), "swiglu");
    gemv(L.ffn_down, g_, t, mlp_out_);
}

void State::forward_rows(int t, bool want_logits_all) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    count_launch(); ck(launch_dequant_rows(m_.embed.type, m_.embed.p, m_.embed.bytes / m_.embed.rows, H, d_ids, t, h_, stream), "embed");
    for (size_t li = 0; li < m_.layers.size(); li++) {
        layer_forward(m_.layers[li], (int)li, t, &kv_[li], d_pos, true);
        if (capture_) {
            if (capture_h_.size() < m_.layers.size() + 1) {
                capture_h_.assign(m_.layers.size() + 1, nullptr);
                for (auto& p : capture_h_) ck(cudaMalloc(&p, (size_t)T_ * H * 4), "capture buffer");
            }
            add_rows_kernel<<<64, 256, 0, stream>>>(h_, mlp_out_, capture_h_[li], (size_t)t * H);
        }
    }
    // final norm (model.rs:430-438): the post-norm rows are what the lm_head and the MTP read
    const int ht = m_.lm_head.type;
    count_launch(); ck(launch_resid_norm_quant(h_, mlp_out_, h_, m_.output_norm, c.rms_norm_eps, H, t, final_, is_kquant(ht) ? q8k_ : nullptr,
                               (ht == T_Q8_0 || ht == T_Q4_0) ? q80_ : nullptr, stream), "output_norm");
    if (capture_ && !capture_h_.empty())
        ck(cudaMemcpyAsync(capture_h_[m_.layers.size()], final_, (size_t)t * H * 4, cudaMemcpyDeviceToDevice, stream), "capture");
    if (want_logits_all) {
        gemv(m_.lm_head, final_, t, logits_);
        count_launch(); ck(launch_argmax(logits_, (int)c.vocab_size, t, d_argmax, stream), "argmax");
    } else {
        // only the last row's logits (prefill): quantise that row alone at row 0
        quant_for(ht, final_ + (size_t)(t - 1) * H, H, 1);
        gemv(m_.lm_head, final_ + (size_t)(t - 1) * H, 1, logits_);
        count_launch(); ck(launch_argmax(logits_, (int)c.vocab_size, 1, d_argmax, stream), "argmax");
    }
}

static void set_dev_int(int* d, int v, cudaStream_t s) {
    // a pageable source is staged before cudaMemcpyAsync returns, so `v` may die with the caller
    ck(cudaMemcpyAsync(d, &v, 4, cudaMemcpyHostToDevice, s), "device int");
}

uint32_t State::prefill(const uint32_t* ids, int n) {
    if (n <= 0) throw std::invalid_argument("prefill: empty prompt");
    if (pos_ + n > max_pos_) throw std::invalid_argument("prefill: the sequence would exceed max_pos");
    for (int off = 0; off < n; off += T_) {
        const int t = std::min(T_, n - off);
        upload_ids(ids + off, t);
        set_dev_int(d_pos, pos_, stream);
        forward_rows(t, false);
        set_dev_int(d_keep, t, stream);  // every row of a prefill chunk is kept
        pos_ += t;
    }
    int32_t a = 0;
    ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
    sync();
    return (uint32_t)a;
}

uint32_t State::step(uint32_t id, float* logits) {
    if (pos_ + 1 > max_pos_) throw std::invalid_argument("step: the sequence would exceed max_pos");
    upload_ids(&id, 1);
    set_dev_int(d_pos, pos_, stream);
    forward_rows(1, true);
    set_dev_int(d_keep, 1, stream);
    pos_ += 1;
    int32_t a = 0;
    ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
    if (logits) ck(cudaMemcpyAsync(logits, logits_, (size_t)m_.cfg.vocab_size * 4, cudaMemcpyDeviceToHost, stream), "logits");
    sync();
    return (uint32_t)a;
}

void State::logits_row(int row, float* out) const {
    ck(cudaMemcpy(out, logits_ + (size_t)row * m_.cfg.vocab_size, (size_t)m_.cfg.vocab_size * 4, cudaMemcpyDeviceToHost), "logits");
}

void State::debug_hidden(int layer, int row, float* out) {
    if (!capture_ || capture_h_.empty() || layer < 0 || layer > (int)m_.layers.size()) throw std::invalid_argument("debug_hidden: no capture");
    ck(cudaStreamSynchronize(stream), "sync");
    ck(cudaMemcpy(out, capture_h_[layer] + (size_t)row * m_.cfg.hidden_size, m_.cfg.hidden_size * 4, cudaMemcpyDeviceToHost), "capture");
}

// The MTP block over t rows at MTP positions mtp_len_.. (layers/mtp.rs:95-130): row i is
// [rmsnorm(embed(tokens[i]), enorm) | rmsnorm(hidden[i], hnorm)] -> eh_proj -> one attention decoder layer with
// its own KV cache -> shared_head_norm, into mtp_hout_.
void State::mtp_rows(int t, const uint32_t* tokens, const float* hidden, bool hidden_is_hout) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const MtpW& M = m_.mtp;
    (void)hidden_is_hout;
    upload_ids(tokens, t);
    count_launch(); ck(launch_dequant_rows(m_.embed.type, m_.embed.p, m_.embed.bytes / m_.embed.rows, H, d_ids, t, embed_, stream), "embed");
    count_launch(); ck(launch_rmsnorm_rows(embed_, H, M.enorm, c.rms_norm_eps, H, t, cat_, 2 * H, stream), "enorm");
    count_launch(); ck(launch_rmsnorm_rows(hidden, H, M.hnorm, c.rms_norm_eps, H, t, cat_ + H, 2 * H, stream), "hnorm");
    quant_for(M.eh_proj.type, cat_, 2 * H, t);
    gemv(M.eh_proj, cat_, t, h_);  // u rows become the block's residual input
    set_dev_int(d_mtp_pos, mtp_len_, stream);
    layer_forward(M.block, 0, t, &mtp_kv_, d_mtp_pos, false);
    count_launch(); ck(launch_resid_norm_quant(h_, mlp_out_, h_, M.head_norm, c.rms_norm_eps, H, t, mtp_hout_, nullptr, nullptr, stream), "head_norm");
    mtp_len_ += t;
}

// The draft of MTP row `row`: the shared lm_head on mtp_hout_[row], greedy (spec.rs:205-215, mtp.rs:132-137).
uint32_t State::mtp_draft_from_row(int row) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    quant_for(m_.lm_head.type, mtp_hout_ + (size_t)row * H, H, 1);
    gemv(m_.lm_head, mtp_hout_ + (size_t)row * H, 1, logits_ + (size_t)(T_ - 1) * c.vocab_size);
    count_launch(); ck(launch_argmax(logits_ + (size_t)(T_ - 1) * c.vocab_size, (int)c.vocab_size, 1, d_argmax + (T_ - 1), stream), "argmax");
    int32_t a = 0;
    ck(cudaMemcpyAsync(&a, d_argmax + (T_ - 1), 4, cudaMemcpyDeviceToHost, stream), "argmax");
    sync();
    return (uint32_t)a;
}

// Drafts from..k-1 by chaining single MTP rows from the previous row's hidden (spec.rs:205-222).
void State::chain_drafts(int from) {
    const int H = (int)m_.cfg.hidden_size;
    for (int i = from; i < k_; i++) {
        const uint32_t last = drafts_[i - 1];
        // hprev = the previous MTP row's post-norm hidden, which the last call left in mtp_hout_[prev]; copy it
        // aside since this row's output overwrites mtp_hout_
        ck(cudaMemcpyAsync(mtp_h_, mtp_hout_ + (size_t)prev_row_ * H, (size_t)H * 4, cudaMemcpyDeviceToDevice, stream), "hprev");
        mtp_rows(1, &last, mtp_h_, true);
        prev_row_ = 0;
        drafts_.push_back(mtp_draft_from_row(0));
    }
}

uint32_t State::spec_prefill(const uint32_t* ids, int n) {
    if (k_ <= 0) throw std::invalid_argument("spec_prefill: state without spec buffers");
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const int p = pos_;
    if (mtp_len_ < p) throw std::logic_error("spec_prefill: the MTP has fewer rows than consumed positions");
    // the prompt's post-final-norm rows, kept for the MTP rows (x_{j+1}, h_j)
    float* normed_all = nullptr;
    ck(cudaMalloc(&normed_all, (size_t)n * H * 4), "prompt rows");
    uint32_t x_t = 0;
    try {
        for (int off = 0; off < n; off += T_) {
            const int t = std::min(T_, n - off);
            upload_ids(ids + off, t);
            set_dev_int(d_pos, pos_, stream);
            forward_rows(t, false);
            set_dev_int(d_keep, t, stream);
            pos_ += t;
            ck(cudaMemcpyAsync(normed_all + (size_t)off * H, final_, (size_t)t * H * 4, cudaMemcpyDeviceToDevice, stream), "rows");
        }
        int32_t a = 0;
        ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
        sync();
        x_t = (uint32_t)a;
        mtp_len_ = p;
        std::vector<uint32_t> xs(n);
        for (int j = 0; j < n; j++) xs[j] = (j + 1 < n) ? ids[j + 1] : x_t;
        for (int off = 0; off < n; off += T_) {
            const int t = std::min(T_, n - off);
            mtp_rows(t, xs.data() + off, normed_all + (size_t)off * H, false);
            prev_row_ = t - 1;
        }
    } catch (...) {
        cudaStreamSynchronize(stream);
        cudaFree(normed_all);
        throw;
    }
    cudaStreamSynchronize(stream);
    cudaFree(normed_all);
    drafts_.clear();
    drafts_.push_back(mtp_draft_from_row(prev_row_));
    chain_drafts(1);
    return x_t;
}

int State::spec_round(uint32_t x_p, uint32_t* out) {
    if (k_ <= 0) throw std::invalid_argument("spec_round: state without spec buffers");
    if ((int)drafts_.size() != k_) throw std::logic_error("spec_round: drafts missing (call spec_prefill first)");
    const int t = k_ + 1;
    const int p = pos_;
    if (p + t > max_pos_) throw std::invalid_argument("spec_round: the sequence would exceed max_pos");
    if (mtp_len_ != p + k_ - 1) throw std::logic_error("spec_round: MTP rows out of step with the position");
    std::vector<uint32_t> batch(t);
    batch[0] = x_p;
    for (int i = 0; i < k_; i++) batch[i + 1] = drafts_[i];
    upload_ids(batch.data(), t);
    set_dev_int(d_pos, p, stream);
    forward_rows(t, true);  // the verify batch
    std::vector<int32_t> am(t);
    ck(cudaMemcpyAsync(am.data(), d_argmax, (size_t)t * 4, cudaMemcpyDeviceToHost, stream), "argmax");
    sync();
    // greedy accept (spec.rs:352-366): the longest prefix where the model's argmax equals the draft
    int m = 0;
    std::vector<uint32_t> emitted;
    while (m < k_) {
        const uint32_t a = (uint32_t)am[m];
        emitted.push_back(a);
        if (a != drafts_[m]) break;
        m++;
    }
    if (m == k_) emitted.push_back((uint32_t)am[k_]);
    const int keep = m + 1;
    // roll back: the DeltaNet layers will commit `keep` rows; the KV caches end at p + keep
    set_dev_int(d_keep, keep, stream);
    pos_ = p + keep;
    counters.rounds++;
    counters.drafted += k_;
    counters.accepted += m;
    counters.emitted += keep;
    counters.hist[m]++;
    // the MTP: forget its draft rows, feed the accepted pairs (emitted_i, normed_i), draft the next round
    mtp_len_ = p;
    mtp_rows(keep, emitted.data(), final_, false);
    prev_row_ = keep - 1;
    drafts_.clear();
    drafts_.push_back(mtp_draft_from_row(prev_row_));
    chain_drafts(1);
    for (int i = 0; i < keep; i++) out[i] = emitted[i];
    return keep;
}

void State::set_drafts(const uint32_t* d, int k) {
    if (k != k_) throw std::invalid_argument("set_drafts: wrong number of drafts");
    for (int i = 0; i < k; i++)
        if (d[i] >= m_.cfg.vocab_size) throw std::invalid_argument("set_drafts: draft outside the vocabulary");
    drafts_.assign(d, d + k);
}

}  // namespace qdec
