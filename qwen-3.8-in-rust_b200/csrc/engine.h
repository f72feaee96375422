// The decode engine: a GGUF model resident in HBM and the per-sequence state of a decode, with the model seam
// of the reference (crates/core/src/model.rs:184-495, spec.rs:184-433): load, prefill, forward_token,
// spec_prefill, spec_round.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <memory>
#include <string>
#include <vector>

#include "config.h"

namespace qdec {

struct DevMat {
    int type = 0;
    int rows = 0, cols = 0;
    const uint8_t* p = nullptr;
    size_t bytes = 0;
};

struct LayerW {
    uint32_t index = 0;
    bool attn = false;
    const float* attn_norm = nullptr;
    const float* post_norm = nullptr;
    // Gated DeltaNet (layers/gated_deltanet.rs:55-90)
    DevMat qkv, gate_z, alpha, beta, ssm_out;
    const float *ssm_a = nullptr, *dt_bias = nullptr, *conv_w = nullptr, *ssm_norm = nullptr;
    // gated GQA (layers/gqa_attention.rs:75-132)
    DevMat q, k, v, o;
    const float *q_norm = nullptr, *k_norm = nullptr;
    // MLP (layers/mlp.rs)
    DevMat ffn_gate, ffn_up, ffn_down;
};

struct MtpW {  // layers/mtp.rs:1-90
    LayerW block;
    DevMat eh_proj;
    const float *enorm = nullptr, *hnorm = nullptr, *head_norm = nullptr;
};

// RoPE positions past max_pos that the tables cover: a speculative round's MTP rows run up to 2k + 1 past the
// sequence position (its scratch re-feed rows and chained drafts).
constexpr int ROPE_SLACK = 64;

struct LoadOptions {
    int device = 0;
    int max_pos = 4096;  // RoPE table length
};

class Model {
  public:
    static std::unique_ptr<Model> load(const std::string& path, const LoadOptions& opt);  // throws
    ~Model();
    ModelConfig cfg;
    int device = 0;
    int max_pos = 0;
    DevMat embed, lm_head;
    const float* output_norm = nullptr;
    std::vector<LayerW> layers;
    bool has_mtp = false;
    MtpW mtp;
    float* rope_cos = nullptr;
    float* rope_sin = nullptr;
    float attn_scaling = 0.f;
    uint64_t weight_bytes = 0;   // bytes resident on the device
    uint64_t decode_bytes = 0;   // weight bytes one plain token reads (model.rs:274)
    uint64_t mtp_bytes = 0;      // the MTP block's bytes (blk.{n_layer})
    double load_secs = 0;
    bool is_stop(uint32_t id) const;

  private:
    uint8_t* blob_ = nullptr;
};

struct SpecCounters {  // spec.rs:21-42
    uint64_t rounds = 0, drafted = 0, accepted = 0, emitted = 0;
    std::vector<uint64_t> hist;
};

class State {
  public:
    State(const Model& m, int spec_k, int max_pos, int max_rows);  // throws
    ~State();
    State(const State&) = delete;
    State& operator=(const State&) = delete;

    // Model::prefill + logits of the last row (model.rs:443-461): returns argmax of the last row's logits.
    uint32_t prefill(const uint32_t* ids, int n);
    // Model::forward_token (model.rs:486-490) + argmax; logits copied out when `logits` is non-null.
    uint32_t step(uint32_t id, float* logits);
    // Model::spec_prefill (spec.rs:229-285): prefill, x_T, MTP over the prompt rows, the first k drafts.
    uint32_t spec_prefill(const uint32_t* ids, int n);
    // Model::spec_round (spec.rs:326-433) with greedy acceptance: emitted ids into `out` (m + 1 of them).
    int spec_round(uint32_t x_p, uint32_t* out);
    // forced drafts for the next round (spec.rs:439-452, used by the identity tests)
    void set_drafts(const uint32_t* d, int k);
    std::vector<uint32_t> drafts() const;

    // debugging / parity: the residual stream after layer `layer` of the last forward's row `row`
    // (layer = n_layer: the post-final-norm row the lm_head read)
    void debug_hidden(int layer, int row, float* out);
    void set_capture(bool on) { capture_ = on; }
    void logits_row(int row, float* out) const;

    int pos() const { return pos_; }
    int mtp_rows() const { return mtp_len_; }
    int spec_k() const { return k_; }
    SpecCounters counters;
    cudaStream_t stream = nullptr;
    uint64_t launches() const { return launches_; }

  private:
    const Model& m_;
    int k_, max_pos_, T_, mtp_cap_ = 0;
    int pos_ = 0, mtp_len_ = 0;
    bool capture_ = false;
    bool drafts_ready_ = false;
    uint64_t launches_ = 0;  // kernels this state has launched
    void count_launch(uint64_t n = 1) { launches_ += n; }
    // the speculative round as one CUDA graph (captured on first use)
    cudaGraphExec_t round_exec_ = nullptr;
    uint64_t round_launches_ = 0;
    int32_t* h_io_ = nullptr;  // pinned: [0] x_p in; [16..] {keep, emitted ids} out
    std::vector<void*> allocs_;
    void* dalloc(size_t bytes);

    // device buffers
    int32_t *d_ids = nullptr, *d_argmax = nullptr;
    // speculative round: verify ids (x_p, drafts), MTP re-feed ids, MTP positions, selected row, emitted ids
    int32_t *d_vids = nullptr, *d_mids = nullptr, *d_emit = nullptr;
    int *d_mpos = nullptr, *d_sel = nullptr;
    int *d_pos = nullptr, *d_keep = nullptr, *d_mtp_pos = nullptr;
    void* amx_scratch_ = nullptr;  // argmax partials and counters
    float *h_ = nullptr, *h_alt_ = nullptr, *embed_ = nullptr, *normed_ = nullptr, *mix_out_ = nullptr, *mlp_out_ = nullptr;
    uint8_t *q8k_ = nullptr, *q80_ = nullptr;
    float *qkv_ = nullptr, *conved_ = nullptr, *z_ = nullptr, *alpha_ = nullptr, *beta_ = nullptr, *heads_ = nullptr;
    float *qg_ = nullptr, *kk_ = nullptr, *vv_ = nullptr, *qr_ = nullptr, *gate_ = nullptr, *attn_ = nullptr;
    float *g_ = nullptr, *u_ = nullptr, *final_ = nullptr, *logits_ = nullptr;
    float *cat_ = nullptr, *mtp_h_ = nullptr, *mtp_hout_ = nullptr;
    size_t q8k_stride_ = 0, q80_stride_ = 0;  // bytes per row of the activation buffers
    struct DnState { float *S, *conv, *pend_x, *pend_decay, *pend_k, *pend_delta; };
    struct KvState { float *k, *v; };
    std::vector<DnState> dn_;
    std::vector<KvState> kv_;
    KvState mtp_kv_{};
    std::vector<float*> capture_h_;  // per layer residual rows when capturing

    void upload_ids(const uint32_t* ids, int n);
    void gemv(const DevMat& w, const float* normed_f32, int rows, float* y);
    void resid_norm(const float* delta, const float* w, int t, float* y_out, bool k8, bool k0);
    void quant_for(int type, const float* x, int n, int rows);
    void layer_forward(const LayerW& L, int li, int t, KvState* kv, const int* pos_dev, bool commit_dn);
    // the t-row forward of the main stack from device ids; logits in logits_, argmax in d_argmax
    void forward_rows(int t, const int32_t* ids_dev, bool want_logits_all);
    // the MTP block over t rows (tokens ids_dev, hidden rows, MTP position of row 0 at *pos_dev) into mtp_hout_
    void mtp_rows(int t, const int32_t* ids_dev, const float* hidden_rows, const int* pos_dev);
    // greedy draft from mtp_h_ (one row) through the shared lm_head into *out_dev
    void enqueue_draft(int32_t* out_dev);
    // drafts from..k-1, each an MTP row chained from the previous one (positions d_mpos[i])
    void enqueue_chain(int from);
    // the whole speculative round on the stream: verify, accept, rollback bookkeeping, MTP re-feed, drafts
    void enqueue_round();
    void sync();
};

}  // namespace qdec
