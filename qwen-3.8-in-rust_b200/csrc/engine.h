// The decode engine: a GGUF model resident in HBM and the per-sequence state of a decode, with the model seam
// of the reference (crates/core/src/model.rs:184-495, spec.rs:184-433): load, prefill, forward_token,
// spec_prefill, spec_round.
#pragma once
#include <cuda_runtime.h>

#include <cstdint>
#include <functional>
#include <memory>
#include <string>
#include <vector>

#include "config.h"
#include "sample.cuh"

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
    int tp_rank = 0, tp_world = 1;  // tensor-parallel shard of this process (world 1: the whole model)
};

// Tensor-parallel shard of one rank.  Every matrix is split by output rows, so each rank computes complete dot
// products for its rows -- the same bits as one GPU -- and the four activations a layer produces sharded (the
// mixer's head outputs, the mixer output, the SwiGLU output image, the FFN output) are all-gathered before the
// next matrix reads them; the residual stream, norms and quantisation are replicated.
//   DeltaNet: K heads [kh_lo, kh_lo + nk) and the V heads p with p % n_k in that range (V head p reads K head
//   p % n_k), in V-head order: groups g = 0 .. n_v/n_k - 1 of nk heads starting at g * n_k + kh_lo.
//   GQA: q heads [qh_lo, qh_lo + nq) and kv heads [kv_lo, kv_lo + nkv) (a kv head may serve two ranks).
//   FFN rows [ff_lo, ff_lo + ff_rows) on 256-row boundaries (the SwiGLU output is exchanged as Q8_K blocks);
//   hidden-size outputs (attn_output, ssm_out, ffn_down, eh_proj) rows [h_lo, h_lo + h_rows);
//   lm_head rows [v_lo, v_lo + v_rows) with a (value, index) argmax exchange.
struct TpPlan {
    int rank = 0, world = 1;
    int kh_lo = 0, nk = 0, nv = 0;
    int qh_lo = 0, nq = 0, kv_lo = 0, nkv = 0;
    int ff_lo = 0, ff_rows = 0, h_lo = 0, h_rows = 0, v_lo = 0, v_rows = 0;
};
// throws ConfigError when the model's dimensions do not split over `world` ranks
TpPlan make_tp_plan(const ModelConfig& c, int rank, int world);

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
    bool loaded_direct = false;  // the weights were read with O_DIRECT (QDEC_LOAD_DIRECT)
    TpPlan tp;                   // this rank's shard (world 1: everything)
    bool is_stop(uint32_t id) const;

  private:
    uint8_t* blob_ = nullptr;
    std::vector<void*> shard_allocs_;  // tensor parallel: the replicated tensors and the rank's row slices, each its own
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
    // Plain greedy decode of several sequences in one forward, one row each (multi-sequence batching on one GPU):
    // every weight matrix is read once for all the rows, while each row's conv window, DeltaNet state, KV cache
    // and position are its own state's.  ids[i] is fed to members[i]; out[i] = its next id, as members[i]->step
    // would give.  The first member's row buffers carry the batch (its max_rows >= members.size()); all members
    // share the model, are greedy, and are on one GPU without tensor parallelism.
    static void batch_step(const std::vector<State*>& members, const uint32_t* ids, uint32_t* out);
    // forced drafts for the next round (spec.rs:439-452, used by the identity tests)
    void set_drafts(const uint32_t* d, int k);
    // the sampler of this state (crates/core/src/sample.rs): temperature <= 0 is greedy; the RNG restarts from
    // cfg.seed.  One GPU only (a tensor-parallel state's logits are split over its ranks).
    void set_sampler(const SamplerCfg& cfg);
    std::vector<uint32_t> drafts() const;

    // tensor parallelism: the exchange block (receive buffers + flags) is exported with a CUDA IPC handle; every
    // rank opens all the others' before the first forward (tp_connect)
    static constexpr int TP_HANDLE_BYTES = 80;
    void tp_export(void* out) const;
    void tp_connect(const void* handles);  // world x TP_HANDLE_BYTES, in rank order
    bool tp_ready() const { return tp_connected_; }
    // exchange timing totals since the state was made: {exchanges, ns copying, ns fencing + flagging, ns waiting}
    void tp_stats(uint64_t out[4]) const;

    // debugging / parity: the residual stream after layer `layer` of the last forward's row `row`
    // (layer = n_layer: the post-final-norm row the lm_head read)
    void debug_hidden(int layer, int row, float* out);
    void set_capture(bool on) { capture_ = on; }
    // parity: the carried state of layer `layer` as the reference holds it after the last call -- the DeltaNet
    // rows this engine commits lazily (the accepted rows of the last forward) applied to a copy.  what = 0: the
    // DeltaNet state f32 [n_v][dk][dv]; 1: its conv window f32 [channels][conv_kernel - 1]; 2 / 3: the K / V
    // cache rows [0, pos) f32 [pos][n_kv][head_dim] (this rank's heads over tensor parallelism).  Returns the
    // floats of the result (0: the layer has no such state); copies them to `out` when it is non-null and
    // holds `cap` floats.
    size_t debug_state(int layer, int what, float* out, size_t cap);
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
    const std::vector<State*>* batch_ = nullptr;  // during batch_step: the state that owns each row
    // plain steps and batch steps as CUDA graphs (captured on first use; a batch graph holds its members' buffers,
    // so it is keyed by their serial numbers and captured again when the members change)
    uint64_t serial_ = 0;
    cudaGraphExec_t step_exec_ = nullptr, batch_exec_ = nullptr;
    uint64_t step_launches_ = 0, batch_launches_ = 0;
    std::vector<uint64_t> batch_key_;
    void graph_run(cudaGraphExec_t* exec, uint64_t* n_launches, const std::function<void()>& enqueue);
    bool drafts_ready_ = false;
    uint64_t launches_ = 0;  // kernels this state has launched
    void count_launch(uint64_t n = 1) { launches_ += n; }
    // the speculative round as one CUDA graph (captured on first use)
    cudaGraphExec_t round_exec_ = nullptr;
    uint64_t round_launches_ = 0;
    int32_t* h_io_ = nullptr;  // pinned: [0] x_p in; [16..] {keep, emitted ids} out
    unsigned* err_io_ = nullptr;  // pinned: the kernels' two error words, read in stream order before each sync
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
    uint8_t* ffn_img_ = nullptr;    // the fused gate/up launch's Q8_K image of h (the down projection's input)
    unsigned* ffn_cnt_ = nullptr;   // its per-256-row-block completion counters (zero at rest)
    unsigned* dn_cnt_ = nullptr;    // the DeltaNet kernel's per-block counters of its head-output quantisation
    float *qkv_ = nullptr, *conved_ = nullptr, *z_ = nullptr, *alpha_ = nullptr, *beta_ = nullptr, *heads_ = nullptr;
    float *qg_ = nullptr, *kk_ = nullptr, *vv_ = nullptr, *qr_ = nullptr, *gate_ = nullptr, *attn_ = nullptr;
    float *g_ = nullptr, *u_ = nullptr, *final_ = nullptr, *logits_ = nullptr, *att_scores_ = nullptr;
    float *cat_ = nullptr, *mtp_h_ = nullptr, *mtp_hout_ = nullptr;
    size_t q8k_stride_ = 0, q80_stride_ = 0;  // bytes per row of the activation buffers
    // tensor-parallel exchange (world > 1): one device allocation, exported over CUDA IPC, holding two line
    // buffers (the peers write into them; consecutive exchanges alternate) and the receive buffers; xepoch_
    // (session count), xerr_ (set when a bounded wait gave up) and xstats_ are local
    static constexpr int XSLOTS = 1024;
    uint8_t* xblk_ = nullptr;
    size_t xblk_bytes_ = 0, xll_bytes_ = 0;  // whole block; one line buffer (2 x the largest exchange)
    uint8_t* xpeer_[8] = {};  // every rank's exchange block as mapped here (xpeer_[rank] = xblk_)
    bool tp_connected_ = false;
    unsigned *xepoch_ = nullptr, *xerr_ = nullptr;
    unsigned long long* xstats_ = nullptr;
    int xslot_ = 0;
    uint64_t xseq_ = 0;  // exchanges enqueued so far (graph replays advance it by an even count)
    size_t xo_mix_ = 0, xo_mlp_ = 0, xo_eh_ = 0, xo_heads_ = 0, xo_attn_ = 0, xo_ffn_ = 0, xo_amx_ = 0, xo_pad_ = 0;
    uint8_t* amx_pairs_ = nullptr;  // this rank's (value, index) per row before the exchange
    bool tp() const { return m_.tp.world > 1; }
    float* xg(size_t off) const { return reinterpret_cast<float*>(xblk_ + off); }
    void begin_session();
    // copy `rows` rows of `segs` (byte ranges {src offset, dst offset, length}) from the local `src` into every
    // rank's exchange buffer at `dst_off`, then wait until every rank's slice has arrived here
    void exchange(const void* src, size_t src_ld, size_t dst_off, size_t dst_ld, const int (*segs)[3], int nseg, int rows);
    void argmax_rows(const float* logits, int t, int32_t* out_dev);
    const float* mix_in() const { return tp() ? xg(xo_mix_) : mix_out_; }
    const float* mlp_in() const { return tp() ? xg(xo_mlp_) : mlp_out_; }

    struct DnState { float *S, *conv, *pend_x, *pend_decay, *pend_k, *pend_delta; };
    struct KvState { float *k, *v; };
    std::vector<DnState> dn_;
    std::vector<KvState> kv_;
    KvState mtp_kv_{};
    std::vector<float*> capture_h_;  // per layer residual rows when capturing

    void upload_ids(const uint32_t* ids, int n);
    void gemv(const DevMat& w, const float* normed_f32, int rows, float* y, const uint8_t* img = nullptr);
    void resid_norm(const float* delta, const float* w, int t, float* y_out, bool k8, bool k0);
    void quant_for(int type, const float* x, int n, int rows);
    void layer_forward(const LayerW& L, int li, int t, KvState* kv, const int* pos_dev, bool commit_dn);
    // the t-row forward of the main stack from device ids; logits in logits_, argmax in d_argmax
    void forward_rows(int t, const int32_t* ids_dev, bool want_logits_all);
    // the MTP block over t rows (tokens ids_dev, hidden rows, MTP position of row 0 at *pos_dev) into mtp_hout_
    void mtp_rows(int t, const int32_t* ids_dev, const float* hidden_rows, const int* pos_dev);
    // draft i from mtp_h_ (one row) through the shared lm_head into d_vids[1 + i]: the argmax, or a sampled id
    // with its processed distribution written densely to q_dense_[i]
    void enqueue_draft(int i);
    // the sampled id of one logits row into *out_dev (q: its processed distribution, dense, when non-null)
    void sample_row(const float* logits, int slot, int32_t* out_dev, float* q);
    bool sampling() const { return samp_.temperature > 0.0f; }
    SamplerCfg samp_{};
    uint64_t* d_rng_ = nullptr;
    void* samp_scratch_ = nullptr;
    int32_t* kept_ids_ = nullptr;  // [k + 2][vocab]: processed rows (verify rows 0..k, one for single draws)
    float* kept_probs_ = nullptr;
    int* kept_n_ = nullptr;
    float* q_dense_ = nullptr;     // [k][vocab]: the drafts' distributions
    float* samp_work_ = nullptr;   // [vocab]
    // drafts from..k-1, each an MTP row chained from the previous one (positions d_mpos[i])
    void enqueue_chain(int from);
    // the whole speculative round on the stream: verify, accept, rollback bookkeeping, MTP re-feed, drafts
    void enqueue_round();
    void sync();
};

}  // namespace qdec
