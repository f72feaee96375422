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
#include <atomic>
#include <chrono>
#include <initializer_list>
#include <cmath>
#include <cstring>
#include <stdexcept>
#include <cstdlib>
#include <thread>
#include <memory>
#include <unordered_map>

#include "common.cuh"
#include "engine.h"
#include "gguf.h"
#include "kernels.cuh"
#include "layers.cuh"
#include "tp.cuh"
#include "sample.cuh"

namespace qdec {

namespace {

void ck(cudaError_t e, const char* what) {
    if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

__global__ void add_rows_kernel(const float* a, const float* b, float* out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

// Greedy acceptance of a verify batch on the device (spec.rs:352-366): m = the longest prefix where the model's
// argmax equals the draft (vids[1 + i] is draft i); the emitted ids are argmax[0..m] (m + 1 of them).  Then the
// rollback bookkeeping of spec.rs:368-415: the DeltaNet layers will commit `keep` = m + 1 rows, the position
// advances by keep, the MTP is truncated to the round's start p and re-fed the kept rows (MTP positions
// p..p+k, rows past keep are scratch that later rows overwrite before anything reads them), then chained at
// p + keep + i - 1 for draft i + 1.  emit = {keep, emitted ids...}.
__global__ void spec_accept_kernel(const int32_t* __restrict__ argmax, const int32_t* __restrict__ vids, int k, int* pos,
                                   int* keep_out, int* mpos, int32_t* mids, int* sel, int32_t* emit) {
    if (threadIdx.x != 0 || blockIdx.x != 0) return;
    int m = 0;
    while (m < k && argmax[m] == vids[1 + m]) m++;
    const int keep = m + 1;
    const int p = *pos;
    emit[0] = keep;
    for (int i = 0; i <= k; i++) {
        const int32_t a = i < keep ? argmax[i] : argmax[keep - 1];
        if (i < keep) emit[1 + i] = a;
        mids[i] = a;  // MTP re-feed tokens (rows past keep: any valid id)
    }
    *keep_out = keep;
    *pos = p + keep;
    mpos[0] = p;
    for (int i = 1; i < k; i++) mpos[i] = p + keep + i - 1;
    *sel = keep - 1;
}

// The committed DeltaNet state with the `*keep` pending rows of the last call applied (the commit of
// deltanet_halves_kernel: S *= decay_i, then S += k_i (x) delta_i, per row in order), into `out`; one thread per
// state element.
__global__ void debug_commit_state_kernel(const float* __restrict__ S, const float* __restrict__ pend_decay,
                                          const float* __restrict__ pend_k, const float* __restrict__ pend_delta,
                                          const int* __restrict__ keep, int n_v, int dk, int dv, float* __restrict__ out) {
    const size_t e = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (e >= (size_t)n_v * dk * dv) return;
    const int j = (int)(e % dv), k = (int)((e / dv) % dk), p = (int)(e / ((size_t)dk * dv));
    float v = S[e];
    for (int i = 0; i < *keep; i++) {
        v = __fmul_rn(v, pend_decay[(size_t)i * n_v + p]);
        v = __fadd_rn(v, __fmul_rn(pend_k[((size_t)i * n_v + p) * dk + k], pend_delta[((size_t)i * n_v + p) * dv + j]));
    }
    out[e] = v;
}

// The conv window with the `*keep` pending inputs shifted in (conv_step_kernel's commit), into `out`.
__global__ void debug_commit_conv_kernel(const float* __restrict__ state, const float* __restrict__ pend_x,
                                         const int* __restrict__ keep, int channels, int K, float* __restrict__ out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= channels) return;
    float st[8];
    for (int j = 0; j < K - 1; j++) st[j] = state[(size_t)c * (K - 1) + j];
    for (int i = 0; i < *keep; i++) {
        for (int j = 0; j < K - 2; j++) st[j] = st[j + 1];
        if (K >= 2) st[K - 2] = pend_x[(size_t)i * channels + c];
    }
    for (int j = 0; j < K - 1; j++) out[(size_t)c * (K - 1) + j] = st[j];
}

// dst[0..n) = src rows[*sel][0..n)
__global__ void select_row_kernel(const float* __restrict__ src, const int* __restrict__ sel, int n, float* __restrict__ dst) {
    const float* r = src + (size_t)(*sel) * n;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) dst[i] = r[i];
}

}  // namespace

// ------------------------------------------------------------------------------------------------ Model

TpPlan make_tp_plan(const ModelConfig& c, int rank, int world) {
    if (world < 1 || world > 8 || rank < 0 || rank >= world)
        throw ConfigError("tensor parallelism: rank " + std::to_string(rank) + " of " + std::to_string(world) + " (1..8 ranks)");
    auto need = [&](bool ok, const char* what) {
        if (!ok) throw ConfigError("tensor parallelism over " + std::to_string(world) + " GPUs: " + what);
    };
    TpPlan p;
    p.rank = rank;
    p.world = world;
    if (!c.deltanet_layers.empty()) {
        need(c.dn_n_k_heads % world == 0, "the DeltaNet K heads do not divide among the ranks");
        need(c.dn_n_v_heads % c.dn_n_k_heads == 0, "the DeltaNet V heads are not a multiple of the K heads");
        p.nk = (int)c.dn_n_k_heads / world;
        p.kh_lo = rank * p.nk;
        p.nv = p.nk * (int)(c.dn_n_v_heads / c.dn_n_k_heads);
    }
    need(c.n_head % world == 0 && c.n_head_kv > 0 && c.n_head % c.n_head_kv == 0, "the attention heads do not divide among the ranks");
    p.nq = (int)c.n_head / world;
    p.qh_lo = rank * p.nq;
    const int group = (int)(c.n_head / c.n_head_kv);
    if (c.n_head_kv % world == 0) {
        p.nkv = (int)c.n_head_kv / world;
        p.kv_lo = rank * p.nkv;
    } else {
        need(group % p.nq == 0, "a rank's query heads would span two kv heads");
        p.nkv = 1;
        p.kv_lo = p.qh_lo / group;
    }
    need(c.intermediate_size % 256 == 0 && (int)c.intermediate_size / 256 >= world, "the FFN width does not split on 256-row blocks");
    const int nb = (int)c.intermediate_size / 256;
    const int b0 = rank * nb / world, b1 = (rank + 1) * nb / world;
    p.ff_lo = b0 * 256;
    p.ff_rows = (b1 - b0) * 256;
    need(c.hidden_size % (8u * world) == 0, "the hidden size does not split into 8-row tiles");
    p.h_rows = (int)c.hidden_size / world;
    p.h_lo = rank * p.h_rows;
    need(c.vocab_size % (8u * world) == 0, "the vocabulary does not split into 8-row tiles");
    p.v_rows = (int)c.vocab_size / world;
    p.v_lo = rank * p.v_rows;
    return p;
}

Model::~Model() {
    for (void* p : shard_allocs_) cudaFree(p);
    if (blob_) cudaFree(blob_);
    if (rope_cos) cudaFree(rope_cos);
    if (rope_sin) cudaFree(rope_sin);
}

bool Model::is_stop(uint32_t id) const {
    return std::find(cfg.stop_ids.begin(), cfg.stop_ids.end(), id) != cfg.stop_ids.end();
}

// Readers of the weight file: QDEC_LOAD_THREADS, else half the hardware threads, 2..16.
static int load_threads() {
    static const int n = [] {
        const char* e = getenv("QDEC_LOAD_THREADS");
        if (e && atoi(e) > 0) return std::min(atoi(e), 64);
        const int hw = (int)std::thread::hardware_concurrency();
        return std::max(2, std::min(16, hw / 2));
    }();
    return n;
}

// QDEC_LOAD_DIRECT=1: the one-GPU load reads the file with O_DIRECT where its file system allows (buffered
// otherwise; a tensor-parallel rank's per-tensor reads stay buffered).
static bool load_direct() {
    const char* e = getenv("QDEC_LOAD_DIRECT");
    return e && atoi(e) > 0;
}

std::unique_ptr<Model> Model::load(const std::string& path, const LoadOptions& opt) {
    const auto t0 = std::chrono::steady_clock::now();
    Gguf g(path);
    std::unique_ptr<Model> m(new Model());
    m->cfg = ModelConfig::from_gguf(g);
    m->device = opt.device;
    m->max_pos = opt.max_pos;
    m->tp = make_tp_plan(m->cfg, opt.tp_rank, opt.tp_world);
    if (!deltanet_dims_supported((int)m->cfg.dn_head_dim_k, (int)m->cfg.dn_head_dim_v))
        throw ConfigError("no device kernel for DeltaNet heads of key dim " + std::to_string(m->cfg.dn_head_dim_k) + " and value dim " +
                          std::to_string(m->cfg.dn_head_dim_v) + " (key 64 or 128, value 32..128 in steps of 32)");
    if (!attention_dims_supported((int)m->cfg.head_dim_k))
        throw ConfigError("no device kernel for attention heads of dim " + std::to_string(m->cfg.head_dim_k) + " (64..256 in steps of 64)");
    ck(cudaSetDevice(opt.device), "cudaSetDevice");
    const ModelConfig& c = m->cfg;
    const TpPlan& P = m->tp;

    // the data section, unchanged, in one allocation: read in 256 MiB chunks by several threads into pinned
    // staging (two buffers), each chunk's upload overlapping the next chunk's read.  A tensor-parallel rank
    // instead reads what it keeps, each into an allocation of its own: the replicated tensors whole (on first
    // use) and only its rows of the sharded ones -- so a rank holds its share of the model, not all of it.
    const uint64_t data_bytes = g.file_size() - g.data_offset();
    const bool per_rank = P.world > 1;
    m->weight_bytes = per_rank ? 0 : data_bytes;
    if (!per_rank) {
        ck(cudaMalloc(&m->blob_, data_bytes + 256), "weights allocation");
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
        // direct reads start at the block boundary at or before the data section: the `head` bytes before it
        // are read and not uploaded (the staging buffers are page-aligned and CH is a multiple of the boundary)
        const bool direct = load_direct() && g.open_direct();
        const uint64_t head = direct ? g.data_offset() % Gguf::DIRECT_ALIGN : 0, base = g.data_offset() - head;
        const uint64_t total = data_bytes + head;
        m->loaded_direct = direct;
        try {
            for (uint64_t off = 0; off < total; off += CH, b ^= 1) {
                const uint64_t len = std::min<uint64_t>(CH, total - off);
                if (used[b]) ck(cudaEventSynchronize(done[b]), "staging wait");
                uint8_t* hb = static_cast<uint8_t*>(host) + b * CH;
                if (direct) g.read_direct_parallel(base + off, hb, len, load_threads());
                else g.read_at_parallel(base + off, hb, len, load_threads());
                const uint64_t skip = off == 0 ? head : 0;
                ck(cudaMemcpyAsync(m->blob_ + off + skip - head, hb + skip, len - skip, cudaMemcpyHostToDevice, s), "weights upload");
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
    const size_t STG = 64ull << 20;
    std::unique_ptr<void, cudaError_t (*)(void*)> stage(nullptr, cudaFreeHost);
    if (per_rank) {
        void* h = nullptr;
        ck(cudaHostAlloc(&h, STG, cudaHostAllocDefault), "pinned staging");
        stage.reset(h);
    }
    auto upload = [&](uint64_t file_off, uint8_t* dst, uint64_t len) {  // file bytes -> device, STG at a time
        for (uint64_t o = 0; o < len; o += STG) {
            const uint64_t n = std::min<uint64_t>(STG, len - o);
            g.read_at_parallel(file_off + o, stage.get(), n, load_threads());
            ck(cudaMemcpy(dst + o, stage.get(), n, cudaMemcpyHostToDevice), "weights upload");
        }
    };
    auto own_alloc = [&](uint64_t bytes, const char* what) {  // (tensor-parallel) an allocation the rank keeps
        uint8_t* d = nullptr;
        ck(cudaMalloc(&d, bytes + 256), what);
        m->shard_allocs_.push_back(d);
        m->weight_bytes += bytes;
        return d;
    };
    std::unordered_map<const TensorInfo*, uint8_t*> resident;  // (tensor-parallel) tensors already read whole
    auto ptr = [&](const TensorInfo& t) -> uint8_t* {
        if (!per_rank) return m->blob_ + t.rel_offset;
        auto it = resident.find(&t);
        if (it != resident.end()) return it->second;
        uint8_t* d = own_alloc(t.byte_size, "replicated tensor allocation");
        upload(t.abs_offset, d, t.byte_size);
        resident.emplace(&t, d);
        return d;
    };
    // K-quant matrices are repacked in place (same bytes) into the tile layout the GEMV streams (rows % 8 == 0),
    // else Q6_K into the split layout; the embedding table keeps the ggml layout because rows of it are
    // dequantised directly
    uint8_t* repack_tmp = nullptr;
    uint64_t repack_cap = 0;
    for (const TensorInfo& t : g.tensors())
        if ((is_kquant(t.type) || t.type == T_Q8_0 || t.type == T_Q4_0) && t.name != "token_embd.weight")
            repack_cap = std::max(repack_cap, t.byte_size);
    if (repack_cap) ck(cudaMalloc(&repack_tmp, repack_cap), "repack buffer");
    auto repack_at = [&](uint8_t* p, int ttype, uint64_t bytes, int rows, int cols, const std::string& name) -> int {
        ck(cudaMemcpy(repack_tmp, p, bytes, cudaMemcpyDeviceToDevice), "repack copy");
        int type = ttype;
        const bool aligned = rows % 8 == 0 && ((uintptr_t)p & 15) == 0;
        if ((ttype == T_Q8_0 || ttype == T_Q4_0) && aligned && cols % 256 == 0) {
            ck(launch_repack_q80_tiles(ttype, repack_tmp, rows, cols, p, 0), "repack");
            type = ttype == T_Q8_0 ? T_Q8_0_TILE : T_Q4_0_TILE;
        } else if (ttype == T_Q8_0 || ttype == T_Q4_0) {
            throw ConfigError("tensor " + name + ": Q8_0/Q4_0 matrices need rows % 8 == 0 and cols % 256 == 0 here");
        } else if (aligned) {
            ck(launch_repack_tiles(ttype, repack_tmp, rows, cols, p, 0), "repack");
            type = ttype == T_Q4_K ? T_Q4_K_TILE : ttype == T_Q5_K ? T_Q5_K_TILE : T_Q6_K_TILE;
        } else if (ttype == T_Q6_K) {
            ck(launch_repack_q6k(repack_tmp, bytes / 210, p, 0), "repack");
            type = T_Q6_K_SPLIT;
        }
        ck(cudaDeviceSynchronize(), "repack");
        return type;
    };
    auto repack = [&](const TensorInfo& t, int rows, int cols) -> int {
        return repack_at(ptr(t), t.type, t.byte_size, rows, cols, t.name);
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
        if ((is_kquant(t.type) || t.type == T_Q8_0 || t.type == T_Q4_0) && name != "token_embd.weight")
            d.type = repack(t, (int)rows, (int)cols);
        return d;
    };
    auto vec = [&](const std::string& name, uint64_t len) -> const float* {
        const TensorInfo& t = g.tensor(name);
        if (t.n_elements != len) throw ConfigError("tensor " + name + ": expected " + std::to_string(len) + " elements");
        if (t.type != T_F32) throw ConfigError("tensor " + name + ": 1-D weights must be F32 here");
        return reinterpret_cast<const float*>(ptr(t));
    };
    // tensor parallelism: a rank keeps the rows `segs` ({first row, count} in order) of a sharded tensor, copied
    // out of the uploaded data section into an allocation of its own (then repacked like a whole matrix)
    using Segs = std::vector<std::pair<uint64_t, uint64_t>>;
    auto shard_copy = [&](const TensorInfo& t, uint64_t row_bytes, const Segs& segs, uint64_t& nrows) -> uint8_t* {
        nrows = 0;
        for (const auto& sg : segs) nrows += sg.second;
        uint8_t* d = own_alloc(nrows * row_bytes, "shard allocation");
        uint64_t o = 0;
        for (const auto& sg : segs) {
            if (per_rank && !resident.count(&t)) upload(t.abs_offset + sg.first * row_bytes, d + o, sg.second * row_bytes);
            else ck(cudaMemcpy(d + o, ptr(t) + sg.first * row_bytes, sg.second * row_bytes, cudaMemcpyDeviceToDevice), "shard copy");
            o += sg.second * row_bytes;
        }
        return d;
    };
    auto mat_rows = [&](const std::string& name, uint64_t rows, uint64_t cols, const Segs& segs) {
        if (P.world == 1) return mat(name, rows, cols);
        const TensorInfo& t = g.tensor(name);
        const auto sh = t.shape_numpy();
        if (sh.size() != 2 || sh[0] != rows || sh[1] != cols)
            throw ConfigError("tensor " + name + ": expected shape [" + std::to_string(rows) + ", " + std::to_string(cols) + "]");
        if (!(t.type == T_F32 || t.type == T_Q4_0 || t.type == T_Q8_0 || is_kquant(t.type)))
            throw ConfigError("tensor " + name + ": no kernel for ggml type " + std::to_string(t.type));
        const uint64_t rb = t.byte_size / rows;
        uint64_t n = 0;
        uint8_t* d = shard_copy(t, rb, segs, n);
        DevMat dm;
        dm.type = t.type;
        dm.rows = (int)n;
        dm.cols = (int)cols;
        dm.p = d;
        dm.bytes = n * rb;
        if (is_kquant(t.type) || t.type == T_Q8_0 || t.type == T_Q4_0) dm.type = repack_at(d, t.type, dm.bytes, (int)n, (int)cols, name);
        return dm;
    };
    auto vec_rows = [&](const std::string& name, uint64_t len, uint64_t per, const Segs& segs) -> const float* {
        const float* full = vec(name, len);
        if (P.world == 1) return full;
        uint64_t n = 0;
        return reinterpret_cast<const float*>(shard_copy(g.tensor(name), per * 4, segs, n));
    };
    const uint64_t H = c.hidden_size;
    const Segs hseg{{(uint64_t)P.h_lo, (uint64_t)P.h_rows}};
    m->embed = mat("token_embd.weight", c.vocab_size, H);
    m->lm_head = mat_rows(c.tie_word_embeddings ? "token_embd.weight" : "output.weight", c.vocab_size, H,
                          Segs{{(uint64_t)P.v_lo, (uint64_t)P.v_rows}});
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
            L.q = mat_rows(p + "attn_q.weight", 2ull * c.n_head * hd, H, Segs{{2ull * P.qh_lo * hd, 2ull * P.nq * hd}});
            L.k = mat_rows(p + "attn_k.weight", (uint64_t)c.n_head_kv * hd, H, Segs{{(uint64_t)P.kv_lo * hd, (uint64_t)P.nkv * hd}});
            L.v = mat_rows(p + "attn_v.weight", (uint64_t)c.n_head_kv * hd, H, Segs{{(uint64_t)P.kv_lo * hd, (uint64_t)P.nkv * hd}});
            L.o = mat_rows(p + "attn_output.weight", H, (uint64_t)c.n_head * hd, hseg);
            L.q_norm = vec(p + "attn_q_norm.weight", hd);
            L.k_norm = vec(p + "attn_k_norm.weight", hd);
        } else {
            // this rank's K heads (q and k rows) and the V heads tied to them (v rows, gate rows, per-head scalars)
            const uint64_t dk = c.dn_head_dim_k, dv = c.dn_head_dim_v, nkg = c.dn_n_k_heads, G = c.dn_n_v_heads / nkg;
            Segs qkv_rows{{P.kh_lo * dk, P.nk * dk}, {nkg * dk + P.kh_lo * dk, P.nk * dk}}, v_rows, head_rows;
            for (uint64_t gi = 0; gi < G; gi++) {
                qkv_rows.push_back({2 * nkg * dk + (gi * nkg + P.kh_lo) * dv, P.nk * dv});
                v_rows.push_back({(gi * nkg + P.kh_lo) * dv, P.nk * dv});
                head_rows.push_back({gi * nkg + P.kh_lo, (uint64_t)P.nk});
            }
            L.qkv = mat_rows(p + "attn_qkv.weight", c.dn_qkv_dim, H, qkv_rows);
            L.gate_z = mat_rows(p + "attn_gate.weight", c.dn_v_dim, H, v_rows);
            L.alpha = mat_rows(p + "ssm_alpha.weight", c.dn_n_v_heads, H, head_rows);
            L.beta = mat_rows(p + "ssm_beta.weight", c.dn_n_v_heads, H, head_rows);
            L.ssm_a = vec_rows(p + "ssm_a", c.dn_n_v_heads, 1, head_rows);
            L.dt_bias = vec_rows(p + "ssm_dt.bias", c.dn_n_v_heads, 1, head_rows);
            L.conv_w = vec_rows(p + "ssm_conv1d.weight", (uint64_t)c.dn_qkv_dim * c.dn_conv_kernel, c.dn_conv_kernel, qkv_rows);
            L.ssm_norm = vec(p + "ssm_norm.weight", c.dn_head_dim_v);
            L.ssm_out = mat_rows(p + "ssm_out.weight", H, c.dn_v_dim, hseg);
        }
        const Segs ffseg{{(uint64_t)P.ff_lo, (uint64_t)P.ff_rows}};
        L.ffn_gate = mat_rows(p + "ffn_gate.weight", c.intermediate_size, H, ffseg);
        L.ffn_up = mat_rows(p + "ffn_up.weight", c.intermediate_size, H, ffseg);
        L.ffn_down = mat_rows(p + "ffn_down.weight", H, c.intermediate_size, hseg);
        return L;
    };
    for (uint32_t i = 0; i < c.n_layer; i++) m->layers.push_back(load_layer(i, c.is_attention(i)));
    if (!c.mtp_layers.empty()) {
        const uint32_t mi = c.mtp_layers[0];
        const std::string p = "blk." + std::to_string(mi) + ".nextn.";
        m->mtp.block = load_layer(mi, true);
        m->mtp.eh_proj = mat_rows(p + "eh_proj.weight", H, 2 * H, hseg);
        m->mtp.enorm = vec(p + "enorm.weight", H);
        m->mtp.hnorm = vec(p + "hnorm.weight", H);
        m->mtp.head_norm = vec(p + "shared_head_norm.weight", H);
        m->has_mtp = true;
    }
    // RoPE tables (rope.rs:10-29): inv_freq[i] = 1 / theta^(2i / rope_dim) in f32, angle = f32(pos) * inv_freq,
    // cos/sin in f32, each half duplicated -- computed on the host with the C library, like the reference
    const int rd = (int)c.rope_dim, half = rd / 2;
    // (ROPE_SLACK extra positions: the MTP rows of a speculative round run up to 2k past the sequence end)
    const int npos = opt.max_pos + ROPE_SLACK;
    std::vector<float> inv(half), cs((size_t)npos * rd), sn((size_t)npos * rd);
    for (int i = 0; i < half; i++) inv[i] = 1.0f / powf(c.rope_freq_base, (float)(2 * i) / (float)rd);
    for (int pos = 0; pos < npos; pos++) {
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
    if (P.world > 1) {  // the bytes this rank streams: its matrix slices (the small replicated vectors left out)
        auto mats = [](const LayerW& L) {
            uint64_t b = 0;
            for (const DevMat* d : {&L.qkv, &L.gate_z, &L.alpha, &L.beta, &L.ssm_out, &L.q, &L.k, &L.v, &L.o, &L.ffn_gate, &L.ffn_up,
                                    &L.ffn_down})
                b += d->bytes;
            return b;
        };
        uint64_t lb = 0;
        for (const LayerW& L : m->layers) lb += mats(L);
        m->decode_bytes = lb + m->lm_head.bytes + 4ull * H + m->embed.bytes / c.vocab_size;
        if (m->has_mtp) m->mtp_bytes = mats(m->mtp.block) + m->mtp.eh_proj.bytes;
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
    static std::atomic<uint64_t> serials{0};
    serial_ = ++serials;
    const ModelConfig& c = m.cfg;
    if (max_pos > m.max_pos) throw std::invalid_argument("max_pos exceeds the model's RoPE table");
    if (spec_k < 0 || 2 * spec_k + 2 > ROPE_SLACK) throw std::invalid_argument("spec_k out of range");
    mtp_cap_ = max_pos + 2 * spec_k + 2;
    if (spec_k > 0 && !m.has_mtp) throw std::invalid_argument("the GGUF has no MTP block (no nextn tensors): speculative decoding needs one");
    T_ = std::max(max_rows, spec_k + 1);
    ck(cudaSetDevice(m.device), "cudaSetDevice");
    ck(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "stream");
    ck(cudaMallocHost(&err_io_, 2 * sizeof(unsigned)), "pinned error words");
    err_io_[0] = err_io_[1] = 0;
    const size_t H = c.hidden_size, FF = c.intermediate_size, T = T_;
    size_t maxw = std::max<size_t>(std::max<size_t>(2 * H, FF), std::max<size_t>(c.dn_v_dim, (size_t)c.n_head * c.head_dim_k));
    q8k_stride_ = maxw / 256 * Q8K_IMG_BYTES;  // the Q8_K device image
    q80_stride_ = maxw / 32 * Q80_IMG_BYTES;  // the Q8_0 row image
    d_ids = (int32_t*)dalloc(T * 4);
    d_argmax = (int32_t*)dalloc(T * 4);
    d_pos = (int*)dalloc(4);
    d_keep = (int*)dalloc(4);
    d_mtp_pos = (int*)dalloc(4);
    amx_scratch_ = dalloc(argmax_scratch_bytes((int)c.vocab_size, (int)T));  // zero-filled by dalloc
    h_ = (float*)dalloc(T * H * 4);
    h_alt_ = (float*)dalloc(T * H * 4);
    embed_ = (float*)dalloc(T * H * 4);
    normed_ = (float*)dalloc(T * maxw * 4);
    mix_out_ = (float*)dalloc(T * H * 4);
    mlp_out_ = (float*)dalloc(T * H * 4);
    q8k_ = (uint8_t*)dalloc(T * q8k_stride_);
    q80_ = (uint8_t*)dalloc(T * q80_stride_);
    ffn_img_ = (uint8_t*)dalloc(T * q8k_stride_);
    ffn_cnt_ = (unsigned*)dalloc((c.intermediate_size / 256 + 1) * sizeof(unsigned));
    dn_cnt_ = (unsigned*)dalloc((c.dn_v_dim / 256 + 1) * sizeof(unsigned));
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
    // attention scores of every row and query head over the longest cache (the MTP cache's)
    att_scores_ = (float*)dalloc(T * c.n_head * (((size_t)std::max(max_pos, mtp_cap_) + 3) & ~(size_t)3) * 4);
    gate_ = (float*)dalloc(T * qd * 4);
    attn_ = (float*)dalloc(T * qd * 4);
    // the persistent per-layer state covers this rank's heads (all of them on one GPU)
    const TpPlan& P = m.tp;
    const size_t kvd_r = (size_t)P.nkv * hd;
    const size_t qkv_r = 2 * (size_t)P.nk * c.dn_head_dim_k + (size_t)P.nv * c.dn_head_dim_v;
    for (const LayerW& L : m.layers) {
        if (L.attn) {
            kv_.push_back({(float*)dalloc((size_t)max_pos * kvd_r * 4), (float*)dalloc((size_t)max_pos * kvd_r * 4)});
            dn_.push_back({});
        } else {
            DnState d;
            d.S = (float*)dalloc((size_t)P.nv * c.dn_head_dim_k * c.dn_head_dim_v * 4);
            d.conv = (float*)dalloc(qkv_r * (c.dn_conv_kernel - 1) * 4);
            d.pend_x = (float*)dalloc(T * qkv_r * 4);
            d.pend_decay = (float*)dalloc(T * P.nv * 4);
            d.pend_k = (float*)dalloc(T * P.nv * c.dn_head_dim_k * 4);
            d.pend_delta = (float*)dalloc(T * P.nv * c.dn_head_dim_v * 4);
            dn_.push_back(d);
            kv_.push_back({});
        }
    }
    if (P.world > 1) {
        // the exchange block: two line buffers (2 bytes of lines per byte of the largest exchange), then the
        // receive buffers (full-width rows)
        const size_t ext = std::max({T * H * 4, T * std::max<size_t>(c.dn_v_dim, 1) * 4, T * qd * 4,
                                     T * std::max<size_t>(FF / 256 * Q8K_IMG_BYTES, FF / 32 * Q80_IMG_BYTES), T * 8 * 16});
        xll_bytes_ = (2 * ext + 255) & ~(size_t)255;
        size_t off = 2 * xll_bytes_;
        auto take = [&](size_t bytes) {
            const size_t o = off;
            off += (bytes + 255) & ~(size_t)255;
            return o;
        };
        xo_mix_ = take(T * H * 4);
        xo_mlp_ = take(T * H * 4);
        xo_eh_ = take(T * H * 4);
        xo_heads_ = take(T * std::max<size_t>(c.dn_v_dim, 1) * 4);
        xo_attn_ = take(T * qd * 4);
        xo_ffn_ = take(T * std::max<size_t>(FF / 256 * Q8K_IMG_BYTES, FF / 32 * Q80_IMG_BYTES));
        xo_amx_ = take(T * 8 * 16);
        xo_pad_ = take(8 * 16);
        xblk_bytes_ = off;
        xblk_ = (uint8_t*)dalloc(xblk_bytes_);
        xpeer_[P.rank] = xblk_;
        xepoch_ = (unsigned*)dalloc(4);
        xerr_ = (unsigned*)dalloc(4);
        xstats_ = (unsigned long long*)dalloc(4 * 8);
        amx_pairs_ = (uint8_t*)dalloc(T * 16);
    }
    if (m.has_mtp) {
        mtp_kv_ = {(float*)dalloc((size_t)mtp_cap_ * kvd_r * 4), (float*)dalloc((size_t)mtp_cap_ * kvd_r * 4)};
        d_vids = (int32_t*)dalloc(T * 4);
        d_mids = (int32_t*)dalloc(T * 4);
        d_mpos = (int*)dalloc(T * 4);
        d_sel = (int*)dalloc(4);
        d_emit = (int32_t*)dalloc((T + 2) * 4);
        ck(cudaMallocHost(&h_io_, 64 * 4), "pinned round buffer");
        cat_ = (float*)dalloc(T * 2 * H * 4);
        mtp_h_ = (float*)dalloc(T * H * 4);
        mtp_hout_ = (float*)dalloc(T * H * 4);
    }
    counters.hist.assign(spec_k + 1, 0);
    ck(cudaDeviceSynchronize(), "state init");  // the zeroed flags are in place before the block is exported
}

State::~State() {
    if (stream) cudaStreamSynchronize(stream);
    for (int k = 0; k < m_.tp.world; k++)
        if (k != m_.tp.rank && xpeer_[k]) cudaIpcCloseMemHandle(xpeer_[k]);
    if (round_exec_) cudaGraphExecDestroy(round_exec_);
    if (step_exec_) cudaGraphExecDestroy(step_exec_);
    if (batch_exec_) cudaGraphExecDestroy(batch_exec_);
    if (h_io_) cudaFreeHost(h_io_);
    if (err_io_) cudaFreeHost(err_io_);
    for (void* p : allocs_) cudaFree(p);
    for (float* p : capture_h_) cudaFree(p);
    if (stream) cudaStreamDestroy(stream);
}

void State::sync() {
    // the error words travel with the stream's work: one synchronisation, no extra round trip per call
    ck(enqueue_kernel_error_read(err_io_, stream), "error words");
    ck(cudaStreamSynchronize(stream), "decode step");
    if (err_io_[0] || err_io_[1]) {
        const unsigned err = err_io_[0] ? err_io_[0] : err_io_[1];
        read_kernel_error(true);  // cleared for the calls after this one
        throw std::runtime_error("a device-side wait gave up (code " + std::to_string(err) + ")");
    }
    if (tp()) {
        unsigned xe = 0;
        ck(cudaMemcpy(&xe, xerr_, 4, cudaMemcpyDeviceToHost), "exchange status");
        if (xe) {
            const unsigned z = 0;
            cudaMemcpy(xerr_, &z, 4, cudaMemcpyHostToDevice);
            throw std::runtime_error("tensor-parallel exchange: the poll gave up, a peer's slice did not arrive in time (slot " +
                                     std::to_string(xe & 0xffff) + ")");
        }
    }
}

void State::tp_export(void* out) const {
    if (!tp()) throw std::logic_error("tp_export: not a tensor-parallel state");
    cudaIpcMemHandle_t h;
    ck(cudaIpcGetMemHandle(&h, xblk_), "exchange export");
    uint8_t* o = static_cast<uint8_t*>(out);
    std::memset(o, 0, TP_HANDLE_BYTES);
    std::memcpy(o, &h, sizeof h);
    const uint64_t bytes = xblk_bytes_;
    const int32_t rw[2] = {m_.tp.rank, m_.tp.world};
    std::memcpy(o + 64, &bytes, 8);
    std::memcpy(o + 72, rw, 8);
}

void State::tp_connect(const void* handles) {
    if (!tp()) throw std::logic_error("tp_connect: not a tensor-parallel state");
    if (tp_connected_) throw std::logic_error("tp_connect: already connected");
    const uint8_t* in = static_cast<const uint8_t*>(handles);
    for (int k = 0; k < m_.tp.world; k++) {
        const uint8_t* hk = in + (size_t)k * TP_HANDLE_BYTES;
        uint64_t bytes = 0;
        int32_t rw[2];
        std::memcpy(&bytes, hk + 64, 8);
        std::memcpy(rw, hk + 72, 8);
        if (rw[0] != k || rw[1] != m_.tp.world)
            throw std::invalid_argument("tp_connect: handle " + std::to_string(k) + " is not rank " + std::to_string(k) + "'s");
        if (bytes != xblk_bytes_)
            throw std::invalid_argument("tp_connect: rank " + std::to_string(k) + " built its state with other sizes (spec_k, max_rows)");
    }
    for (int k = 0; k < m_.tp.world; k++) {
        if (k == m_.tp.rank) continue;
        cudaIpcMemHandle_t h;
        std::memcpy(&h, in + (size_t)k * TP_HANDLE_BYTES, sizeof h);
        void* p = nullptr;
        ck(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess), "exchange import");
        xpeer_[k] = static_cast<uint8_t*>(p);
    }
    tp_connected_ = true;
}

void State::tp_stats(uint64_t out[4]) const {
    for (int i = 0; i < 4; i++) out[i] = 0;
    if (!tp()) return;
    ck(cudaStreamSynchronize(stream), "sync");
    ck(cudaMemcpy(out, xstats_, 4 * 8, cudaMemcpyDeviceToHost), "exchange stats");
}

void State::begin_session() {
    if (!tp()) return;
    if (!tp_connected_) throw std::logic_error("tensor-parallel state used before tp_connect");
    count_launch();
    ck(launch_tp_epoch(xepoch_, stream), "epoch");
    xslot_ = 0;
}

void State::exchange(const void* src, size_t src_ld, size_t dst_off, size_t dst_ld, const int (*segs)[3], int nseg, int rows) {
    if (xslot_ >= XSLOTS) throw std::logic_error("exchange: too many exchanges in one session");
    if ((size_t)rows * dst_ld * 2 > xll_bytes_) throw std::logic_error("exchange: larger than the line buffers");
    XArgs a{};
    a.src = static_cast<const uint8_t*>(src);
    a.src_ld = (long long)src_ld;
    a.dst_ld = (long long)dst_ld;
    a.nseg = nseg;
    a.rows = rows;
    for (int i = 0; i < nseg; i++) a.seg_src[i] = segs[i][0], a.seg_dst[i] = segs[i][1], a.seg_len[i] = segs[i][2];
    const size_t ll = (xseq_++ & 1) * xll_bytes_;  // consecutive exchanges alternate between the line buffers
    for (int k = 0; k < m_.tp.world; k++) a.ll[k] = xpeer_[k] + ll;
    a.ll_local = xblk_ + ll;
    a.out = xblk_ + dst_off;
    a.epoch = xepoch_;
    a.err = xerr_;
    a.stats = xstats_;
    a.slot = xslot_++;
    a.rank = m_.tp.rank;
    a.world = m_.tp.world;
    count_launch();
    ck(launch_exchange(a, stream), "exchange");
}

// Greedy ids of t logits rows: on one GPU the argmax kernel; over TP ranks each rank reduces its vocabulary
// slice to (value, global index), the pairs are exchanged and combined in rank order with the strict > rule,
// which is the whole row's first maximum (model.rs:505-513).
void State::argmax_rows(const float* logits, int t, int32_t* out_dev) {
    if (!tp()) {
        count_launch();
        ck(launch_argmax(logits, (int)m_.cfg.vocab_size, t, out_dev, amx_scratch_, stream), "argmax");
        return;
    }
    const TpPlan& P = m_.tp;
    count_launch();
    ck(launch_argmax_pairs(logits, P.v_rows, t, amx_pairs_, P.v_lo, P.rank == 0, amx_scratch_, stream), "argmax");
    const int seg[1][3] = {{0, 16 * P.rank, 16}};
    exchange(amx_pairs_, 16, xo_amx_, 16 * (size_t)P.world, seg, 1, t);
    count_launch();
    ck(launch_argmax_combine(xblk_ + xo_amx_, P.world, t, out_dev, stream), "argmax combine");
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
    for (int t : ts) if (is_q80(t)) return true;
    return false;
}

void State::gemv(const DevMat& w, const float* normed_f32, int rows, float* y, const uint8_t* img) {
    // activation rows are laid out back to back at the stride of this weight's width; `img` (when given)
    // replaces the state's own Q8_K / Q8_0 image
    if (is_kquant(w.type)) {
        // weights are written once at load, so the GEMV may stream them before its predecessor finishes
        count_launch((rows + 3) / 4);
        ck(launch_gemv_img(w.type, w.p, w.rows, w.cols, img ? img : q8k_, rows, y, stream, true), "gemv");
        return;
    }
    if (w.type == T_Q8_0_TILE || w.type == T_Q4_0_TILE) {
        count_launch((rows + 3) / 4);
        ck(launch_gemv_q80_img(w.type, w.p, w.rows, w.cols, img ? img : q80_, rows, y, stream, true), "gemv");
        return;
    }
    if (w.type != T_F32) throw std::logic_error("gemv: a Q8_0/Q4_0 matrix outside the tile layout");
    count_launch((rows + 3) / 4);
    ck(launch_gemv(w.type, w.p, w.rows, w.cols, normed_f32, rows, y, stream), "gemv");
}

// h = h + delta (delta null: h as it is) into the other residual buffer, normed and quantised on the way.
void State::resid_norm(const float* delta, const float* w, int t, float* y_out, bool k8, bool k0) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    count_launch();
    ck(launch_resid_norm_quant(h_, delta, delta ? h_alt_ : nullptr, w, c.rms_norm_eps, H, t, y_out, k8 ? q8k_ : nullptr,
                               k0 ? q80_ : nullptr, stream),
       "rmsnorm");
    if (delta) std::swap(h_, h_alt_);
}

void State::quant_for(int type, const float* x, int n, int rows) {
    count_launch(); ck(launch_quant_rows(x, n, rows, is_kquant(type) ? q8k_ : nullptr, is_q80(type) ? q80_ : nullptr, stream),
       "quantise");
}

// One decoder layer over t rows (layers/mod.rs:335-377): the residual stream h_ enters as (h_ + mlp_in()) of
// the previous layer (or the layer input `first_in` for layer 0 / the MTP block), leaves in h_ + mlp_in().
// Over TP ranks the matrices produce this rank's rows; the head outputs, the mixer output, the SwiGLU image
// and the FFN output are exchanged so that every rank continues from the full rows.
void State::layer_forward(const LayerW& L, int li, int t, KvState* kv, const int* pos_dev, bool commit_dn) {
    const ModelConfig& c = m_.cfg;
    const TpPlan& P = m_.tp;
    const int H = (int)c.hidden_size;
    const float eps = c.rms_norm_eps;
    if (L.attn) {
        const int hd = (int)c.head_dim_k;
        const bool k8 = needs_q8k({L.q.type, L.k.type, L.v.type}), k0 = needs_q80({L.q.type, L.k.type, L.v.type});
        resid_norm(li == 0 ? nullptr : mlp_in(), L.attn_norm, t, normed_, k8, k0);
        gemv(L.q, normed_, t, qg_);
        gemv(L.k, normed_, t, kk_);
        gemv(L.v, normed_, t, vv_);
        // the rows' own positions and KV caches: all t rows this state's, or (batch_step) row i member i's
        const size_t nqh = (size_t)P.nq * hd;  // floats per row of q, gate and the attention output
        for (int i = 0; i < (batch_ ? t : 1); i++) {
            State* o = batch_ ? (*batch_)[i] : this;
            const int r0 = batch_ ? i : 0, tn = batch_ ? 1 : t;
            KvState* kvo = batch_ ? &o->kv_[li] : kv;
            const int* po = batch_ ? o->d_pos : pos_dev;
            QkArgs qa{qg_ + (size_t)r0 * L.q.rows, kk_ + (size_t)r0 * L.k.rows, vv_ + (size_t)r0 * L.v.rows, L.q_norm, L.k_norm,
                      m_.rope_cos, m_.rope_sin, po, qr_ + r0 * nqh, gate_ + r0 * nqh, kvo->k, kvo->v, P.nq, P.nkv, hd,
                      (int)c.rope_dim, eps};
            count_launch(); ck(launch_qk_norm_rope(qa, tn, stream), "qk_norm_rope");
            AttnArgs aa{qr_ + r0 * nqh, gate_ + r0 * nqh, kvo->k, kvo->v, po, attn_ + r0 * nqh, P.nq, P.nkv, hd,
                        batch_ ? o->max_pos_ : kv == &mtp_kv_ ? mtp_cap_ : max_pos_,
                        m_.attn_scaling, batch_ ? o->att_scores_ : att_scores_};
            count_launch(3); ck(launch_attention(aa, tn, stream), "attention");  // scores, softmax, values
        }
        const float* attn_full = attn_;
        if (tp()) {
            const int seg[1][3] = {{0, P.qh_lo * hd * 4, P.nq * hd * 4}};
            exchange(attn_, (size_t)P.nq * hd * 4, xo_attn_, (size_t)c.n_head * hd * 4, seg, 1, t);
            attn_full = xg(xo_attn_);
        }
        quant_for(L.o.type, attn_full, L.o.cols, t);
        gemv(L.o, attn_full, t, mix_out_);
    } else {
        const bool k8 = needs_q8k({L.qkv.type, L.gate_z.type, L.alpha.type, L.beta.type});
        const bool k0 = needs_q80({L.qkv.type, L.gate_z.type, L.alpha.type, L.beta.type});
        resid_norm(li == 0 ? nullptr : mlp_in(), L.attn_norm, t, normed_, k8, k0);
        gemv(L.qkv, normed_, t, qkv_);
        gemv(L.gate_z, normed_, t, z_);
        const bool ab_fused = L.alpha.type == T_F32 && L.beta.type == T_F32 && L.alpha.cols == H && L.beta.cols == H &&
                              t <= 8 && H <= 5120 && H % 4 == 0;
        if (ab_fused) {
            // the DeltaNet kernel computes alpha and beta of its head itself (before its wait, alongside the conv)
        } else if (L.alpha.type == T_F32 && L.beta.type == T_F32 && L.alpha.cols == L.beta.cols) {
            // ssm_alpha and ssm_beta read the same normed rows: one launch (gated_deltanet.rs:148-149)
            count_launch();
            // normed_ comes from the norm two launches back: the pair runs alongside the gate_z GEMV
            ck(launch_gemv_f32_pair((const float*)L.alpha.p, L.alpha.rows, alpha_, (const float*)L.beta.p, L.beta.rows, beta_,
                                    L.alpha.cols, normed_, t, stream, true),
               "alpha/beta");
        } else {
            gemv(L.alpha, normed_, t, alpha_);
            gemv(L.beta, normed_, t, beta_);
        }
        const int channels = L.qkv.rows;  // this rank's q, k and v channels
        const int dk = (int)c.dn_head_dim_k, dv = (int)c.dn_head_dim_v, nvdv = P.nv * dv;
        // one GPU: the kernel also quantises its head outputs for ssm_out (over TP ranks the f32 heads are
        // exchanged first and the full rows quantised after)
        const int ot = L.ssm_out.type;
        const bool q_fused = !tp() && (is_kquant(ot) || is_q80(ot)) && 256 % dv == 0 && nvdv % 256 == 0;
        // the rows' own conv windows and recurrent states: all t rows this state's, or (batch_step) row i
        // member i's
        for (int i = 0; i < (batch_ ? t : 1); i++) {
            const State* o = batch_ ? (*batch_)[i] : this;
            const int r0 = batch_ ? i : 0, tn = batch_ ? 1 : t;
            const DnState& d = o->dn_[li];
            const int* keep = commit_dn ? o->d_keep : nullptr;
            count_launch(); ck(launch_conv_step(d.conv, L.conv_w, (int)c.dn_conv_kernel, channels, qkv_ + (size_t)r0 * channels, tn,
                                conved_ + (size_t)r0 * channels, d.pend_x, keep, o->T_, stream), "conv");
            DeltaArgs da{d.S, conved_ + (size_t)r0 * channels, alpha_ + (size_t)r0 * P.nv, beta_ + (size_t)r0 * P.nv,
                         z_ + (size_t)r0 * L.gate_z.rows, L.ssm_a, L.dt_bias, L.ssm_norm, heads_ + (size_t)r0 * nvdv,
                         d.pend_decay, d.pend_k, d.pend_delta, keep, tn, o->T_, P.nk, P.nv, dk, dv, P.nk * dk, channels, eps,
                         ab_fused ? (const float*)L.alpha.p : nullptr, ab_fused ? (const float*)L.beta.p : nullptr,
                         ab_fused ? normed_ + (size_t)r0 * H : nullptr, H,
                         q_fused && is_kquant(ot) ? q8k_ + (size_t)r0 * (nvdv / 256) * Q8K_IMG_BYTES : nullptr,
                         q_fused && is_q80(ot) ? q80_ + (size_t)r0 * (nvdv / 32) * Q80_IMG_BYTES : nullptr, dn_cnt_};
            count_launch(); ck(launch_deltanet_heads(da, stream), "deltanet");
        }
        const float* heads_full = heads_;
        if (tp()) {
            // local V heads g * nk + j are global heads g * n_k + kh_lo + j
            const int G = (int)(c.dn_n_v_heads / c.dn_n_k_heads);
            int seg[4][3];
            for (int gi = 0; gi < G; gi++) {
                seg[gi][0] = gi * P.nk * dv * 4;
                seg[gi][1] = (gi * (int)c.dn_n_k_heads + P.kh_lo) * dv * 4;
                seg[gi][2] = P.nk * dv * 4;
            }
            exchange(heads_, (size_t)P.nv * dv * 4, xo_heads_, (size_t)c.dn_v_dim * 4, seg, G, t);
            heads_full = xg(xo_heads_);
        }
        if (!q_fused) quant_for(L.ssm_out.type, heads_full, L.ssm_out.cols, t);
        gemv(L.ssm_out, heads_full, t, mix_out_);
    }
    if (tp()) {
        const int seg[1][3] = {{0, P.h_lo * 4, P.h_rows * 4}};
        exchange(mix_out_, (size_t)P.h_rows * 4, xo_mix_, (size_t)H * 4, seg, 1, t);
    }
    // h = x + mixer(x); then the MLP on post_attention_norm(h) (mlp.rs:53-64)
    const bool k8 = needs_q8k({L.ffn_gate.type, L.ffn_up.type}), k0 = needs_q80({L.ffn_gate.type, L.ffn_up.type});
    resid_norm(mix_in(), L.post_norm, t, normed_, k8, k0);
    const int dt = L.ffn_down.type;
    const int ffr = L.ffn_gate.rows;  // this rank's FFN rows
    // gate, up, silu(gate) * up and its Q8_K quantisation in one launch (the verify's and decode's few columns;
    // a prompt chunk takes the tensor-core GEMM and the separate step)
    const bool fused = L.ffn_gate.type == L.ffn_up.type && L.ffn_gate.rows == L.ffn_up.rows && L.ffn_gate.cols == L.ffn_up.cols &&
                       gemv7_supported(L.ffn_gate.type) && is_kquant(dt) && ffr % 256 == 0 &&
                       !gemm_tc_applies(L.ffn_gate.type, t);
    const uint8_t* down_img = nullptr;  // the down projection's input image: the fused launch's, else the default
    if (fused) {
        count_launch((t + 3) / 4);
        ck(launch_gemv7_swiglu(L.ffn_gate.type, L.ffn_gate.p, L.ffn_up.p, ffr, L.ffn_gate.cols, q8k_, t, g_, ffn_img_, ffn_cnt_,
                               stream, true),
           "gate/up/swiglu");
        down_img = ffn_img_;
    } else if (L.ffn_gate.type == L.ffn_up.type && L.ffn_gate.cols == L.ffn_up.cols &&
        (L.ffn_gate.type == T_Q4_K_TILE || L.ffn_gate.type == T_Q5_K_TILE || L.ffn_gate.type == T_Q6_K_TILE)) {
        // gate and up read the same normed rows: one launch over both (mlp.rs:55, matvec2)
        count_launch((t + 3) / 4);
        ck(launch_gemv_img_pair(L.ffn_gate.type, L.ffn_gate.p, L.ffn_gate.rows, g_, L.ffn_up.p, L.ffn_up.rows, u_, L.ffn_gate.cols,
                                q8k_, t, stream, true),
           "gate/up");
    } else {
        gemv(L.ffn_gate, normed_, t, g_);
        gemv(L.ffn_up, normed_, t, u_);
    }
    if (!fused) {
        count_launch(); ck(launch_swiglu_quant(g_, u_, ffr, t, nullptr, is_kquant(dt) ? q8k_ : nullptr,
                               is_q80(dt) ? q80_ : nullptr, stream), "swiglu");
    }
    if (tp()) {
        const size_t FF = c.intermediate_size;
        if (is_kquant(dt)) {
            const int seg[1][3] = {{0, P.ff_lo / 256 * Q8K_IMG_BYTES, ffr / 256 * Q8K_IMG_BYTES}};
            exchange(down_img ? down_img : q8k_, (size_t)ffr / 256 * Q8K_IMG_BYTES, xo_ffn_, FF / 256 * Q8K_IMG_BYTES, seg, 1, t);
        } else {
            // Q8_0 image row: [codes: 32 B per block][{d, sum}: 8 B per block]
            const int seg[2][3] = {{0, P.ff_lo, ffr}, {ffr, (int)FF + P.ff_lo / 32 * 8, ffr / 32 * 8}};
            exchange(q80_, (size_t)ffr / 32 * Q80_IMG_BYTES, xo_ffn_, FF / 32 * Q80_IMG_BYTES, seg, 2, t);
        }
        gemv(L.ffn_down, g_, t, mlp_out_, xblk_ + xo_ffn_);
        const int seg[1][3] = {{0, P.h_lo * 4, P.h_rows * 4}};
        exchange(mlp_out_, (size_t)P.h_rows * 4, xo_mlp_, (size_t)H * 4, seg, 1, t);
    } else {
        gemv(L.ffn_down, g_, t, mlp_out_, down_img);
    }
}

void State::forward_rows(int t, const int32_t* ids_dev, bool want_logits_all) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    begin_session();
    count_launch(); ck(launch_dequant_rows(m_.embed.type, m_.embed.p, m_.embed.bytes / m_.embed.rows, H, ids_dev, t, h_, stream), "embed");
    for (size_t li = 0; li < m_.layers.size(); li++) {
        layer_forward(m_.layers[li], (int)li, t, &kv_[li], d_pos, true);
        if (capture_) {
            if (capture_h_.size() < m_.layers.size() + 1) {
                capture_h_.assign(m_.layers.size() + 1, nullptr);
                for (auto& p : capture_h_) ck(cudaMalloc(&p, (size_t)T_ * H * 4), "capture buffer");
            }
            add_rows_kernel<<<64, 256, 0, stream>>>(h_, mlp_in(), capture_h_[li], (size_t)t * H);
        }
    }
    // final norm (model.rs:430-438): the post-norm rows are what the lm_head and the MTP read
    const int ht = m_.lm_head.type;
    resid_norm(mlp_in(), m_.output_norm, t, final_, is_kquant(ht), is_q80(ht));
    if (capture_ && !capture_h_.empty())
        ck(cudaMemcpyAsync(capture_h_[m_.layers.size()], final_, (size_t)t * H * 4, cudaMemcpyDeviceToDevice, stream), "capture");
    if (want_logits_all) {
        gemv(m_.lm_head, final_, t, logits_);
        argmax_rows(logits_, t, d_argmax);
    } else {
        // only the last row's logits (prefill): quantise that row alone at row 0
        quant_for(ht, final_ + (size_t)(t - 1) * H, H, 1);
        gemv(m_.lm_head, final_ + (size_t)(t - 1) * H, 1, logits_);
        argmax_rows(logits_, 1, d_argmax);
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
        forward_rows(t, d_ids, false);
        set_dev_int(d_keep, t, stream);  // every row of a prefill chunk is kept
        pos_ += t;
    }
    set_dev_int(d_pos, pos_, stream);
    if (sampling()) sample_row(logits_, 0, d_argmax, nullptr);  // the prompt's last row (run.rs:313-318)
    int32_t a = 0;
    ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
    sync();
    return (uint32_t)a;
}

// The kernels `enqueue` puts on the stream, captured into *exec on first use and replayed after (their launch
// count is added on every replay).
void State::graph_run(cudaGraphExec_t* exec, uint64_t* n_launches, const std::function<void()>& enqueue) {
    if (!*exec) {
        const uint64_t before = launches_;
        cudaGraph_t g = nullptr;
        ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "capture");
        try {
            enqueue();
        } catch (...) {
            cudaStreamEndCapture(stream, &g);
            if (g) cudaGraphDestroy(g);
            throw;
        }
        ck(cudaStreamEndCapture(stream, &g), "capture");
        cudaError_t e = cudaGraphInstantiate(exec, g, 0);
        cudaGraphDestroy(g);
        if (e != cudaSuccess) *exec = nullptr;
        ck(e, "graph");
        ck(cudaGraphUpload(*exec, stream), "graph upload");
        *n_launches = launches_ - before;
        launches_ = before;
    }
    ck(cudaGraphLaunch(*exec, stream), "graph launch");
    launches_ += *n_launches;
}

uint32_t State::step(uint32_t id, float* logits) {
    if (pos_ + 1 > max_pos_) throw std::invalid_argument("step: the sequence would exceed max_pos");
    upload_ids(&id, 1);
    set_dev_int(d_pos, pos_, stream);
    // one GPU: the step's kernels as one graph (debugging captures allocate per layer and run eagerly)
    if (capture_ || tp()) forward_rows(1, d_ids, true);
    else graph_run(&step_exec_, &step_launches_, [&] { forward_rows(1, d_ids, true); });
    set_dev_int(d_keep, 1, stream);
    pos_ += 1;
    set_dev_int(d_pos, pos_, stream);
    if (sampling()) sample_row(logits_, 0, d_argmax, nullptr);  // run.rs:348
    int32_t a = 0;
    ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
    if (logits && tp()) throw std::invalid_argument("step: logits are split over the tensor-parallel ranks");
    if (logits) ck(cudaMemcpyAsync(logits, logits_, (size_t)m_.cfg.vocab_size * 4, cudaMemcpyDeviceToHost, stream), "logits");
    sync();
    return (uint32_t)a;
}

void State::batch_step(const std::vector<State*>& ms, const uint32_t* ids, uint32_t* out) {
    const int B = (int)ms.size();
    if (B < 1 || !ids || !out) throw std::invalid_argument("batch_step: no sequences");
    State& L = *ms[0];
    if (B > L.T_) throw std::invalid_argument("batch_step: more sequences than the first state's max_rows");
    for (int i = 0; i < B; i++) {
        const State* s = ms[i];
        if (!s) throw std::invalid_argument("batch_step: a null state");
        for (int j = 0; j < i; j++)
            if (ms[j] == s) throw std::invalid_argument("batch_step: a state appears twice");
        if (&s->m_ != &L.m_) throw std::invalid_argument("batch_step: the states belong to different models");
        if (s->tp()) throw std::invalid_argument("batch_step: tensor-parallel states");
        if (s->sampling()) throw std::invalid_argument("batch_step: a state with a sampler (batching is greedy)");
        if (s->pos_ + 1 > s->max_pos_) throw std::invalid_argument("batch_step: a sequence would exceed its max_pos");
    }
    // the members' own queued work first: the batch runs on the first member's stream
    for (int i = 1; i < B; i++) ms[i]->sync();
    L.upload_ids(ids, B);
    std::vector<uint64_t> key((size_t)B);
    for (int i = 0; i < B; i++) key[(size_t)i] = ms[(size_t)i]->serial_;
    if (key != L.batch_key_ && L.batch_exec_) {  // other members: the captured kernels hold the old ones' buffers
        cudaGraphExecDestroy(L.batch_exec_);
        L.batch_exec_ = nullptr;
    }
    L.batch_key_ = key;
    L.batch_ = &ms;
    try {
        if (L.capture_) L.forward_rows(B, L.d_ids, true);
        else L.graph_run(&L.batch_exec_, &L.batch_launches_, [&] { L.forward_rows(B, L.d_ids, true); });
    } catch (...) {
        L.batch_ = nullptr;
        throw;
    }
    L.batch_ = nullptr;
    for (State* s : ms) {  // as step(): the row is kept, the position advances
        set_dev_int(s->d_keep, 1, L.stream);
        s->pos_ += 1;
        set_dev_int(s->d_pos, s->pos_, L.stream);
    }
    std::vector<int32_t> a(B);
    ck(cudaMemcpyAsync(a.data(), L.d_argmax, (size_t)B * 4, cudaMemcpyDeviceToHost, L.stream), "argmax");
    L.sync();
    for (int i = 0; i < B; i++) out[i] = (uint32_t)a[i];
}

void State::logits_row(int row, float* out) const {
    if (tp()) throw std::invalid_argument("logits: split over the tensor-parallel ranks");
    ck(cudaMemcpy(out, logits_ + (size_t)row * m_.cfg.vocab_size, (size_t)m_.cfg.vocab_size * 4, cudaMemcpyDeviceToHost), "logits");
}

void State::debug_hidden(int layer, int row, float* out) {
    if (!capture_ || capture_h_.empty() || layer < 0 || layer > (int)m_.layers.size()) throw std::invalid_argument("debug_hidden: no capture");
    ck(cudaStreamSynchronize(stream), "sync");
    ck(cudaMemcpy(out, capture_h_[layer] + (size_t)row * m_.cfg.hidden_size, m_.cfg.hidden_size * 4, cudaMemcpyDeviceToHost), "capture");
}

size_t State::debug_state(int layer, int what, float* out, size_t cap) {
    const ModelConfig& c = m_.cfg;
    const TpPlan& P = m_.tp;
    if (layer < 0 || layer >= (int)m_.layers.size()) throw std::invalid_argument("debug_state: no such layer");
    const LayerW& L = m_.layers[layer];
    size_t n = 0;
    if (!L.attn && (what == 0 || what == 1)) {
        n = what == 0 ? (size_t)P.nv * c.dn_head_dim_k * c.dn_head_dim_v : (size_t)L.qkv.rows * (c.dn_conv_kernel - 1);
    } else if (L.attn && (what == 2 || what == 3)) {
        n = (size_t)pos_ * P.nkv * c.head_dim_k;
    }
    if (!out || n == 0) return n;
    if (cap < n) throw std::invalid_argument("debug_state: output buffer too small");
    ck(cudaStreamSynchronize(stream), "sync");
    if (what >= 2) {
        const KvState& kv = kv_[layer];
        ck(cudaMemcpy(out, what == 2 ? kv.k : kv.v, n * 4, cudaMemcpyDeviceToHost), "kv rows");
        return n;
    }
    const DnState& d = dn_[layer];
    float* tmp = nullptr;
    ck(cudaMalloc(&tmp, n * 4), "debug buffer");
    cudaError_t e;
    if (what == 0) {
        debug_commit_state_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(
            d.S, d.pend_decay, d.pend_k, d.pend_delta, d_keep, P.nv, (int)c.dn_head_dim_k, (int)c.dn_head_dim_v, tmp);
    } else {
        debug_commit_conv_kernel<<<(L.qkv.rows + 255) / 256, 256, 0, stream>>>(d.conv, d.pend_x, d_keep, L.qkv.rows,
                                                                               (int)c.dn_conv_kernel, tmp);
    }
    e = cudaGetLastError();
    if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
    if (e == cudaSuccess) e = cudaMemcpy(out, tmp, n * 4, cudaMemcpyDeviceToHost);
    cudaFree(tmp);
    ck(e, "debug state");
    return n;
}

// The MTP block over t rows (layers/mtp.rs:95-130): row i is [rmsnorm(embed(ids[i]), enorm) |
// rmsnorm(hidden[i], hnorm)] -> eh_proj -> one attention decoder layer with its own KV cache at MTP positions
// *pos_dev + i -> shared_head_norm, into mtp_hout_.
void State::mtp_rows(int t, const int32_t* ids_dev, const float* hidden, const int* pos_dev) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const MtpW& M = m_.mtp;
    begin_session();
    count_launch(); ck(launch_dequant_rows(m_.embed.type, m_.embed.p, m_.embed.bytes / m_.embed.rows, H, ids_dev, t, embed_, stream), "embed");
    count_launch(); ck(launch_rmsnorm_rows(embed_, H, M.enorm, c.rms_norm_eps, H, t, cat_, 2 * H, stream), "enorm");
    count_launch(); ck(launch_rmsnorm_rows(hidden, H, M.hnorm, c.rms_norm_eps, H, t, cat_ + H, 2 * H, stream), "hnorm");
    quant_for(M.eh_proj.type, cat_, 2 * H, t);
    if (tp()) {
        const TpPlan& P = m_.tp;
        gemv(M.eh_proj, cat_, t, mix_out_);
        const int seg[1][3] = {{0, P.h_lo * 4, P.h_rows * 4}};
        exchange(mix_out_, (size_t)P.h_rows * 4, xo_eh_, (size_t)H * 4, seg, 1, t);
        ck(cudaMemcpyAsync(h_, xg(xo_eh_), (size_t)t * H * 4, cudaMemcpyDeviceToDevice, stream), "eh rows");
    } else {
        gemv(M.eh_proj, cat_, t, h_);  // u rows become the block's residual input
    }
    layer_forward(M.block, 0, t, &mtp_kv_, pos_dev, false);
    resid_norm(mlp_in(), M.head_norm, t, mtp_hout_, false, false);
}

// The draft of the MTP row held in mtp_h_: the shared lm_head, greedy (spec.rs:205-215, mtp.rs:132-137).
void State::enqueue_draft(int i) {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    float* lg = logits_ + (size_t)(T_ - 1) * c.vocab_size;
    begin_session();
    quant_for(m_.lm_head.type, mtp_h_, H, 1);
    gemv(m_.lm_head, mtp_h_, 1, lg);
    if (sampling()) sample_row(lg, k_ + 1, d_vids + 1 + i, q_dense_ + (size_t)i * c.vocab_size);  // spec.rs:190-203
    else argmax_rows(lg, 1, d_vids + 1 + i);
}

void State::sample_row(const float* logits, int slot, int32_t* out_dev, float* q) {
    const int V = (int)m_.cfg.vocab_size;
    int32_t* ids = kept_ids_ + (size_t)slot * V;
    float* probs = kept_probs_ + (size_t)slot * V;
    count_launch(4);
    ck(launch_sample_process(logits, V, samp_, samp_scratch_, ids, probs, kept_n_ + slot, stream), "sampler");
    ck(launch_sample_draw(d_rng_, ids, probs, kept_n_ + slot, out_dev, stream), "sampler draw");
    if (q) {
        count_launch();
        ck(launch_sample_dense(ids, probs, kept_n_ + slot, V, q, stream), "sampler q");
    }
}

void State::set_sampler(const SamplerCfg& cfg) {
    if (cfg.temperature > 0.0f && tp()) throw std::invalid_argument("sampling: a tensor-parallel state's logits are split over its ranks");
    if (cfg.top_k < 0) throw std::invalid_argument("sampling: top_k < 0");
    ck(cudaStreamSynchronize(stream), "sync");
    const int V = (int)m_.cfg.vocab_size;
    if (cfg.temperature > 0.0f && !d_rng_) {
        const size_t slots = (size_t)k_ + 2;
        d_rng_ = (uint64_t*)dalloc(32);
        samp_scratch_ = dalloc(sampler_sort_scratch_bytes(V));
        kept_ids_ = (int32_t*)dalloc(slots * V * 4);
        kept_probs_ = (float*)dalloc(slots * V * 4);
        kept_n_ = (int*)dalloc(slots * 4);
        q_dense_ = (float*)dalloc((size_t)std::max(k_, 1) * V * 4);
        samp_work_ = (float*)dalloc((size_t)V * 4);
    }
    if (d_rng_) {
        uint64_t st[4];
        sampler_seed_state(cfg.seed, st);
        ck(cudaMemcpy(d_rng_, st, sizeof st, cudaMemcpyHostToDevice), "sampler seed");
    }
    samp_ = cfg;
    if (round_exec_) {  // the captured round holds the previous mode's kernels
        cudaGraphExecDestroy(round_exec_);
        round_exec_ = nullptr;
    }
}

// Drafts from..k-1 by chaining single MTP rows (spec.rs:205-222): draft i comes from the MTP row of token
// draft i-1 (d_vids[i]) and the previous MTP row's post-norm hidden (mtp_h_), at MTP position d_mpos[i].
void State::enqueue_chain(int from) {
    const int H = (int)m_.cfg.hidden_size;
    for (int i = from; i < k_; i++) {
        mtp_rows(1, d_vids + i, mtp_h_, d_mpos + i);
        ck(cudaMemcpyAsync(mtp_h_, mtp_hout_, (size_t)H * 4, cudaMemcpyDeviceToDevice, stream), "hprev");
        enqueue_draft(i);
    }
}

uint32_t State::spec_prefill(const uint32_t* ids, int n) {
    if (k_ <= 0) throw std::invalid_argument("spec_prefill: state without spec buffers");
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const int p = pos_;
    if (n <= 0) throw std::invalid_argument("spec_prefill: empty prompt");
    if (p + n > max_pos_) throw std::invalid_argument("spec_prefill: the sequence would exceed max_pos");
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
            forward_rows(t, d_ids, false);
            set_dev_int(d_keep, t, stream);
            pos_ += t;
            ck(cudaMemcpyAsync(normed_all + (size_t)off * H, final_, (size_t)t * H * 4, cudaMemcpyDeviceToDevice, stream), "rows");
        }
        if (sampling()) sample_row(logits_, 0, d_argmax, nullptr);  // x_T (spec.rs:241)
        int32_t a = 0;
        ck(cudaMemcpyAsync(&a, d_argmax, 4, cudaMemcpyDeviceToHost, stream), "argmax");
        sync();
        x_t = (uint32_t)a;
        // MTP rows (x_{j+1}, h_j) at MTP positions p + j (spec.rs:241-262), chunks of T_ rows
        std::vector<int32_t> xs(n), mp(T_);
        for (int j = 0; j < n; j++) xs[j] = (int32_t)((j + 1 < n) ? ids[j + 1] : x_t);
        for (int off = 0; off < n; off += T_) {
            const int t = std::min(T_, n - off);
            mp[0] = p + off;
            ck(cudaMemcpy(d_mids, xs.data() + off, (size_t)t * 4, cudaMemcpyHostToDevice), "mtp ids");
            ck(cudaMemcpy(d_mpos, mp.data(), 4, cudaMemcpyHostToDevice), "mtp pos");
            mtp_rows(t, d_mids, normed_all + (size_t)off * H, d_mpos);
            if (off + t == n) ck(cudaMemcpyAsync(mtp_h_, mtp_hout_ + (size_t)(t - 1) * H, (size_t)H * 4, cudaMemcpyDeviceToDevice, stream), "hlast");
            sync();
        }
        // the first draft from the last prompt row, then the chain at p + n, p + n + 1, ...
        enqueue_draft(0);
        for (int i = 1; i < k_; i++) mp[i] = p + n + i - 1;
        ck(cudaMemcpyAsync(d_mpos, mp.data(), (size_t)T_ * 4, cudaMemcpyHostToDevice, stream), "mtp pos");
        enqueue_chain(1);
        set_dev_int(d_pos, pos_, stream);  // the device position the next round starts from
        sync();
    } catch (...) {
        cudaStreamSynchronize(stream);
        cudaFree(normed_all);
        throw;
    }
    cudaFree(normed_all);
    mtp_len_ = p + n + k_ - 1;
    drafts_ready_ = true;
    return x_t;
}

void State::enqueue_round() {
    const ModelConfig& c = m_.cfg;
    const int H = (int)c.hidden_size;
    const int t = k_ + 1;
    const uint64_t xseq0 = xseq_;
    ck(cudaMemcpyAsync(d_vids, h_io_, 4, cudaMemcpyHostToDevice, stream), "x_p");
    forward_rows(t, d_vids, true);  // the verify batch: x_p, d_1..d_k
    if (sampling()) {
        // the target's processed distribution of every verify row, then accept_or_resample in order (spec.rs:367-379)
        const int V = (int)c.vocab_size;
        for (int r = 0; r < t; r++) {
            count_launch(3);
            ck(launch_sample_process(logits_ + (size_t)r * V, V, samp_, samp_scratch_, kept_ids_ + (size_t)r * V,
                                     kept_probs_ + (size_t)r * V, kept_n_ + r, stream),
               "sampler");
        }
        SpecAcceptArgs sa{d_rng_, kept_ids_, kept_probs_, kept_n_, (size_t)V, q_dense_, V, d_vids, k_, d_pos, d_keep, d_mpos,
                          d_mids, d_sel, d_emit, samp_work_};
        count_launch();
        ck(launch_spec_accept_sampled(sa, stream), "accept");
    } else {
        count_launch();
        spec_accept_kernel<<<1, 32, 0, stream>>>(d_argmax, d_vids, k_, d_pos, d_keep, d_mpos, d_mids, d_sel, d_emit);
        ck(cudaGetLastError(), "accept");
    }
    // the MTP re-feed: all t rows (rows past keep are scratch; their cache slots are rewritten before any read)
    mtp_rows(t, d_mids, final_, d_mpos);
    count_launch();
    select_row_kernel<<<8, 256, 0, stream>>>(mtp_hout_, d_sel, H, mtp_h_);
    ck(cudaGetLastError(), "select row");
    enqueue_draft(0);
    enqueue_chain(1);
    if (tp() && ((xseq_ - xseq0) & 1)) {
        // an even number of exchanges per round keeps consecutive exchanges on alternate line buffers from one
        // replay of the round graph to the next: pad with a 16-byte exchange
        const int seg[1][3] = {{0, 16 * m_.tp.rank, 16}};
        exchange(amx_pairs_, 16, xo_pad_, 16 * (size_t)m_.tp.world, seg, 1, 1);
    }
    ck(cudaMemcpyAsync(h_io_ + 16, d_emit, (size_t)(k_ + 2) * 4, cudaMemcpyDeviceToHost, stream), "emitted");
}

int State::spec_round(uint32_t x_p, uint32_t* out) {
    if (k_ <= 0) throw std::invalid_argument("spec_round: state without spec buffers");
    if (!drafts_ready_) throw std::logic_error("spec_round: drafts missing (call spec_prefill first)");
    const int t = k_ + 1;
    const int p = pos_;
    if (p + t > max_pos_) throw std::invalid_argument("spec_round: the sequence would exceed max_pos");
    if (mtp_len_ != p + k_ - 1) throw std::logic_error("spec_round: MTP rows out of step with the position");
    if (x_p >= m_.cfg.vocab_size) throw std::invalid_argument("spec_round: token id outside the vocabulary");
    h_io_[0] = (int32_t)x_p;
    if (capture_) {
        enqueue_round();  // debugging captures allocate and copy per layer: run the round eagerly
    } else {
        if (!round_exec_) {
            const uint64_t before = launches_;
            cudaGraph_t g = nullptr;
            ck(cudaStreamBeginCapture(stream, cudaStreamCaptureModeThreadLocal), "round capture");
            try {
                enqueue_round();
            } catch (...) {
                cudaStreamEndCapture(stream, &g);
                if (g) cudaGraphDestroy(g);
                throw;
            }
            ck(cudaStreamEndCapture(stream, &g), "round capture");
            cudaError_t e = cudaGraphInstantiate(&round_exec_, g, 0);
            cudaGraphDestroy(g);
            ck(e, "round graph");
            ck(cudaGraphUpload(round_exec_, stream), "round graph upload");
            round_launches_ = launches_ - before;
            launches_ = before;
        }
        ck(cudaGraphLaunch(round_exec_, stream), "round");
        launches_ += round_launches_;
    }
    sync();
    const int keep = h_io_[16];
    if (keep < 1 || keep > t) throw std::runtime_error("spec_round: device acceptance returned an invalid count");
    for (int i = 0; i < keep; i++) out[i] = (uint32_t)h_io_[17 + i];
    pos_ = p + keep;
    mtp_len_ = p + keep + k_ - 1;
    counters.rounds++;
    counters.drafted += k_;
    counters.accepted += keep - 1;
    counters.emitted += keep;
    counters.hist[keep - 1]++;
    return keep;
}

void State::set_drafts(const uint32_t* d, int k) {
    if (k != k_) throw std::invalid_argument("set_drafts: wrong number of drafts");
    if (!drafts_ready_) throw std::logic_error("set_drafts: no round pending (call spec_prefill first)");
    std::vector<int32_t> v(k);
    for (int i = 0; i < k; i++) {
        if (d[i] >= m_.cfg.vocab_size) throw std::invalid_argument("set_drafts: draft outside the vocabulary");
        v[i] = (int32_t)d[i];
    }
    ck(cudaStreamSynchronize(stream), "sync");
    ck(cudaMemcpy(d_vids + 1, v.data(), (size_t)k * 4, cudaMemcpyHostToDevice), "drafts");
}

std::vector<uint32_t> State::drafts() const {
    std::vector<uint32_t> out;
    if (!drafts_ready_ || k_ <= 0) return out;
    std::vector<int32_t> v(k_);
    ck(cudaStreamSynchronize(stream), "sync");
    ck(cudaMemcpy(v.data(), d_vids + 1, (size_t)k_ * 4, cudaMemcpyDeviceToHost), "drafts");
    for (int x : v) out.push_back((uint32_t)x);
    return out;
}

}  // namespace qdec
