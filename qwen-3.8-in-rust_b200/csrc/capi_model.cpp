// The model-level C ABI (include/qdec.h): the reference's model seam (crates/core/src/model.rs, spec.rs) over
// the engine, with every C++ exception turned into a status code and a message.
#include <cstring>
#include <memory>
#include <mutex>
#include <vector>
#include <new>
#include <stdexcept>

#include "../../include/qdec.h"
#include "capi_util.h"
#include "engine.h"
#include "gguf.h"
#include "synth.h"

struct qdec_model {
    std::unique_ptr<qdec::Model> m;
    // states made from this model and not yet freed; qdec_close with states alive defers the delete to the last
    // qdec_state_free (a state reads its model until it is gone)
    std::mutex mu;
    int live = 0;
    bool closed = false;
};
struct qdec_state {
    std::unique_ptr<qdec::State> s;
    qdec_model* owner;
};

namespace {
template <typename F>
int guard(const char* what, F&& f) {
    try {
        qdec::clear_error();
        return f();
    } catch (const qdec::GgufError& e) {
        return qdec::fail(QDEC_EFORMAT, "%s: %s", what, e.what());
    } catch (const qdec::ConfigError& e) {
        return qdec::fail(QDEC_EFORMAT, "%s: %s", what, e.what());
    } catch (const std::invalid_argument& e) {
        return qdec::fail(QDEC_EINVAL, "%s: %s", what, e.what());
    } catch (const std::logic_error& e) {
        return qdec::fail(QDEC_ESTATE, "%s: %s", what, e.what());
    } catch (const std::bad_alloc&) {
        return qdec::fail(QDEC_ENOMEM, "%s: out of host memory", what);
    } catch (const std::runtime_error& e) {
        const char* msg = e.what();
        if (strstr(msg, "gave up")) return qdec::fail(QDEC_ETIMEOUT, "%s: %s", what, msg);
        if (strstr(msg, "out of memory") || strstr(msg, "allocation")) return qdec::fail(QDEC_ENOMEM, "%s: %s", what, msg);
        if (strstr(msg, "cannot") || strstr(msg, "io error") || strstr(msg, "write failed")) return qdec::fail(QDEC_EIO, "%s: %s", what, msg);
        return qdec::fail(QDEC_ECUDA, "%s: %s", what, msg);
    } catch (const std::exception& e) {
        return qdec::fail(QDEC_ECUDA, "%s: %s", what, e.what());
    }
}
}  // namespace

extern "C" {

int qdec_open(const char* path, const qdec_opts* opts, qdec_model** out) {
    if (!path || !out) return qdec::fail(QDEC_EINVAL, "qdec_open: null argument");
    *out = nullptr;
    return guard("qdec_open", [&] {
        qdec::LoadOptions o;
        if (opts) {
            o.device = opts->device;
            if (opts->max_pos > 0) o.max_pos = opts->max_pos;
        }
        auto m = qdec::Model::load(path, o);
        *out = new qdec_model{std::move(m)};
        return QDEC_OK;
    });
}

int qdec_open_tp(const char* path, const qdec_opts* opts, int tp_rank, int tp_world, qdec_model** out) {
    if (!path || !out) return qdec::fail(QDEC_EINVAL, "qdec_open_tp: null argument");
    *out = nullptr;
    return guard("qdec_open_tp", [&] {
        qdec::LoadOptions o;
        if (opts) {
            o.device = opts->device;
            if (opts->max_pos > 0) o.max_pos = opts->max_pos;
        }
        o.tp_rank = tp_rank;
        o.tp_world = tp_world;
        auto m = qdec::Model::load(path, o);
        *out = new qdec_model{std::move(m)};
        return QDEC_OK;
    });
}

int qdec_tp_plan(const char* path, int tp_rank, int tp_world, int32_t out[16]) {
    if (!path || !out) return qdec::fail(QDEC_EINVAL, "qdec_tp_plan: null argument");
    return guard("qdec_tp_plan", [&] {
        qdec::Gguf g(path);
        const qdec::TpPlan p = qdec::make_tp_plan(qdec::ModelConfig::from_gguf(g), tp_rank, tp_world);
        const int32_t v[16] = {p.rank, p.world, p.kh_lo, p.nk, p.nv, p.qh_lo, p.nq, p.kv_lo, p.nkv, p.ff_lo, p.ff_rows,
                               p.h_lo, p.h_rows, p.v_lo, p.v_rows, 0};
        std::memcpy(out, v, sizeof v);
        return QDEC_OK;
    });
}

int qdec_tp_plan_dims(const uint32_t dims[8], int tp_rank, int tp_world, int32_t out[16]) {
    if (!dims || !out) return qdec::fail(QDEC_EINVAL, "qdec_tp_plan_dims: null argument");
    return guard("qdec_tp_plan_dims", [&] {
        qdec::ModelConfig c;
        c.hidden_size = dims[0];
        c.intermediate_size = dims[1];
        c.vocab_size = dims[2];
        c.n_head = dims[3];
        c.n_head_kv = dims[4];
        c.dn_n_k_heads = dims[5];
        c.dn_n_v_heads = dims[6];
        if (dims[7]) c.deltanet_layers.push_back(0);
        const qdec::TpPlan p = qdec::make_tp_plan(c, tp_rank, tp_world);
        const int32_t v[16] = {p.rank, p.world, p.kh_lo, p.nk, p.nv, p.qh_lo, p.nq, p.kv_lo, p.nkv, p.ff_lo, p.ff_rows,
                               p.h_lo, p.h_rows, p.v_lo, p.v_rows, 0};
        std::memcpy(out, v, sizeof v);
        return QDEC_OK;
    });
}

int qdec_set_sampler(qdec_state* s, float temperature, int top_k, float top_p, float min_p, uint64_t seed) {
    if (!s) return qdec::fail(QDEC_EINVAL, "qdec_set_sampler: null state");
    return guard("qdec_set_sampler", [&] {
        qdec::SamplerCfg c;
        c.temperature = temperature;
        c.top_k = top_k;
        c.top_p = top_p;
        c.min_p = min_p;
        c.seed = seed;
        s->s->set_sampler(c);
        return QDEC_OK;
    });
}

int qdec_tp_export(const qdec_state* s, void* handle_out) {
    if (!s || !handle_out) return qdec::fail(QDEC_EINVAL, "qdec_tp_export: null argument");
    return guard("qdec_tp_export", [&] {
        s->s->tp_export(handle_out);
        return QDEC_OK;
    });
}

int qdec_tp_stats(const qdec_state* s, uint64_t out4[4]) {
    if (!s || !out4) return qdec::fail(QDEC_EINVAL, "qdec_tp_stats: null argument");
    return guard("qdec_tp_stats", [&] {
        s->s->tp_stats(out4);
        return QDEC_OK;
    });
}

int qdec_tp_connect(qdec_state* s, const void* handles) {
    if (!s || !handles) return qdec::fail(QDEC_EINVAL, "qdec_tp_connect: null argument");
    return guard("qdec_tp_connect", [&] {
        s->s->tp_connect(handles);
        return QDEC_OK;
    });
}

int qdec_close(qdec_model* m) {
    if (!m) return QDEC_OK;
    {
        std::lock_guard<std::mutex> g(m->mu);
        if (m->live > 0) {
            m->closed = true;
            return QDEC_OK;
        }
    }
    delete m;
    return QDEC_OK;
}

int qdec_model_loaded_direct(const qdec_model* m) { return m && m->m->loaded_direct ? 1 : 0; }

int qdec_model_get_info(const qdec_model* m, qdec_model_info* info) {
    if (!m || !info) return qdec::fail(QDEC_EINVAL, "qdec_model_get_info: null argument");
    const qdec::ModelConfig& c = m->m->cfg;
    info->n_layer = c.n_layer;
    info->hidden = c.hidden_size;
    info->ffn = c.intermediate_size;
    info->vocab = c.vocab_size;
    info->n_head = c.n_head;
    info->n_head_kv = c.n_head_kv;
    info->head_dim = c.head_dim_k;
    info->dn_n_k_heads = c.dn_n_k_heads;
    info->dn_n_v_heads = c.dn_n_v_heads;
    info->dn_head_dim_k = c.dn_head_dim_k;
    info->dn_head_dim_v = c.dn_head_dim_v;
    info->n_full_attention = (uint32_t)c.full_attention_layers.size();
    info->has_mtp = m->m->has_mtp;
    info->weight_bytes = m->m->weight_bytes;
    info->decode_bytes = m->m->decode_bytes;
    info->lm_head_bytes = m->m->lm_head.bytes;
    info->mtp_bytes = m->m->mtp_bytes;
    info->load_secs = m->m->load_secs;
    return QDEC_OK;
}

int qdec_is_stop(const qdec_model* m, uint32_t id) { return m && m->m->is_stop(id) ? 1 : 0; }

int qdec_state_new(qdec_model* m, int spec_k, int max_pos, int max_rows, qdec_state** out) {
    if (!m || !out || spec_k < 0 || max_pos <= 0 || max_rows <= 0)
        return qdec::fail(QDEC_EINVAL, "qdec_state_new: bad argument");
    *out = nullptr;
    return guard("qdec_state_new", [&] {
        {
            std::lock_guard<std::mutex> g(m->mu);
            if (m->closed) throw std::logic_error("the model is closed");
        }
        auto s = std::make_unique<qdec::State>(*m->m, spec_k, max_pos, max_rows);
        *out = new qdec_state{std::move(s), m};
        std::lock_guard<std::mutex> g(m->mu);
        m->live++;
        return QDEC_OK;
    });
}

int qdec_state_free(qdec_state* s) {
    if (!s) return QDEC_OK;
    qdec_model* m = s->owner;
    delete s;
    bool last = false;
    {
        std::lock_guard<std::mutex> g(m->mu);
        last = --m->live == 0 && m->closed;
    }
    if (last) delete m;
    return QDEC_OK;
}

int qdec_state_pos(const qdec_state* s) { return s ? s->s->pos() : -1; }

int qdec_prefill(qdec_state* s, const uint32_t* ids, int n, uint32_t* first_out) {
    if (!s || !ids || n <= 0 || !first_out) return qdec::fail(QDEC_EINVAL, "qdec_prefill: bad argument");
    return guard("qdec_prefill", [&] {
        *first_out = s->s->prefill(ids, n);
        return QDEC_OK;
    });
}

int qdec_step(qdec_state* s, uint32_t id, uint32_t* next_out, float* logits_out) {
    if (!s || !next_out) return qdec::fail(QDEC_EINVAL, "qdec_step: bad argument");
    return guard("qdec_step", [&] {
        *next_out = s->s->step(id, logits_out);
        return QDEC_OK;
    });
}

int qdec_batch_step(qdec_state* const* states, int n, const uint32_t* ids, uint32_t* next_out) {
    if (!states || n <= 0 || !ids || !next_out) return qdec::fail(QDEC_EINVAL, "qdec_batch_step: bad argument");
    std::vector<qdec::State*> ms((size_t)n);
    for (int i = 0; i < n; i++) {
        if (!states[i]) return qdec::fail(QDEC_EINVAL, "qdec_batch_step: state %d is null", i);
        ms[(size_t)i] = states[i]->s.get();
    }
    return guard("qdec_batch_step", [&] {
        qdec::State::batch_step(ms, ids, next_out);
        return QDEC_OK;
    });
}

int qdec_spec_prefill(qdec_state* s, const uint32_t* ids, int n, uint32_t* x_out) {
    if (!s || !ids || n <= 0 || !x_out) return qdec::fail(QDEC_EINVAL, "qdec_spec_prefill: bad argument");
    return guard("qdec_spec_prefill", [&] {
        *x_out = s->s->spec_prefill(ids, n);
        return QDEC_OK;
    });
}

int qdec_spec_round(qdec_state* s, uint32_t x_p, uint32_t* emitted_out, int* n_emitted) {
    if (!s || !emitted_out || !n_emitted) return qdec::fail(QDEC_EINVAL, "qdec_spec_round: bad argument");
    return guard("qdec_spec_round", [&] {
        *n_emitted = s->s->spec_round(x_p, emitted_out);
        return QDEC_OK;
    });
}

int qdec_set_drafts(qdec_state* s, const uint32_t* drafts, int k) {
    if (!s || !drafts) return qdec::fail(QDEC_EINVAL, "qdec_set_drafts: bad argument");
    return guard("qdec_set_drafts", [&] {
        s->s->set_drafts(drafts, k);
        return QDEC_OK;
    });
}

int qdec_get_drafts(const qdec_state* s, uint32_t* drafts_out, int k) {
    if (!s || !drafts_out) return qdec::fail(QDEC_EINVAL, "qdec_get_drafts: bad argument");
    const auto& d = s->s->drafts();
    if ((int)d.size() != k) return qdec::fail(QDEC_ESTATE, "qdec_get_drafts: %zu drafts held, %d asked", d.size(), k);
    for (int i = 0; i < k; i++) drafts_out[i] = d[i];
    return QDEC_OK;
}

int qdec_spec_counters(const qdec_state* s, uint64_t out4[4]) {
    if (!s || !out4) return qdec::fail(QDEC_EINVAL, "qdec_spec_counters: bad argument");
    const auto& c = s->s->counters;
    out4[0] = c.rounds;
    out4[1] = c.drafted;
    out4[2] = c.accepted;
    out4[3] = c.emitted;
    return QDEC_OK;
}

void* qdec_state_stream(const qdec_state* s) { return s ? (void*)s->s->stream : nullptr; }

uint64_t qdec_state_launches(const qdec_state* s) { return s ? s->s->launches() : 0; }

int qdec_set_capture(qdec_state* s, int on) {
    if (!s) return qdec::fail(QDEC_EINVAL, "qdec_set_capture: null state");
    s->s->set_capture(on != 0);
    return QDEC_OK;
}

int qdec_debug_state(qdec_state* s, int layer, int what, float* out, size_t* n_floats) {
    if (!s || !n_floats) return qdec::fail(QDEC_EINVAL, "qdec_debug_state: bad argument");
    return guard("qdec_debug_state", [&] {
        *n_floats = s->s->debug_state(layer, what, out, *n_floats);
        return QDEC_OK;
    });
}

int qdec_debug_hidden(qdec_state* s, int layer, int row, float* out) {
    if (!s || !out) return qdec::fail(QDEC_EINVAL, "qdec_debug_hidden: bad argument");
    return guard("qdec_debug_hidden", [&] {
        s->s->debug_hidden(layer, row, out);
        return QDEC_OK;
    });
}

int qdec_debug_logits(qdec_state* s, int row, float* out) {
    if (!s || !out) return qdec::fail(QDEC_EINVAL, "qdec_debug_logits: bad argument");
    return guard("qdec_debug_logits", [&] {
        s->s->logits_row(row, out);
        return QDEC_OK;
    });
}

int qdec_synth_gguf(const char* path, const char* preset, uint64_t seed, int threads) {
    if (!path || !preset) return qdec::fail(QDEC_EINVAL, "qdec_synth_gguf: null argument");
    return guard("qdec_synth_gguf", [&] {
        qdec::synth_gguf(path, preset, seed, threads);
        return QDEC_OK;
    });
}

}  // extern "C"
