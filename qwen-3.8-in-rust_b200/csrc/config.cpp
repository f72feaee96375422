// ModelConfig::from_gguf: every field from a GGUF key or a derivation; a missing or mistyped key is a hard
// error naming it, nothing falls back to a default (crates/core/src/config.rs:146-260, arch.rs:61-90).
#include "config.h"

#include <algorithm>
#include <cstdarg>
#include <sstream>

namespace qdec {

namespace {

[[noreturn]] void inconsistent(const std::string &what, const std::string &detail) {
    throw ConfigError("metadata is inconsistent: " + what + ": " + detail);
}
[[noreturn]] void missing_tensor(const std::string &name) {
    throw ConfigError("tensor " + name + " is required to derive the config but is not in the file");
}
std::string shp(const std::vector<uint64_t> &v) {
    std::ostringstream o;
    o << "[";
    for (size_t i = 0; i < v.size(); i++) o << (i ? ", " : "") << v[i];
    o << "]";
    return o.str();
}

// The one architecture this engine knows (arch.rs:61-77): any other general.architecture is refused.
const uint32_t QWEN35_EXTRA_STOP_IDS[] = {248044};

}  // namespace

bool ModelConfig::is_attention(uint32_t layer) const {
    return std::find(full_attention_layers.begin(), full_attention_layers.end(), layer) != full_attention_layers.end();
}

ModelConfig ModelConfig::from_gguf(const Gguf &g) {
    ModelConfig c;
    c.architecture = g.get_str("general.architecture");
    if (c.architecture != "qwen35")
        throw ConfigError("unknown architecture \"" + c.architecture + "\": this engine knows only [\"qwen35\"]");
    auto k = [&](const char *s) { return c.architecture + "." + s; };
    c.block_count = g.get_u32(k("block_count"));
    c.nextn_predict_layers = g.get_u32(k("nextn_predict_layers"));
    if (c.nextn_predict_layers >= c.block_count)
        inconsistent("nextn_predict_layers", std::to_string(c.nextn_predict_layers) + " >= block_count " + std::to_string(c.block_count));
    c.n_layer = c.block_count - c.nextn_predict_layers;
    c.context_length = g.get_u32(k("context_length"));
    c.hidden_size = g.get_u32(k("embedding_length"));
    c.intermediate_size = g.get_u32(k("feed_forward_length"));
    c.n_head = g.get_u32(k("attention.head_count"));
    c.n_head_kv = g.get_u32(k("attention.head_count_kv"));
    c.head_dim_k = g.get_u32(k("attention.key_length"));
    c.head_dim_v = g.get_u32(k("attention.value_length"));
    c.rms_norm_eps = g.get_f32(k("attention.layer_norm_rms_epsilon"));
    c.full_attention_interval = g.get_u32(k("full_attention_interval"));
    c.rope_freq_base = g.get_f32(k("rope.freq_base"));
    c.rope_dim = g.get_u32(k("rope.dimension_count"));
    c.rope_sections = g.get_array_i32(k("rope.dimension_sections"));
    c.dn_conv_kernel = g.get_u32(k("ssm.conv_kernel"));
    c.dn_head_dim_k = g.get_u32(k("ssm.state_size"));
    c.dn_n_k_heads = g.get_u32(k("ssm.group_count"));
    c.dn_n_v_heads = g.get_u32(k("ssm.time_step_rank"));
    c.dn_inner_size = g.get_u32(k("ssm.inner_size"));
    c.name = g.get_str("general.name");
    c.file_type = g.get_u32("general.file_type");
    c.quantization_version = g.get_u32("general.quantization_version");
    c.bos_id = g.get_u32("tokenizer.ggml.bos_token_id");
    const uint32_t eos = g.get_u32("tokenizer.ggml.eos_token_id");
    c.pad_id = g.get_u32("tokenizer.ggml.padding_token_id");
    c.add_bos = g.get_bool("tokenizer.ggml.add_bos_token");
    c.tokenizer_model = g.get_str("tokenizer.ggml.model");
    c.tokenizer_pre = g.get_str("tokenizer.ggml.pre");
    c.vocab_size = (uint32_t)g.get_array("tokenizer.ggml.tokens").arr.size();
    c.eos_ids.push_back(eos);
    if (g.has("tokenizer.ggml.eot_token_id")) {
        const uint32_t eot = g.get_u32("tokenizer.ggml.eot_token_id");
        if (std::find(c.eos_ids.begin(), c.eos_ids.end(), eot) == c.eos_ids.end()) c.eos_ids.push_back(eot);
    }

    if (c.n_head_kv == 0 || c.n_head % c.n_head_kv)
        inconsistent("head_count / head_count_kv", std::to_string(c.n_head) + " / " + std::to_string(c.n_head_kv));
    if (c.dn_n_v_heads == 0 || c.dn_inner_size % c.dn_n_v_heads)
        inconsistent("ssm.inner_size / ssm.time_step_rank", std::to_string(c.dn_inner_size) + " / " + std::to_string(c.dn_n_v_heads));
    c.dn_head_dim_v = c.dn_inner_size / c.dn_n_v_heads;
    if (c.dn_n_k_heads == 0 || c.dn_n_v_heads % c.dn_n_k_heads)
        inconsistent("ssm.time_step_rank / ssm.group_count", std::to_string(c.dn_n_v_heads) + " / " + std::to_string(c.dn_n_k_heads));
    if (c.rope_dim > c.head_dim_k)
        inconsistent("rope.dimension_count", std::to_string(c.rope_dim) + " > key_length " + std::to_string(c.head_dim_k));
    int sec = 0;
    for (int32_t s : c.rope_sections) sec += s;
    if ((uint32_t)sec * 2 != c.rope_dim)
        inconsistent("rope.dimension_sections", "sum " + std::to_string(sec) + " * 2 != rope.dimension_count " + std::to_string(c.rope_dim));

    if (!g.has_tensor("token_embd.weight")) missing_tensor("token_embd.weight");
    const TensorInfo &embd = g.tensor("token_embd.weight");
    if (embd.shape.size() != 2 || embd.shape[0] != c.hidden_size || embd.shape[1] != c.vocab_size)
        inconsistent("token_embd.weight shape", shp(embd.shape) + " vs [embedding_length " + std::to_string(c.hidden_size) +
                                                     ", len(tokens) " + std::to_string(c.vocab_size) + "]");
    c.tie_word_embeddings = !g.has_tensor("output.weight");
    if (!c.tie_word_embeddings && g.tensor("output.weight").shape != embd.shape)
        inconsistent("output.weight shape", shp(g.tensor("output.weight").shape) + " vs token_embd " + shp(embd.shape));
    if (!g.has_tensor("output_norm.weight")) missing_tensor("output_norm.weight");

    c.q_dim = c.n_head * c.head_dim_k;
    c.kv_dim = c.n_head_kv * c.head_dim_k;
    c.dn_k_dim = c.dn_n_k_heads * c.dn_head_dim_k;
    c.dn_v_dim = c.dn_n_v_heads * c.dn_head_dim_v;
    c.dn_qkv_dim = 2 * c.dn_k_dim + c.dn_v_dim;

    int gate = -1;
    for (uint32_t i = 0; i < c.n_layer; i++) {
        const std::string p = "blk." + std::to_string(i) + ".";
        const bool has_attn = g.has_tensor(p + "attn_q.weight");
        const bool has_ssm = g.has_tensor(p + "ssm_a");
        const bool by_rule = (i + 1) % c.full_attention_interval == 0;
        if (has_attn && !has_ssm) {
            if (!by_rule) inconsistent("layer_types", "blk." + std::to_string(i) + " has attn_q but (i+1) % " + std::to_string(c.full_attention_interval) + " != 0");
            const TensorInfo &q = g.tensor(p + "attn_q.weight");
            if (q.shape.size() != 2 || q.shape[0] != c.hidden_size) inconsistent("attn_q shape", "blk." + std::to_string(i) + ": " + shp(q.shape));
            int gt;
            if (q.shape[1] == 2ull * c.q_dim) gt = 1;
            else if (q.shape[1] == c.q_dim) gt = 0;
            else inconsistent("attn_q rows", "blk." + std::to_string(i) + ": " + std::to_string(q.shape[1]) + " is neither q_dim " + std::to_string(c.q_dim) + " nor 2*q_dim");
            if (gate == -1) gate = gt;
            else if (gate != gt) inconsistent("attn_output_gate", "differs at blk." + std::to_string(i));
            const TensorInfo &kt = g.tensor(p + "attn_k.weight");
            if (kt.shape != std::vector<uint64_t>{c.hidden_size, c.kv_dim})
                inconsistent("attn_k shape", "blk." + std::to_string(i) + ": " + shp(kt.shape));
            c.full_attention_layers.push_back(i);
        } else if (!has_attn && has_ssm) {
            if (by_rule) inconsistent("layer_types", "blk." + std::to_string(i) + " has ssm_a but (i+1) % " + std::to_string(c.full_attention_interval) + " == 0");
            const TensorInfo &qkv = g.tensor(p + "attn_qkv.weight");
            if (qkv.shape != std::vector<uint64_t>{c.hidden_size, c.dn_qkv_dim})
                inconsistent("attn_qkv shape", "blk." + std::to_string(i) + ": " + shp(qkv.shape));
            const TensorInfo &conv = g.tensor(p + "ssm_conv1d.weight");
            if (conv.shape != std::vector<uint64_t>{c.dn_conv_kernel, c.dn_qkv_dim})
                inconsistent("ssm_conv1d shape", "blk." + std::to_string(i) + ": " + shp(conv.shape));
            const TensorInfo &a = g.tensor(p + "ssm_a");
            if (a.shape != std::vector<uint64_t>{c.dn_n_v_heads}) inconsistent("ssm_a shape", "blk." + std::to_string(i) + ": " + shp(a.shape));
            c.deltanet_layers.push_back(i);
        } else if (has_attn && has_ssm) {
            inconsistent("layer_types", "blk." + std::to_string(i) + " has both attn_q and ssm_a");
        } else {
            inconsistent("layer_types", "blk." + std::to_string(i) + " has neither attn_q nor ssm_a");
        }
    }
    if (gate == -1) inconsistent("layer_types", "no full-attention layer found");
    c.attn_output_gate = gate == 1;
    for (uint32_t m = c.n_layer; m < c.block_count; m++) {
        const std::string n = "blk." + std::to_string(m) + ".nextn.eh_proj.weight";
        if (!g.has_tensor(n)) missing_tensor(n);
        c.mtp_layers.push_back(m);
        if (g.has_tensor("blk." + std::to_string(m) + ".nextn.embed_tokens.weight") ||
            g.has_tensor("blk." + std::to_string(m) + ".nextn.shared_head.head.weight"))
            c.mtp_dedicated_embeddings = true;
    }
    c.gqa_group = c.n_head / c.n_head_kv;
    c.dn_state_elems_per_layer = (uint64_t)c.dn_n_v_heads * c.dn_head_dim_k * c.dn_head_dim_v;
    c.dn_conv_state_elems_per_layer = (uint64_t)c.dn_qkv_dim * (c.dn_conv_kernel - 1);
    c.stop_ids = c.eos_ids;
    for (uint32_t id : QWEN35_EXTRA_STOP_IDS)
        if (std::find(c.stop_ids.begin(), c.stop_ids.end(), id) == c.stop_ids.end()) c.stop_ids.push_back(id);
    return c;
}

std::string ModelConfig::describe() const {
    std::ostringstream o;
    o << "architecture " << architecture << " (" << name << ")\n"
      << "blocks " << block_count << " (" << n_layer << " + " << nextn_predict_layers << " MTP)\n"
      << "hidden " << hidden_size << " ffn " << intermediate_size << " vocab " << vocab_size << "\n"
      << "attention heads " << n_head << "/" << n_head_kv << " x " << head_dim_k << ", rope " << rope_dim << " theta " << rope_freq_base << "\n"
      << "deltanet k " << dn_n_k_heads << "x" << dn_head_dim_k << " v " << dn_n_v_heads << "x" << dn_head_dim_v << " conv " << dn_conv_kernel << "\n"
      << "full-attention layers " << full_attention_layers.size() << ", deltanet layers " << deltanet_layers.size() << "\n";
    return o.str();
}

}  // namespace qdec
