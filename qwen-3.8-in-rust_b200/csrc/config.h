// The model contract, built only from GGUF metadata and the tensor index (crates/core/src/config.rs:146-260),
// plus the architecture constants the metadata does not carry (crates/core/src/arch.rs:61-90).
#pragma once
#include <cstdint>
#include <stdexcept>
#include <string>
#include <vector>

#include "gguf.h"

namespace qdec {

struct ConfigError : std::runtime_error {
    using std::runtime_error::runtime_error;
};

struct ModelConfig {
    std::string architecture, name;
    uint32_t file_type = 0, quantization_version = 0;
    uint32_t block_count = 0, nextn_predict_layers = 0, n_layer = 0, context_length = 0;
    uint32_t hidden_size = 0, intermediate_size = 0, vocab_size = 0;
    uint32_t n_head = 0, n_head_kv = 0, head_dim_k = 0, head_dim_v = 0;
    float rms_norm_eps = 0.f;
    uint32_t full_attention_interval = 0;
    float rope_freq_base = 0.f;
    uint32_t rope_dim = 0;
    std::vector<int32_t> rope_sections;
    uint32_t dn_conv_kernel = 0, dn_head_dim_k = 0, dn_n_k_heads = 0, dn_n_v_heads = 0, dn_inner_size = 0, dn_head_dim_v = 0;
    uint32_t bos_id = 0, pad_id = 0;
    std::vector<uint32_t> eos_ids;
    bool add_bos = false;
    std::string tokenizer_model, tokenizer_pre;
    // derived
    std::vector<uint32_t> full_attention_layers, deltanet_layers, mtp_layers;
    uint32_t gqa_group = 0, q_dim = 0, kv_dim = 0;
    bool attn_output_gate = false, tie_word_embeddings = false, mtp_dedicated_embeddings = false;
    uint32_t dn_k_dim = 0, dn_v_dim = 0, dn_qkv_dim = 0;
    uint64_t dn_state_elems_per_layer = 0, dn_conv_state_elems_per_layer = 0;
    // stop ids: GGUF EOS ids plus the architecture's extra ones (arch.rs:79-90)
    std::vector<uint32_t> stop_ids;

    static ModelConfig from_gguf(const Gguf &g);  // throws ConfigError / GgufError
    bool is_attention(uint32_t layer) const;
    std::string describe() const;
};

}  // namespace qdec
