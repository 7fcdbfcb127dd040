// ModelConfig: architecture constants of a hybrid Gated-DeltaNet + gated-attention
// Qwen3.5 model. Same fields, defaults (the Qwen3.5-0.8B text_config) and layer rule as
// the reference's include/model_config.h:11-76, so callers of the reference compile
// against this header unchanged.
#pragma once
#include <cstdint>
#include <string>

struct ModelConfig {
    std::string name = "qwen3.5-0.8b";
    int64_t n_params = 800'000'000;
    int hidden_size = 1024;
    int n_layers_total = 24;
    int n_layers_gdn = 18;
    int n_layers_attn = 6;
    int gdn_k_heads = 16;
    int gdn_v_heads = 16;
    int gdn_k_head_dim = 128;
    int gdn_v_head_dim = 128;
    int gdn_conv_kernel = 4;
    int gdn_n_heads = 16;    // alias of gdn_v_heads
    int gdn_head_dim = 128;  // alias of gdn_v_head_dim
    int attn_q_heads = 8;
    int attn_kv_heads = 2;
    int attn_head_dim = 256;
    bool attn_output_gate = true;
    bool attn_qk_norm = true;
    int ffn_intermediate = 3584;
    int vocab_size = 248320;
    int native_max_context = 262144;
    float rms_norm_eps = 1e-6f;
    bool tie_word_embeddings = true;
    double rope_theta = 10'000'000.0;
    float partial_rotary_factor = 0.25f;
    int attn_interval = 4;

    // Layer L (0-based) is full attention iff (L + 1) % attn_interval == 0
    // (include/model_config.h:60-62 of the reference).
    bool is_attention_layer(int layer) const { return ((layer + 1) % attn_interval == 0); }
};

// load_model_config (src/config_loader.cpp:59-108): reads config.json, preferring its
// text_config object; absent keys keep their defaults. Returns false if the file cannot
// be read (cfg keeps the defaults).
bool load_model_config(const std::string& config_json_path, ModelConfig& cfg);

enum class Precision { FP32 = 4, FP16 = 2, INT8 = 1, INT4_PACKED = 0 };
