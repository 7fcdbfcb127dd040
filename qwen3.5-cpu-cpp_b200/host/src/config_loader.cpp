// load_model_config: same contract as the reference's src/config_loader.cpp:59-108 --
// config.json's text_config object is preferred (flat configs also work), keys that are
// absent keep their defaults, the GDN aliases follow the value side, and the layer split
// is derived from full_attention_interval. Keys are looked up in text_config and, when
// not found there, in its nested objects (rope_parameters carries rope_theta and
// partial_rotary_factor in current Qwen3.5 configs).
#include <fstream>
#include <iostream>
#include <iterator>
#include <string>

#include "json_lite.h"
#include "model_config.h"

using qwh::JValue;

static const JValue* key(const JValue& tc, const char* k) {
    if (const JValue* v = tc.get(k)) return v;
    return tc.find_deep(k);
}
static void set_int(const JValue& tc, const char* k, int& dst) {
    const JValue* v = key(tc, k);
    if (v && v->kind == JValue::NUM) dst = (int)(v->num + (v->num >= 0 ? 0.5 : -0.5));
}

bool load_model_config(const std::string& path, ModelConfig& cfg) {
    std::ifstream f(path, std::ios::binary);
    if (!f.is_open()) {
        std::cerr << "[config] cannot open " << path << " -- using built-in defaults\n";
        return false;
    }
    std::string all((std::istreambuf_iterator<char>(f)), std::istreambuf_iterator<char>());
    JValue root;
    std::string err;
    if (!qwh::parse_json(all.data(), all.size(), root, &err)) {
        std::cerr << "[config] " << path << ": " << err << " -- using built-in defaults\n";
        return false;
    }
    const JValue* tcp = root.get("text_config");
    const JValue& tc = (tcp && tcp->kind == JValue::OBJ) ? *tcp : root;

    set_int(tc, "hidden_size", cfg.hidden_size);
    set_int(tc, "num_hidden_layers", cfg.n_layers_total);
    set_int(tc, "full_attention_interval", cfg.attn_interval);
    set_int(tc, "num_attention_heads", cfg.attn_q_heads);
    set_int(tc, "num_key_value_heads", cfg.attn_kv_heads);
    set_int(tc, "head_dim", cfg.attn_head_dim);
    set_int(tc, "linear_num_key_heads", cfg.gdn_k_heads);
    set_int(tc, "linear_num_value_heads", cfg.gdn_v_heads);
    set_int(tc, "linear_key_head_dim", cfg.gdn_k_head_dim);
    set_int(tc, "linear_value_head_dim", cfg.gdn_v_head_dim);
    set_int(tc, "linear_conv_kernel_dim", cfg.gdn_conv_kernel);
    set_int(tc, "intermediate_size", cfg.ffn_intermediate);
    set_int(tc, "vocab_size", cfg.vocab_size);
    set_int(tc, "max_position_embeddings", cfg.native_max_context);
    cfg.gdn_n_heads = cfg.gdn_v_heads;
    cfg.gdn_head_dim = cfg.gdn_v_head_dim;
    if (cfg.attn_interval > 0) {
        cfg.n_layers_attn = cfg.n_layers_total / cfg.attn_interval;
        cfg.n_layers_gdn = cfg.n_layers_total - cfg.n_layers_attn;
    }
    if (const JValue* v = key(tc, "rms_norm_eps"); v && v->kind == JValue::NUM) cfg.rms_norm_eps = (float)v->num;
    if (const JValue* v = key(tc, "rope_theta"); v && v->kind == JValue::NUM) cfg.rope_theta = v->num;
    if (const JValue* v = key(tc, "partial_rotary_factor"); v && v->kind == JValue::NUM)
        cfg.partial_rotary_factor = (float)v->num;
    if (const JValue* v = key(tc, "tie_word_embeddings"); v && v->kind == JValue::BOOL) cfg.tie_word_embeddings = v->b;
    cfg.n_params = (int64_t)cfg.vocab_size * cfg.hidden_size +
                   (int64_t)cfg.n_layers_total * 12 * cfg.hidden_size * cfg.hidden_size;
    std::cout << "[config] " << path << ": hidden=" << cfg.hidden_size << " layers=" << cfg.n_layers_total << " ("
              << cfg.n_layers_gdn << " gdn / " << cfg.n_layers_attn << " attn) ffn=" << cfg.ffn_intermediate
              << " vocab=" << cfg.vocab_size << " tie=" << cfg.tie_word_embeddings << "\n";
    return true;
}
