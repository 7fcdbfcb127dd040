// Conversions between the C ABI structs and the C++ API types.
#pragma once
#include "memory_budget.h"
#include "model_config.h"
#include "qwen_cuda.h"
#include "safetensors_loader.h"

#include <string>
#include <vector>

namespace qwh {

inline void to_c(const ModelConfig& m, qwc_config& c) {
    c.hidden_size = m.hidden_size;
    c.n_layers_total = m.n_layers_total;
    c.n_layers_gdn = m.n_layers_gdn;
    c.n_layers_attn = m.n_layers_attn;
    c.gdn_k_heads = m.gdn_k_heads;
    c.gdn_v_heads = m.gdn_v_heads;
    c.gdn_k_head_dim = m.gdn_k_head_dim;
    c.gdn_v_head_dim = m.gdn_v_head_dim;
    c.gdn_conv_kernel = m.gdn_conv_kernel;
    c.attn_q_heads = m.attn_q_heads;
    c.attn_kv_heads = m.attn_kv_heads;
    c.attn_head_dim = m.attn_head_dim;
    c.ffn_intermediate = m.ffn_intermediate;
    c.vocab_size = m.vocab_size;
    c.native_max_context = m.native_max_context;
    c.attn_interval = m.attn_interval;
    c.tie_word_embeddings = m.tie_word_embeddings ? 1 : 0;
    c.rms_norm_eps = m.rms_norm_eps;
    c.partial_rotary_factor = m.partial_rotary_factor;
    c.rope_theta = m.rope_theta;
    c.n_params = m.n_params;
}

inline void from_c(const qwc_config& c, ModelConfig& m) {
    m.hidden_size = c.hidden_size;
    m.n_layers_total = c.n_layers_total;
    m.n_layers_gdn = c.n_layers_gdn;
    m.n_layers_attn = c.n_layers_attn;
    m.gdn_k_heads = c.gdn_k_heads;
    m.gdn_v_heads = c.gdn_v_heads;
    m.gdn_k_head_dim = c.gdn_k_head_dim;
    m.gdn_v_head_dim = c.gdn_v_head_dim;
    m.gdn_conv_kernel = c.gdn_conv_kernel;
    m.gdn_n_heads = c.gdn_v_heads;
    m.gdn_head_dim = c.gdn_v_head_dim;
    m.attn_q_heads = c.attn_q_heads;
    m.attn_kv_heads = c.attn_kv_heads;
    m.attn_head_dim = c.attn_head_dim;
    m.ffn_intermediate = c.ffn_intermediate;
    m.vocab_size = c.vocab_size;
    m.native_max_context = c.native_max_context;
    m.attn_interval = c.attn_interval;
    m.tie_word_embeddings = c.tie_word_embeddings != 0;
    m.rms_norm_eps = c.rms_norm_eps;
    m.partial_rotary_factor = c.partial_rotary_factor;
    m.rope_theta = c.rope_theta;
    m.n_params = c.n_params;
}

inline MemoryBudget from_c(const qwc_budget& b) {
    MemoryBudget m;
    m.weight_bytes = b.weight_bytes;
    m.gdn_state_bytes = b.gdn_state_bytes;
    m.gdn_conv_bytes = b.gdn_conv_bytes;
    m.kv_cache_bytes = b.kv_cache_bytes;
    m.activation_bytes = b.activation_bytes;
    m.vision_scratch_bytes = b.vision_scratch_bytes;
    return m;
}

// The checkpoint's tensors as a qwc_tensor table (names kept alive in `names`).
inline void tensor_table(const SafeTensors& st, std::vector<std::string>& names, std::vector<qwc_tensor>& out) {
    names.clear();
    out.clear();
    names.reserve(st.entries().size());
    for (const auto& kv : st.entries()) names.push_back(kv.first);
    for (const auto& n : names) {
        const SafeTensors::Entry* e = st.find(n);
        WeightView v = st.view(n);
        if (!e || !v.ok()) continue;
        qwc_tensor t{};
        t.name = n.c_str();
        t.dtype = v.bf16 ? QWC_DTYPE_BF16 : QWC_DTYPE_F32;
        t.ndim = (int)std::min<size_t>(e->shape.size(), 4);
        for (int i = 0; i < t.ndim; ++i) t.shape[i] = e->shape[i];
        if (e->shape.size() > 4) {  // fold trailing dims
            for (size_t i = 4; i < e->shape.size(); ++i) t.shape[3] *= e->shape[i];
        }
        t.data = v.bf16 ? (const void*)v.bf16 : (const void*)v.f32;
        out.push_back(t);
    }
}

}  // namespace qwh
