// The memory equation: compute_budget / solve_max_context / the scratch estimators with
// the reference's formulas (src/memory_budget.cpp:4-81), evaluated by the C ABI so that
// C++ and FFI callers get identical numbers.
#include "memory_budget.h"

#include <algorithm>

#include "capi_bridge.h"
#include "qwen_cuda.h"

size_t estimate_activation_scratch(const ModelConfig& cfg) {
    size_t ffn = (size_t)cfg.ffn_intermediate * sizeof(float) * 2;
    size_t attn = (size_t)(cfg.attn_q_heads * cfg.attn_head_dim + 2 * cfg.attn_kv_heads * cfg.attn_head_dim) * sizeof(float);
    size_t gdn = (size_t)(3 * cfg.gdn_n_heads * cfg.gdn_head_dim) * sizeof(float);
    return std::max({ffn, attn, gdn});
}

size_t estimate_vision_scratch(int max_tiles, int vit_dim, int patches_per_tile) {
    size_t patch = (size_t)max_tiles * patches_per_tile * vit_dim * sizeof(float);
    size_t work = (size_t)patches_per_tile * vit_dim * sizeof(float) * 2;
    return patch + work;
}

MemoryBudget compute_budget(const ModelConfig& cfg, int bpw, int max_context, int kvb, int max_vision_tiles,
                            int vit_dim) {
    qwc_config c;
    qwh::to_c(cfg, c);
    qwc_budget b{};
    qwc_compute_budget(&c, bpw, max_context, kvb, max_vision_tiles, vit_dim, &b);
    MemoryBudget m = qwh::from_c(b);
    m.activation_bytes = estimate_activation_scratch(cfg);
    return m;
}

int64_t solve_max_context(const ModelConfig& cfg, size_t ram, size_t wb, size_t gb, size_t ab, size_t vb,
                          size_t margin, int kvb) {
    qwc_config c;
    qwh::to_c(cfg, c);
    return qwc_solve_max_context(&c, ram, wb, gb, ab, vb, margin, kvb);
}
