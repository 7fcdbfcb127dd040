// The memory equation (include/memory_budget.h:6-62 of the reference): bytes per arena
// for a model and a context length, and its inverse (max context under a byte ceiling).
// On the GPU these size the device arenas of libqwen_cuda.
#pragma once
#include <cstddef>
#include <cstdint>
#include "model_config.h"

struct MemoryBudget {
    size_t weight_bytes = 0;
    size_t gdn_state_bytes = 0;
    size_t gdn_conv_bytes = 0;
    size_t kv_cache_bytes = 0;
    size_t activation_bytes = 0;
    size_t vision_scratch_bytes = 0;
    size_t total() const {
        return weight_bytes + gdn_state_bytes + gdn_conv_bytes + kv_cache_bytes + activation_bytes +
               vision_scratch_bytes;
    }
};

inline size_t gdn_conv_state_bytes(const ModelConfig& cfg) {
    size_t key_dim = (size_t)cfg.gdn_k_heads * cfg.gdn_k_head_dim;
    size_t value_dim = (size_t)cfg.gdn_v_heads * cfg.gdn_v_head_dim;
    return (size_t)cfg.n_layers_gdn * (key_dim * 2 + value_dim) * (cfg.gdn_conv_kernel - 1) * sizeof(float);
}

MemoryBudget compute_budget(const ModelConfig& cfg, int bytes_per_weight, int max_context,
                            int kv_bytes_per_elem, int max_vision_tiles = 4, int vit_dim = 1024);

int64_t solve_max_context(const ModelConfig& cfg, size_t ram_budget_bytes, size_t weight_bytes,
                          size_t gdn_state_bytes, size_t activation_bytes, size_t vision_scratch_bytes,
                          size_t safety_margin_bytes, int kv_bytes_per_elem);

size_t estimate_activation_scratch(const ModelConfig& cfg);
size_t estimate_vision_scratch(int max_tiles, int vit_dim, int patches_per_tile = 256);
